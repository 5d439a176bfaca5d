// Instantiation of the fused preparation kernels for __half inputs.
#include "prep_impl.cuh"

namespace convrot {
CONVROT_PREP_INSTANTIATE(__half)
}  // namespace convrot
