// Instantiation of the fused preparation kernels for float inputs.
#include "prep_impl.cuh"

namespace convrot {
CONVROT_PREP_INSTANTIATE(float)
}  // namespace convrot
