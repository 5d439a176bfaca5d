// Instantiation of the fused preparation kernels for __nv_bfloat16 inputs.
#include "prep_impl.cuh"

namespace convrot {
CONVROT_PREP_INSTANTIATE(__nv_bfloat16)
}  // namespace convrot
