// C ABI of the fused preparation kernels (prep_impl.cuh).
#include "prep_impl.cuh"

namespace convrot {

extern template int launch_t<__nv_bfloat16, kModeI8>(const void*, int64_t, int64_t, int, void*, float*, cudaStream_t);
extern template int launch_t<__nv_bfloat16, kModePacked>(const void*, int64_t, int64_t, int, void*, float*, cudaStream_t);
extern template int launch_t<__nv_bfloat16, kModeRotate>(const void*, int64_t, int64_t, int, void*, float*, cudaStream_t);
extern template int launch_t<__half, kModeI8>(const void*, int64_t, int64_t, int, void*, float*, cudaStream_t);
extern template int launch_t<__half, kModePacked>(const void*, int64_t, int64_t, int, void*, float*, cudaStream_t);
extern template int launch_t<__half, kModeRotate>(const void*, int64_t, int64_t, int, void*, float*, cudaStream_t);
extern template int launch_t<float, kModeI8>(const void*, int64_t, int64_t, int, void*, float*, cudaStream_t);
extern template int launch_t<float, kModePacked>(const void*, int64_t, int64_t, int, void*, float*, cudaStream_t);
extern template int launch_t<float, kModeRotate>(const void*, int64_t, int64_t, int, void*, float*, cudaStream_t);

template <int MODE>
static int prep_entry(const void* x, int dtype, int64_t rows, int64_t K, int G, void* out, float* scales,
                      void* stream) {
  CONVROT_REQUIRE(valid_dtype(dtype), CONVROT_ERR_INVALID, "unknown dtype code %d", dtype);
  CONVROT_REQUIRE(rows >= 0 && K > 0, CONVROT_ERR_INVALID, "invalid shape (%lld, %lld)", static_cast<long long>(rows),
                  static_cast<long long>(K));
  CONVROT_REQUIRE(G >= 1, CONVROT_ERR_INVALID, "group size must be positive, got %d", G);
  if (G > 1) {
    int v = G;
    while (v > 1 && v % 4 == 0) v /= 4;
    CONVROT_REQUIRE(v == 1, CONVROT_ERR_INVALID, "Regular Hadamard size must be a power of 4, got %d", G);
  }
  CONVROT_REQUIRE(K % G == 0, CONVROT_ERR_INVALID, "features %lld not divisible by ConvRot group size %d",
                  static_cast<long long>(K), G);
  CONVROT_REQUIRE(K % 16 == 0, CONVROT_ERR_UNSUPPORTED, "features %lld must be a multiple of 16",
                  static_cast<long long>(K));
  CONVROT_REQUIRE(rows == 0 || (x && out), CONVROT_ERR_INVALID, "null pointer");
  CONVROT_REQUIRE(MODE == kModeRotate || rows == 0 || scales, CONVROT_ERR_INVALID, "null scales pointer");
  CONVROT_REQUIRE(aligned_to(x, 16) && aligned_to(out, 16), CONVROT_ERR_INVALID,
                  "x and the output must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case CONVROT_BF16: return launch_t<__nv_bfloat16, MODE>(x, rows, K, G, out, scales, s);
    case CONVROT_F16: return launch_t<__half, MODE>(x, rows, K, G, out, scales, s);
    default: return launch_t<float, MODE>(x, rows, K, G, out, scales, s);
  }
}

}  // namespace convrot

extern "C" {

int convrot_prepare_i8(const void* x, int dtype, int64_t rows, int64_t features, int group_size, int8_t* q_i8,
                       float* scales, void* stream) {
  return convrot::prep_entry<convrot::kModeI8>(x, dtype, rows, features, group_size, q_i8, scales, stream);
}

int convrot_prepare_packed(const void* x, int dtype, int64_t rows, int64_t features, int group_size,
                           uint8_t* q_packed, float* scales, void* stream) {
  return convrot::prep_entry<convrot::kModePacked>(x, dtype, rows, features, group_size, q_packed, scales, stream);
}

int convrot_rotate(const void* x, int dtype, int64_t rows, int64_t features, int group_size, void* out,
                   void* stream) {
  if (group_size == 1) {
    convrot::set_error("group size 1 is not a rotation");
    return CONVROT_ERR_INVALID;
  }
  return convrot::prep_entry<convrot::kModeRotate>(x, dtype, rows, features, group_size, out, nullptr, stream);
}

}  // extern "C"
