// DiT attention glue for the benchmark model of flux_dit.py (not part of the
// ConvRot path): the per-head RMSNorm of q and k, the rotary embedding, and
// the move of q, k, v from the projection's (batch, tokens, 3, heads, 128)
// rows into the (batch, heads, tokens, 128) layout that attention reads, at
// a token offset -- so the text and image streams of a double block land
// side by side without a separate concatenation.  One warp per (batch,
// token, head): each lane holds 4 of the 128 values of q, k and v.
//
// Numerics follow the torch ops of flux_dit.py: RMSNorm in float32,
// y = bf16(x * rsqrt(mean(x^2) + eps) * scale); rotation of the pairs
// (y[2j], y[2j+1]) by (cos, sin) in float32, rounded once to bf16.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace {

constexpr int kDim = 128;

__device__ __forceinline__ float2 ld_bf16x2(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}

__device__ __forceinline__ void norm_rope(const __nv_bfloat16* src, const __nv_bfloat16* scale, const float4 rot,
                                          float eps, int lane, __nv_bfloat16* dst) {
  // lane holds elements 4 lane .. 4 lane + 3: pairs 2 lane and 2 lane + 1
  const uint2 raw = *reinterpret_cast<const uint2*>(src + 4 * lane);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
  float ss = a.x * a.x + a.y * a.y + b.x * b.x + b.y * b.y;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
  const float rstd = rsqrtf(ss / kDim + eps);
  const float2 sa = ld_bf16x2(scale + 4 * lane), sb = ld_bf16x2(scale + 4 * lane + 2);
  // RMSNorm output, rounded to bf16 as the norm's own result
  const float2 ya = __bfloat1622float2(__floats2bfloat162_rn(a.x * rstd * sa.x, a.y * rstd * sa.y));
  const float2 yb = __bfloat1622float2(__floats2bfloat162_rn(b.x * rstd * sb.x, b.y * rstd * sb.y));
  // (x0 + i x1) (c + i s)
  const __nv_bfloat162 oa = __floats2bfloat162_rn(ya.x * rot.x - ya.y * rot.y, ya.x * rot.y + ya.y * rot.x);
  const __nv_bfloat162 ob = __floats2bfloat162_rn(yb.x * rot.z - yb.y * rot.w, yb.x * rot.w + yb.y * rot.z);
  uint2 out;
  out.x = *reinterpret_cast<const uint32_t*>(&oa);
  out.y = *reinterpret_cast<const uint32_t*>(&ob);
  *reinterpret_cast<uint2*>(dst + 4 * lane) = out;
}

// qkv row (b, l) at qkv + (b * tokens + l) * row_stride; q, k, v of head h at
// offsets h * 128, (heads + h) * 128, (2 heads + h) * 128 of the row.
// rot: (batch, tokens_total, 64) complex64 (cos, sin pairs).  Outputs
// (batch, heads, tokens_total, 128) at token l_off + l.
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(
    const __nv_bfloat16* __restrict__ qkv, int64_t row_stride, int batch, int tokens, int heads,
    const __nv_bfloat16* __restrict__ q_scale, const __nv_bfloat16* __restrict__ k_scale, float eps,
    const float2* __restrict__ rot, int l_off, int tokens_total, __nv_bfloat16* __restrict__ q_out,
    __nv_bfloat16* __restrict__ k_out, __nv_bfloat16* __restrict__ v_out) {
  const int lane = threadIdx.x & 31;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t total = static_cast<int64_t>(batch) * tokens * heads;
  if (item >= total) return;
  const int h = static_cast<int>(item % heads);
  const int64_t bl = item / heads;
  const int l = static_cast<int>(bl % tokens);
  const int b = static_cast<int>(bl / tokens);
  const __nv_bfloat16* row = qkv + bl * row_stride;
  const int lt = l_off + l;
  const float4 r = *reinterpret_cast<const float4*>(rot + (static_cast<int64_t>(b) * tokens_total + lt) * (kDim / 2) +
                                                    2 * lane);
  const int64_t dst = ((static_cast<int64_t>(b) * heads + h) * tokens_total + lt) * kDim;
  norm_rope(row + h * kDim, q_scale, r, eps, lane, q_out + dst);
  norm_rope(row + (heads + h) * kDim, k_scale, r, eps, lane, k_out + dst);
  *reinterpret_cast<uint2*>(v_out + dst + 4 * lane) =
      *reinterpret_cast<const uint2*>(row + (2 * heads + h) * kDim + 4 * lane);
}

// tanh-approximated GELU in float32 with every rounding spelled out, the
// form the fused W4A4 prep of the same concatenation uses
// (convrot_gelu_concat_prepare_i8), so both give the same bits
__device__ __forceinline__ float gelu_tanh(float x) {
  // tanh(u) = 1 - 2 / (1 + e^2u) from the exponential and approximate-division
  // intrinsics: a fraction of tanhf's instructions, and it saturates to +-1
  // exactly as tanhf does
  const float x3 = __fmul_rn(__fmul_rn(x, x), x);
  const float u = __fmul_rn(0.7978845608028654f, __fadd_rn(x, __fmul_rn(0.044715f, x3)));
  const float t = __fsub_rn(1.0f, __fdividef(2.0f, __fadd_rn(1.0f, __expf(__fmul_rn(2.0f, u)))));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
}

// out row r = [a[r, 0:da], gelu_tanh(m[r, 0:dm])]: the input of a single
// block's output projection, with the MLP half's activation applied on the
// way (float32 math, one bf16 rounding, as torch's tanh-approximated GELU).
// 8 elements (16 bytes) per thread; da and dm multiples of 8.
__global__ void __launch_bounds__(256) gelu_concat_kernel(const __nv_bfloat16* __restrict__ a, int64_t a_stride,
                                                         const __nv_bfloat16* __restrict__ m, int64_t m_stride,
                                                         int64_t rows, int da, int dm,
                                                         __nv_bfloat16* __restrict__ out) {
  const int vecs = (da + dm) / 8;
  const int64_t total = rows * vecs;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / vecs;
    const int c = static_cast<int>(i % vecs) * 8;
    uint4 v;
    if (c < da) {
      v = *reinterpret_cast<const uint4*>(a + r * a_stride + c);
    } else {
      const uint4 x = *reinterpret_cast<const uint4*>(m + r * m_stride + (c - da));
      const uint32_t xw[4] = {x.x, x.y, x.z, x.w};
      uint32_t yw[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&xw[j]));
        const __nv_bfloat162 y = __floats2bfloat162_rn(gelu_tanh(f.x), gelu_tanh(f.y));
        yw[j] = *reinterpret_cast<const uint32_t*>(&y);
      }
      v = make_uint4(yw[0], yw[1], yw[2], yw[3]);
    }
    *reinterpret_cast<uint4*>(out + r * (da + dm) + c) = v;
  }
}

}  // namespace

extern "C" int flux_gelu_concat(const void* a, int64_t a_stride, const void* m, int64_t m_stride, int64_t rows,
                                int64_t da, int64_t dm, void* out, void* stream) {
  if (rows == 0) return 0;
  if (rows < 0 || da % 8 || dm % 8 || a_stride % 8 || m_stride % 8) return -1;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(out)) % 16)
    return -1;
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  gelu_concat_kernel<<<sms * 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(a), a_stride, static_cast<const __nv_bfloat16*>(m), m_stride, rows,
      static_cast<int>(da), static_cast<int>(dm), static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

extern "C" int flux_qk_norm_rope(const void* qkv, int64_t row_stride, int64_t batch, int64_t tokens, int64_t heads,
                                 const void* q_scale, const void* k_scale, float eps, const void* rot, int64_t l_off,
                                 int64_t tokens_total, void* q_out, void* k_out, void* v_out, void* stream) {
  if (batch <= 0 || tokens <= 0 || heads <= 0) return batch == 0 || tokens == 0 ? 0 : -1;
  if (row_stride % 4 || l_off < 0 || l_off + tokens > tokens_total) return -1;
  const uintptr_t align = reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(q_out) |
                          reinterpret_cast<uintptr_t>(k_out) | reinterpret_cast<uintptr_t>(v_out) |
                          reinterpret_cast<uintptr_t>(q_scale) | reinterpret_cast<uintptr_t>(k_scale);
  if (align % 8 || reinterpret_cast<uintptr_t>(rot) % 16) return -1;
  const int64_t items = batch * tokens * heads;
  const int warps = 8;
  const int64_t blocks = (items + warps - 1) / warps;
  qk_norm_rope_kernel<<<static_cast<unsigned>(blocks), warps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(qkv), row_stride, static_cast<int>(batch), static_cast<int>(tokens),
      static_cast<int>(heads), static_cast<const __nv_bfloat16*>(q_scale), static_cast<const __nv_bfloat16*>(k_scale),
      eps, static_cast<const float2*>(rot), static_cast<int>(l_off), static_cast<int>(tokens_total),
      static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(k_out), static_cast<__nv_bfloat16*>(v_out));
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
