// Modulated LayerNorm fused into the ConvRot activation preparation.
//
// In a FLUX-style DiT block the input of the qkv, first-MLP and single-block
// projections is xm = (1 + scale) * LayerNorm(x) + shift, with shift and
// scale one vector per sample.  Computed as separate ops, that costs three
// HBM round trips of the activation before the prep kernel reads xm again.
// This kernel reads each row of x once and writes the int8 codes and the row
// scale of prepare(xm): the reference names the preparation passes as the
// remaining cost of its path (docs/design.md:54-64); the norm and modulation
// come from the FLUX block that feeds the linear.
//
// Per row (one CTA):
//   1. mean and variance of x in float32, two passes over the row held in
//      registers (sum, then sum of squared deviations), each a warp-shuffle
//      tree plus one exchange through shared memory;
//   2. y = bf16((x - mean) * rsqrt(var + eps)), t = bf16(1 + scale[c]) and
//      xm = bf16(fma(y, t, shift[c])) -- the rounding points of
//      torch.layer_norm (bf16 out) and torch.addcmul(shift, y, 1 + scale);
//   3. the radix-4 rotation, row absmax, scale and codes of prep_kernel
//      (prep_impl.cuh), bit for bit what prepare_i8(xm) gives for the same xm.
// Only step 1's summation order is this kernel's own: a last-bit difference in
// the mean or rstd can move a y or xm across a bf16 rounding boundary, and a
// code then by one.
//
// The same kernel serves a second producer: the input of a FLUX single
// block's output projection, cat(a, gelu_tanh(m)) -- the attention output
// and the MLP half of the block's fused input projection, a column slice of a
// wider tensor.  Then each row is read from its two sources, the GELU is
// applied on load (float32, explicit roundings, one bf16 rounding), and steps
// 1-2 are skipped: the codes are bit for bit prepare_i8 of the concatenation.
#include "prep_impl.cuh"

namespace convrot {
namespace {

using bf16 = __nv_bfloat16;
using bf162 = __nv_bfloat162;

constexpr int kSrcModNorm = 0, kSrcGeluCat = 1;

struct ModNorm {
  const bf16* shift;   // (samples, features) with row stride mod_stride
  const bf16* scale;
  int64_t rows_per_mod;  // rows (tokens) per sample
  int64_t mod_stride;    // elements between consecutive samples' vectors
  float eps;
  // kSrcGeluCat: row r = [a[r, 0:da], gelu(m[r, 0:K - da])], a = x
  const bf16* m;
  int64_t a_stride, m_stride;
  int da;
};

// tanh-approximated GELU in float32 with every rounding spelled out (so that
// no compiler contraction changes it): 0.5 x (1 + tanh(c (x + 0.044715 x^3)))
__device__ __forceinline__ float gelu_tanh(float x) {
  // tanh(u) = 1 - 2 / (1 + e^2u) from the exponential and approximate-division
  // intrinsics: a fraction of tanhf's instructions, and it saturates to +-1
  // exactly as tanhf does
  const float x3 = __fmul_rn(__fmul_rn(x, x), x);
  const float u = __fmul_rn(0.7978845608028654f, __fadd_rn(x, __fmul_rn(0.044715f, x3)));
  const float t = __fsub_rn(1.0f, __fdividef(2.0f, __fadd_rn(1.0f, __expf(__fmul_rn(2.0f, u)))));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
}

__device__ __forceinline__ void gelu16(Raw16<bf16>& r) {
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    uint32_t* w = reinterpret_cast<uint32_t*>(&r.v[q]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const bf162*>(&w[i]));
      const bf162 g = __floats2bfloat162_rn(gelu_tanh(f.x), gelu_tanh(f.y));
      w[i] = *reinterpret_cast<const uint32_t*>(&g);
    }
  }
}

// 16 consecutive elements of a row starting at column c (c and da multiples
// of 16, so a unit never straddles the two sources)
template <int SRC>
__device__ __forceinline__ void load_unit(Raw16<bf16>& r, const bf16* x, const ModNorm& mn, int64_t row, int K,
                                          int c) {
  if constexpr (SRC == kSrcModNorm) {
    load16(r, x + row * static_cast<int64_t>(K) + c);
  } else if (c < mn.da) {
    load16(r, x + row * mn.a_stride + c);
  } else {
    load16(r, mn.m + row * mn.m_stride + (c - mn.da));
    gelu16(r);
  }
}

__device__ __forceinline__ float block_sum(float v, float* red, int tid, int nthr) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  __syncthreads();  // red may still be read by the previous reduction
  if ((tid & 31) == 0) red[tid >> 5] = v;
  __syncthreads();
  float s = (tid & 31) < (nthr >> 5) ? red[tid & 31] : 0.0f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
  return s;
}

__device__ __forceinline__ float block_max(float v, float* red, int tid, int nthr) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  __syncthreads();
  if ((tid & 31) == 0) red[tid >> 5] = v;
  __syncthreads();
  float m = (tid & 31) < (nthr >> 5) ? red[tid & 31] : 0.0f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  return m;
}

// xm of 16 consecutive elements starting at column c, in place in r.
__device__ __forceinline__ void modulate16(Raw16<bf16>& r, int c, float mean, float rstd, const bf16* shift,
                                           const bf16* scale) {
  const uint4* sp = reinterpret_cast<const uint4*>(shift + c);
  const uint4* cp = reinterpret_cast<const uint4*>(scale + c);
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const uint4 sh = __ldg(sp + q), sc = __ldg(cp + q);
    const uint32_t shw[4] = {sh.x, sh.y, sh.z, sh.w}, scw[4] = {sc.x, sc.y, sc.z, sc.w};
    uint32_t* xw = reinterpret_cast<uint32_t*>(&r.v[q]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 xf = __bfloat1622float2(*reinterpret_cast<const bf162*>(&xw[i]));
      const float2 sf = __bfloat1622float2(*reinterpret_cast<const bf162*>(&shw[i]));
      const float2 cf = __bfloat1622float2(*reinterpret_cast<const bf162*>(&scw[i]));
      // torch.layer_norm in bf16: (x - mean) * rstd in float32, one rounding
      const float2 y = __bfloat1622float2(__floats2bfloat162_rn((xf.x - mean) * rstd, (xf.y - mean) * rstd));
      // 1 + scale, rounded to bf16 as its own op; then addcmul's one rounding
      const float2 t = __bfloat1622float2(__floats2bfloat162_rn(1.0f + cf.x, 1.0f + cf.y));
      const bf162 out = __floats2bfloat162_rn(__fmaf_rn(y.x, t.x, sf.x), __fmaf_rn(y.y, t.y, sf.y));
      xw[i] = *reinterpret_cast<const uint32_t*>(&out);
    }
  }
}

__device__ __forceinline__ float sum16(const Raw16<bf16>& r) {
  float s = 0.0f;
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const uint32_t w[4] = {r.v[q].x, r.v[q].y, r.v[q].z, r.v[q].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const bf162*>(&w[i]));
      s += f.x + f.y;
    }
  }
  return s;
}

__device__ __forceinline__ float sumsq16(const Raw16<bf16>& r, float mean) {
  float s = 0.0f;
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const uint32_t w[4] = {r.v[q].x, r.v[q].y, r.v[q].z, r.v[q].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const bf162*>(&w[i]));
      const float dx = f.x - mean, dy = f.y - mean;
      s = __fmaf_rn(dx, dx, s);
      s = __fmaf_rn(dy, dy, s);
    }
  }
  return s;
}

// One CTA per row; the rotation and quantization below follow prep_kernel's
// unstaged bf16 path (fast quantizer, int8 codes) step for step.
template <int G, int UPT, int SRC>
__global__ void __launch_bounds__(256) modnorm_prep_kernel(const bf16* __restrict__ x, int64_t rows, int K, int half,
                                                             const ModNorm mn, int8_t* __restrict__ out,
                                                             float* __restrict__ scales) {
  using E = Elem<bf16>;
  using P = bf162;
  static_assert(G == 64 || G == 256, "modulated-norm prep covers groups 64 and 256");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  P* sm = reinterpret_cast<P*>(smem_raw);
  __shared__ float red[32];

  const int tid = threadIdx.x;
  const int nthr = blockDim.x;
  const int units = half >> 4;
  constexpr float kNorm = G == 64 ? 0.125f : 0.0625f;

  int s_unit[UPT], s_col[UPT];
#pragma unroll
  for (int j = 0; j < UPT; ++j) {
    const int t = tid + j * nthr;
    s_unit[j] = swz(t << 4);
    s_col[j] = G == 64 ? swz(64 * (t >> 2) + 4 * (t & 3)) : swz(256 * (t >> 4) + (t & 15));
  }
  grid_dependency_wait();  // x, shift and scale may come from the previous kernel of the stream
  grid_dependents_launch();

  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    Raw16<bf16> rlo[UPT], rhi[UPT];
#pragma unroll
    for (int j = 0; j < UPT; ++j) {
      const int u = tid + j * nthr;
      if (u < units) {
        const int p0 = u << 4;
        load_unit<SRC>(rlo[j], x, mn, row, K, p0);
        if (p0 + half < K) load_unit<SRC>(rhi[j], x, mn, row, K, p0 + half);
        else zero16(rhi[j]);
      }
    }
    if constexpr (SRC == kSrcModNorm) {
    const int64_t sample = row / mn.rows_per_mod;
    const bf16* shift = mn.shift + sample * mn.mod_stride;
    const bf16* scale = mn.scale + sample * mn.mod_stride;
    // 1. row statistics (float32, two passes over the registers)
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < UPT; ++j)
      if (tid + j * nthr < units) s += sum16(rlo[j]) + sum16(rhi[j]);  // zero-filled tails add 0
    const float mean = block_sum(s, red, tid, nthr) / static_cast<float>(K);
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < UPT; ++j) {
      const int u = tid + j * nthr;
      if (u < units) {
        ss += sumsq16(rlo[j], mean);
        if ((u << 4) + half < K) ss += sumsq16(rhi[j], mean);
      }
    }
    const float var = block_sum(ss, red, tid, nthr) / static_cast<float>(K);
    const float rstd = rsqrtf(var + mn.eps);
    // 2. normalize and modulate in place
#pragma unroll
    for (int j = 0; j < UPT; ++j) {
      const int u = tid + j * nthr;
      if (u < units) {
        const int p0 = u << 4;
        modulate16(rlo[j], p0, mean, rstd, shift, scale);
        if (p0 + half < K) modulate16(rhi[j], p0 + half, mean, rstd, shift, scale);
      }
    }
    }  // kSrcModNorm
    // 3. rotate (strides 1 and 4 in registers, 16 and 64 over shared memory)
#pragma unroll
    for (int j = 0; j < UPT; ++j) {
      const int u = tid + j * nthr;
      if (u < units) {
        P v[16];
        interleave<E>(v, rlo[j], rhi[j]);
        stages_1_4<E, G, false>(v);
#pragma unroll
        for (int m = 0; m < 4; ++m) st_chunk(sm, s_unit[j] ^ swz(4 * m), v[4 * m], v[4 * m + 1], v[4 * m + 2], v[4 * m + 3]);
      }
    }
    __syncwarp();
    P amax2 = E::splat(0.0f);
#pragma unroll
    for (int j = 0; j < UPT; ++j) {
      const int t = tid + j * nthr;
      if (t >= units) continue;
      P w[16];
      if constexpr (G == 64) {
#pragma unroll
        for (int i = 0; i < 4; ++i) ld_chunk(sm, s_col[j] ^ swz(16 * i), w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
#pragma unroll
        for (int c = 0; c < 4; ++c) bfly4<E, false>(w[c], w[4 + c], w[8 + c], w[12 + c]);
        absmax_bf16x2(w, amax2);
#pragma unroll
        for (int i = 0; i < 4; ++i) st_chunk(sm, s_col[j] ^ swz(16 * i), w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = sm[s_col[j] ^ swz(16 * i)];
        stages_1_4<E, 16, false>(w);
        absmax_bf16x2(w, amax2);
#pragma unroll
        for (int i = 0; i < 16; ++i) sm[s_col[j] ^ swz(16 * i)] = w[i];
      }
    }
    // row absmax, scale (core.py:149-158), codes
    float amax = fmaxf(__low2float(amax2), __high2float(amax2)) * kNorm;
    const float rmax = block_max(amax, red, tid, nthr);
    const float floor_v = __bfloat162float(__float2bfloat16_rn(1.0e-10f));
    const float maximum = __bfloat162float(__float2bfloat16_rn(fmaxf(rmax, floor_v)));
    const float sc = __bfloat162float(__float2bfloat16_rn(__fdiv_rn(maximum, 7.0f)));
    const float rscale = __fdiv_rn(1.0f, sc) * kNorm;
    if (tid == 0) scales[row] = sc;
#pragma unroll
    for (int j = 0; j < UPT; ++j) {
      const int u = tid + j * nthr;
      if (u >= units) continue;
      P w[16];
#pragma unroll
      for (int m = 0; m < 4; ++m) ld_chunk(sm, s_unit[j] ^ swz(4 * m), w[4 * m], w[4 * m + 1], w[4 * m + 2], w[4 * m + 3]);
      emit_unit_bf16<kModeI8>(out, row, K, half, u << 4, w, rscale);
    }
    if (row + gridDim.x < rows) __syncthreads();  // the pair-words are rewritten by the next row
  }
}

template <int G, int SRC>
int launch_modnorm(const bf16* x, int64_t rows, int K, int half, const ModNorm& mn, int8_t* out, float* scales,
                   cudaStream_t stream) {
  const int units = half / 16;
  int upt = 1;
  while (upt < 4 && (units + upt - 1) / upt > 256) upt *= 2;
  const int threads = ((units + upt - 1) / upt + 31) / 32 * 32;
  CONVROT_REQUIRE(threads <= 256, CONVROT_ERR_UNSUPPORTED, "features %d too large for the fused kernel", K);
  const size_t smem = static_cast<size_t>(half) * sizeof(bf162);
  CONVROT_REQUIRE(smem <= 227 * 1024, CONVROT_ERR_UNSUPPORTED, "features %d too large for the fused kernel", K);
  auto run = [&](auto kernel) -> int {
    CONVROT_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(rows < 2147483647LL ? rows : 2147483647LL), 1, 1);
    cfg.blockDim = dim3(static_cast<unsigned>(threads), 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CONVROT_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, x, rows, K, half, mn, out, scales));
    return check_launch("convrot fused-producer prep kernel");
  };
  switch (upt) {
    case 1: return run(modnorm_prep_kernel<G, 1, SRC>);
    case 2: return run(modnorm_prep_kernel<G, 2, SRC>);
    default: return run(modnorm_prep_kernel<G, 4, SRC>);
  }
}

}  // namespace
}  // namespace convrot

extern "C" {

int convrot_modnorm_prepare_i8(const void* x, int dtype, int64_t rows, int64_t features, int group_size,
                               const void* shift, const void* scale, int64_t rows_per_mod, int64_t mod_stride,
                               float eps, int8_t* q_i8, float* scales, void* stream) {
  using namespace convrot;
  CONVROT_REQUIRE(dtype == CONVROT_BF16, CONVROT_ERR_UNSUPPORTED,
                  "the modulated-norm prep takes bfloat16 activations (dtype %d)", dtype);
  CONVROT_REQUIRE(group_size == 64 || group_size == 256, CONVROT_ERR_UNSUPPORTED,
                  "the modulated-norm prep covers groups 64 and 256, got %d", group_size);
  CONVROT_REQUIRE(rows >= 0 && features > 0 && features % group_size == 0, CONVROT_ERR_INVALID,
                  "invalid shape (%lld, %lld) for group %d", static_cast<long long>(rows),
                  static_cast<long long>(features), group_size);
  CONVROT_REQUIRE(features <= (1 << 20), CONVROT_ERR_UNSUPPORTED, "features too large");
  CONVROT_REQUIRE(rows_per_mod > 0 && mod_stride >= features, CONVROT_ERR_INVALID,
                  "rows_per_mod must be positive and mod_stride >= features (got %lld, %lld)",
                  static_cast<long long>(rows_per_mod), static_cast<long long>(mod_stride));
  CONVROT_REQUIRE(mod_stride % 8 == 0, CONVROT_ERR_INVALID,
                  "mod_stride must be a multiple of 8 elements (16-byte vectors), got %lld",
                  static_cast<long long>(mod_stride));
  CONVROT_REQUIRE(eps >= 0.0f, CONVROT_ERR_INVALID, "eps must be non-negative");
  if (rows == 0) return CONVROT_OK;
  CONVROT_REQUIRE(x && shift && scale && q_i8 && scales, CONVROT_ERR_INVALID, "null pointer");
  CONVROT_REQUIRE(aligned_to(x, 16) && aligned_to(shift, 16) && aligned_to(scale, 16) && aligned_to(q_i8, 16),
                  CONVROT_ERR_INVALID, "x, shift, scale and the codes must be 16-byte aligned");
  const int64_t groups = features / group_size;
  const int64_t half = ((groups + 1) / 2) * group_size;
  CONVROT_REQUIRE(half % 16 == 0, CONVROT_ERR_UNSUPPORTED, "unsupported feature count %lld",
                  static_cast<long long>(features));
  ModNorm mn{static_cast<const __nv_bfloat16*>(shift), static_cast<const __nv_bfloat16*>(scale), rows_per_mod,
             mod_stride, eps, nullptr, 0, 0, 0};
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int k = static_cast<int>(features), h = static_cast<int>(half);
  if (group_size == 64) return launch_modnorm<64, kSrcModNorm>(xb, rows, k, h, mn, q_i8, scales, s);
  return launch_modnorm<256, kSrcModNorm>(xb, rows, k, h, mn, q_i8, scales, s);
}

int convrot_gelu_concat_prepare_i8(const void* a, int64_t a_stride, int64_t da, const void* m, int64_t m_stride,
                                   int64_t dm, int64_t rows, int group_size, int8_t* q_i8, float* scales,
                                   void* stream) {
  using namespace convrot;
  const int64_t features = da + dm;
  CONVROT_REQUIRE(group_size == 64 || group_size == 256, CONVROT_ERR_UNSUPPORTED,
                  "the GELU-concatenation prep covers groups 64 and 256, got %d", group_size);
  CONVROT_REQUIRE(rows >= 0 && da > 0 && dm > 0 && features % group_size == 0, CONVROT_ERR_INVALID,
                  "invalid shape: rows %lld, widths %lld + %lld for group %d", static_cast<long long>(rows),
                  static_cast<long long>(da), static_cast<long long>(dm), group_size);
  CONVROT_REQUIRE(da % 16 == 0, CONVROT_ERR_UNSUPPORTED, "the first part's width must be a multiple of 16, got %lld",
                  static_cast<long long>(da));
  CONVROT_REQUIRE(a_stride >= da && m_stride >= dm && a_stride % 8 == 0 && m_stride % 8 == 0, CONVROT_ERR_INVALID,
                  "row strides must cover the widths and be multiples of 8 elements (%lld, %lld)",
                  static_cast<long long>(a_stride), static_cast<long long>(m_stride));
  CONVROT_REQUIRE(features <= (1 << 20), CONVROT_ERR_UNSUPPORTED, "features too large");
  if (rows == 0) return CONVROT_OK;
  CONVROT_REQUIRE(a && m && q_i8 && scales, CONVROT_ERR_INVALID, "null pointer");
  CONVROT_REQUIRE(aligned_to(a, 16) && aligned_to(m, 16) && aligned_to(q_i8, 16), CONVROT_ERR_INVALID,
                  "a, m and the codes must be 16-byte aligned");
  const int64_t groups = features / group_size;
  const int64_t half = ((groups + 1) / 2) * group_size;
  CONVROT_REQUIRE(half % 16 == 0, CONVROT_ERR_UNSUPPORTED, "unsupported feature count %lld",
                  static_cast<long long>(features));
  ModNorm mn{nullptr, nullptr, 1, 0, 0.0f, static_cast<const __nv_bfloat16*>(m), a_stride, m_stride,
             static_cast<int>(da)};
  const auto* ab = static_cast<const __nv_bfloat16*>(a);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int k = static_cast<int>(features), h = static_cast<int>(half);
  if (group_size == 64) return launch_modnorm<64, kSrcGeluCat>(ab, rows, k, h, mn, q_i8, scales, s);
  return launch_modnorm<256, kSrcGeluCat>(ab, rows, k, h, mn, q_i8, scales, s);
}

}  // extern "C"
