// W4A4 GEMM for at most 8 activation rows on sm_100a: a weight-streaming
// kernel whose weights go from HBM straight into MMA fragments.
//
// With m <= 8 (the modulation linears of a DiT at m = batch, decode-style
// calls) the op does 2 m multiply-adds per packed weight nibble: ~16 integer
// ops per weight byte, far below any tensor-core roofline ridge, so the bound
// is reading the K * N / 2 packed weight bytes from HBM once.  A tile kernel
// stages weights through shared memory and TMEM, and each of its stages waits
// on the previous hand-off; at m <= 8 those waits, not bandwidth, set its
// time.  Here every thread loads its weight bytes with plain 8- or 16-byte
// global loads into registers, turns them into int8 MMA fragments with byte
// permutes, and issues register-operand MMAs
//
//   C[n, r] (int32) += W16[n, k] x A[r, k]^T,
//   mma.sync.m16n8k32.row.col.s32.s8.s8.s32,
//
// with 16 weight columns on the MMA's M side and the (up to 8) activation
// rows on its N side.  Each nibble is placed in the high half of its byte, so
// the fragment holds 16 w exactly and C holds 16 dot, exact in int32 (K * 49
// * 16 < 2^31 for K < 2.7 M); the epilogue shifts it back.
//
// Fragment construction.  The MMA only requires that the threads agree on
// which real column each fragment row is and which real k each fragment k
// index is, so both are chosen to match what a thread loads:
// * K x packed-N weights: thread (g = lane / 4, t = lane % 4) loads rows
//   k0 + 8t .. + 7, 16 columns each (8 bytes).  A 4 x 4 byte transpose of
//   four rows (8 byte permutes) gives words of 4 consecutive k for one byte
//   position, i.e. for a column pair; shift / mask split the pair.  MMA j of
//   an 8-column chunk takes columns 2j (fragment row g) and 2j + 1 (row
//   g + 8); fragment k index 4t + i is real k k0 + 8t + i, and 16 + 4t + i
//   is k0 + 8t + 4 + i, so the activation fragment is the 8 bytes of row g
//   at k0 + 8t, one load.
// * N x packed-K weights: a 32-bit word of a weight row is 8 consecutive k
//   of one column; the low nibbles (even k) and high nibbles (odd k) are the
//   two fragment k halves, and the activation bytes are permuted to match.
//
// K is split over the 8 warps of a CTA and over a cluster of up to 8 CTAs;
// partial sums meet in shared memory, then the cluster's rank-0 CTA adds its
// peers' over distributed shared memory (exact integer sums) and runs the
// reference epilogue out = T(fl(fl(float(dot) * xs[r]) * ws[n]) + bias[n])
// (core.py:932-936).  No loop waits on another CTA except the two cluster
// barriers, which every CTA reaches.
#include "common.cuh"

namespace convrot {
namespace gemv {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxRows = 8;      // activation rows (the MMA's N)
constexpr int kMaxCluster = 8;
constexpr int kCbKN = 128;       // columns per CTA, K x packed-N weights (8 groups x 16)
constexpr int kCbNK = 64;        // columns per CTA, N x packed-K weights (4 MMAs x 16)
constexpr uint32_t kHi = 0xF0F0F0F0u;

struct Params {
  const int8_t* act;
  const uint8_t* qweight;
  const float* xscales;
  const float* wscales;
  const float* bias;
  void* out;
  int M, N, K;
  int cluster;
};

__device__ __forceinline__ void mma_s8(int32_t (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t dsmem_ld(uint32_t cluster_addr) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(cluster_addr) : "memory");
  return v;
}

// [lo, hi) of `units` K units for (cluster rank, warp)
__device__ __forceinline__ void k_range(int units, int rank, int ranks, int warp, int& lo, int& hi) {
  const int c0 = static_cast<int>(static_cast<int64_t>(units) * rank / ranks);
  const int c1 = static_cast<int>(static_cast<int64_t>(units) * (rank + 1) / ranks);
  lo = c0 + static_cast<int>(static_cast<int64_t>(c1 - c0) * warp / kWarps);
  hi = c0 + static_cast<int>(static_cast<int64_t>(c1 - c0) * (warp + 1) / kWarps);
}

// ---- K x packed-N weights ----------------------------------------------------
// One unit = 32 k.  A thread holds rows k0 + 8t + i (i < 8) of its group's 16
// columns: x[i].x = columns 0-7, x[i].y = 8-15 (byte b = columns 2b, 2b + 1).

struct KnStep {
  uint2 x[8];
  uint2 a;  // activation row g, k0 + 8t .. + 7
};

__device__ __forceinline__ void kn_load(KnStep& s, const Params& p, int unit, int col, bool col_ok, int g, int t) {
  const int k = unit * 32 + 8 * t;
  const size_t row_bytes = static_cast<size_t>(p.N) / 2;
  const uint8_t* w = p.qweight + static_cast<size_t>(k) * row_bytes + col / 2;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    s.x[i] = col_ok ? __ldg(reinterpret_cast<const uint2*>(w + i * row_bytes)) : make_uint2(0u, 0u);
  s.a = g < p.M ? __ldg(reinterpret_cast<const uint2*>(p.act + static_cast<size_t>(g) * p.K + k)) : make_uint2(0u, 0u);
}

// 4 x 4 byte transpose: out[b] = byte b of w0..w3 (w0's in the low byte)
__device__ __forceinline__ void transpose4(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, uint32_t (&out)[4]) {
  const uint32_t t0 = __byte_perm(w0, w1, 0x5140), t1 = __byte_perm(w0, w1, 0x7362);
  const uint32_t t2 = __byte_perm(w2, w3, 0x5140), t3 = __byte_perm(w2, w3, 0x7362);
  out[0] = __byte_perm(t0, t2, 0x5410);
  out[1] = __byte_perm(t0, t2, 0x7632);
  out[2] = __byte_perm(t1, t3, 0x5410);
  out[3] = __byte_perm(t1, t3, 0x7632);
}

// acc[c][j]: rows (2t, 2t + 1) x columns 8c + 2j, 8c + 2j + 1 of the group
__device__ __forceinline__ void kn_mma(const KnStep& s, int32_t (&acc)[2][4][4]) {
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint32_t q0[4], q1[4];  // k quads 0-3 and 4-7, per column pair
    transpose4(c ? s.x[0].y : s.x[0].x, c ? s.x[1].y : s.x[1].x, c ? s.x[2].y : s.x[2].x,
               c ? s.x[3].y : s.x[3].x, q0);
    transpose4(c ? s.x[4].y : s.x[4].x, c ? s.x[5].y : s.x[5].x, c ? s.x[6].y : s.x[6].x,
               c ? s.x[7].y : s.x[7].x, q1);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      mma_s8(acc[c][j], (q0[j] << 4) & kHi, q0[j] & kHi, (q1[j] << 4) & kHi, q1[j] & kHi, s.a.x, s.a.y);
  }
}

// ---- N x packed-K weights ----------------------------------------------------
// One unit = 128 k.  A thread holds, for MMA j, 32 k (16 bytes) at k0 + 32t of
// columns 16j + g and 16j + g + 8.

struct NkStep {
  uint4 wa[4], wb[4];
  uint4 a0, a1;  // activation row g, k0 + 32t .. + 31
};

__device__ __forceinline__ void nk_load(NkStep& s, const Params& p, int unit, int n0, int g, int t) {
  const int k = unit * 128 + 32 * t;
  const bool k_ok = k < p.K;  // K % 32 == 0: a thread's 32 k are all in or all out
  const size_t row_bytes = static_cast<size_t>(p.K) / 2;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int ca = n0 + 16 * j + g, cb = ca + 8;
    s.wa[j] = (k_ok && ca < p.N) ? __ldg(reinterpret_cast<const uint4*>(p.qweight + ca * row_bytes + k / 2))
                                 : make_uint4(0u, 0u, 0u, 0u);
    s.wb[j] = (k_ok && cb < p.N) ? __ldg(reinterpret_cast<const uint4*>(p.qweight + cb * row_bytes + k / 2))
                                 : make_uint4(0u, 0u, 0u, 0u);
  }
  if (k_ok && g < p.M) {
    const uint4* a = reinterpret_cast<const uint4*>(p.act + static_cast<size_t>(g) * p.K + k);
    s.a0 = __ldg(a);
    s.a1 = __ldg(a + 1);
  } else {
    s.a0 = s.a1 = make_uint4(0u, 0u, 0u, 0u);
  }
}

__device__ __forceinline__ uint32_t word(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// acc[j]: rows (2t, 2t + 1) x columns 16j + g, 16j + g + 8
__device__ __forceinline__ void nk_mma(const NkStep& s, int32_t (&acc)[4][4]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {  // 8 k per q: fragment k 4t + i = even k 2i, 16 + 4t + i = odd k 2i + 1
    const uint32_t lo = word(q < 2 ? s.a0 : s.a1, (2 * q) & 3), hi = word(q < 2 ? s.a0 : s.a1, (2 * q + 1) & 3);
    const uint32_t b0 = __byte_perm(lo, hi, 0x6420), b1 = __byte_perm(lo, hi, 0x7531);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t xa = word(s.wa[j], q), xb = word(s.wb[j], q);
      mma_s8(acc[j], (xa << 4) & kHi, (xb << 4) & kHi, xa & kHi, xb & kHi, b0, b1);
    }
  }
}

// ---- the kernel ----------------------------------------------------------------

template <int LAYOUT, typename TOut>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(const Params p) {
  constexpr int CB = LAYOUT == CONVROT_LAYOUT_KN ? kCbKN : kCbNK;
  __shared__ __align__(16) int32_t red[kWarps][kMaxRows * CB];  // per-warp partial sums [row][column]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int rank = p.cluster > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int n0 = static_cast<int>(blockIdx.x) / p.cluster * CB;

  grid_dependency_wait();  // the activation codes may come from the previous kernel of the stream
  grid_dependents_launch();

  int32_t* mine = red[warp];
  if constexpr (LAYOUT == CONVROT_LAYOUT_KN) {
    int32_t acc[2][4][4] = {};
    const int col = n0 + 16 * g;
    const bool col_ok = col < p.N;  // N % 16 == 0: a group's 16 columns are all in or all out
    int lo, hi;
    k_range(p.K / 32, rank, p.cluster, warp, lo, hi);
    KnStep s0, s1;
    if (lo < hi) kn_load(s0, p, lo, col, col_ok, g, t);
    int u = lo;
    // two steps of loads in flight: step u + 1 is loaded while step u computes
    for (; u + 1 < hi; u += 2) {
      kn_load(s1, p, u + 1, col, col_ok, g, t);
      kn_mma(s0, acc);
      if (u + 2 < hi) kn_load(s0, p, u + 2, col, col_ok, g, t);
      kn_mma(s1, acc);
    }
    if (u < hi) kn_mma(s0, acc);
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int cl = 16 * g + 8 * c + 2 * j;
        mine[(2 * t) * CB + cl] = acc[c][j][0];
        mine[(2 * t + 1) * CB + cl] = acc[c][j][1];
        mine[(2 * t) * CB + cl + 1] = acc[c][j][2];
        mine[(2 * t + 1) * CB + cl + 1] = acc[c][j][3];
      }
  } else {
    int32_t acc[4][4] = {};
    int lo, hi;
    k_range((p.K + 127) / 128, rank, p.cluster, warp, lo, hi);
    NkStep s0, s1;
    if (lo < hi) nk_load(s0, p, lo, n0, g, t);
    int u = lo;
    for (; u + 1 < hi; u += 2) {
      nk_load(s1, p, u + 1, n0, g, t);
      nk_mma(s0, acc);
      if (u + 2 < hi) nk_load(s0, p, u + 2, n0, g, t);
      nk_mma(s1, acc);
    }
    if (u < hi) nk_mma(s0, acc);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int cl = 16 * j + g;
      mine[(2 * t) * CB + cl] = acc[j][0];
      mine[(2 * t + 1) * CB + cl] = acc[j][1];
      mine[(2 * t) * CB + cl + 8] = acc[j][2];
      mine[(2 * t + 1) * CB + cl + 8] = acc[j][3];
    }
  }
  __syncthreads();

  // this CTA's partial of rows < M: the sum over its warps, into red[0]
  const int items = p.M * CB;
  for (int i = threadIdx.x; i < items; i += kThreads) {
    int32_t v = red[0][i];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) v += red[w][i];
    red[0][i] = v;
  }
  if (p.cluster > 1) cluster_sync();
  else __syncthreads();

  if (rank == 0) {
    TOut* out = static_cast<TOut*>(p.out);
    for (int i = threadIdx.x; i < items; i += kThreads) {
      const int r = i / CB, n = n0 + i % CB;
      uint32_t v = static_cast<uint32_t>(red[0][i]);
      uint32_t rem[kMaxCluster];
#pragma unroll
      for (int q = 1; q < kMaxCluster; ++q)
        rem[q] = q < p.cluster ? dsmem_ld(mapa_shared(&red[0][i], static_cast<uint32_t>(q))) : 0u;
#pragma unroll
      for (int q = 1; q < kMaxCluster; ++q) v += rem[q];
      if (n < p.N) {
        const int32_t dot = static_cast<int32_t>(v) >> 4;  // 16 * dot exactly
        const float b = p.bias ? __ldg(p.bias + n) : 0.0f;
        const float y = __fadd_rn(__fmul_rn(__fmul_rn(__int2float_rn(dot), __ldg(p.xscales + r)), __ldg(p.wscales + n)), b);
        out[static_cast<int64_t>(r) * p.N + n] = cvt_out<TOut>(y);
      }
    }
  }
  // no CTA leaves while the rank-0 CTA may still read its shared memory
  if (p.cluster > 1) cluster_sync();
}

template <int LAYOUT, typename TOut>
static int launch_t(const Params& p, int col_blocks, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(col_blocks * p.cluster), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(p.cluster);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see grid_dependency_wait
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  CONVROT_CUDA_CHECK(cudaLaunchKernelEx(&cfg, gemv_kernel<LAYOUT, TOut>, p));
  return check_launch("w4a4 gemv");
}

}  // namespace gemv

bool gemv_supported(int layout, int64_t m, int64_t n, int64_t k) {
  if (m < 1 || m > gemv::kMaxRows || k % 32 != 0) return false;
  return layout == CONVROT_LAYOUT_NK || n % 16 == 0;
}

// Called by convrot_w4a4_gemm after its argument checks, for shapes that
// gemv_supported accepts.
int launch_gemv(const int8_t* act, const uint8_t* qweight, int layout, const float* xscales, const float* wscales,
                const float* bias, void* out, int out_dtype, int64_t m, int64_t n, int64_t k, cudaStream_t stream) {
  using namespace gemv;
  Params p;
  p.act = act;
  p.qweight = qweight;
  p.xscales = xscales;
  p.wscales = wscales;
  p.bias = bias;
  p.out = out;
  p.M = static_cast<int>(m);
  p.N = static_cast<int>(n);
  p.K = static_cast<int>(k);
  const int cb = layout == CONVROT_LAYOUT_KN ? kCbKN : kCbNK;
  const int unit = layout == CONVROT_LAYOUT_KN ? 32 : 128;
  const int units = static_cast<int>((k + unit - 1) / unit);
  const int col_blocks = static_cast<int>((n + cb - 1) / cb);
  // split K over a cluster so that about two CTAs run per SM, with at least
  // one K unit per warp
  int c = 2 * device_sm_count() / col_blocks;
  if (c > kMaxCluster) c = kMaxCluster;
  if (c > units / kWarps) c = units / kWarps;
  p.cluster = c < 1 ? 1 : c;
  if (layout == CONVROT_LAYOUT_NK) {
    switch (out_dtype) {
      case CONVROT_BF16: return launch_t<CONVROT_LAYOUT_NK, __nv_bfloat16>(p, col_blocks, stream);
      case CONVROT_F16: return launch_t<CONVROT_LAYOUT_NK, __half>(p, col_blocks, stream);
      default: return launch_t<CONVROT_LAYOUT_NK, float>(p, col_blocks, stream);
    }
  }
  switch (out_dtype) {
    case CONVROT_BF16: return launch_t<CONVROT_LAYOUT_KN, __nv_bfloat16>(p, col_blocks, stream);
    case CONVROT_F16: return launch_t<CONVROT_LAYOUT_KN, __half>(p, col_blocks, stream);
    default: return launch_t<CONVROT_LAYOUT_KN, float>(p, col_blocks, stream);
  }
}

}  // namespace convrot
