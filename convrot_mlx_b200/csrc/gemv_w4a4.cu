// W4A4 GEMM for at most 8 activation rows on sm_100a: a weight-streaming
// kernel whose weights go from HBM straight into MMA fragments.
//
// With m <= 8 (the modulation linears of a DiT at m = batch, decode-style
// calls) the op does 2 m multiply-adds per packed weight nibble: ~16 integer
// ops per weight byte, far below any tensor-core roofline ridge, so the bound
// is reading the K * N / 2 packed weight bytes from HBM once.  A tile kernel
// stages weights through shared memory and TMEM, and each of its stages waits
// on the previous hand-off; at m <= 8 those waits, not bandwidth, set its
// time.  Here each warp streams its share of the weights through a small
// ring of its own in shared memory, filled by cp.async copies that its lanes
// issue several K units ahead (no barrier with any other warp), reads them
// into registers, turns them into int8 MMA fragments with byte permutes, and
// issues register-operand MMAs
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
// * K x packed-N weights: thread (g = lane / 4, t = lane % 4) reads rows
//   k0 + 8t .. + 7, 16 columns each (8 bytes).  A 4 x 4 byte transpose of
//   four rows (8 byte permutes) gives words of 4 consecutive k for one byte
//   position, i.e. for a column pair; shift / mask split the pair.  MMA j of
//   an 8-column chunk takes columns 2j (fragment row g) and 2j + 1 (row
//   g + 8); fragment k index 4t + i is real k k0 + 8t + i, and 16 + 4t + i
//   is k0 + 8t + 4 + i, so the activation fragment is the 8 bytes of row g
//   at k0 + 8t, one read.
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

// ---- each warp's ring of K units in shared memory ----------------------------
// A warp keeps DEPTH - 1 units of its K slice in flight as cp.async copies
// (issued by its own lanes, no registers held) while it computes on the
// oldest; bytes in flight are bounded by shared memory, not registers.

// `BYTES` (8 or 16) global -> shared; only `src_bytes` are read, the rest of
// the destination is zero-filled (0 reads nothing)
template <int BYTES>
__device__ __forceinline__ void cp_async(uint32_t dst, const void* src, uint32_t src_bytes) {
  if constexpr (BYTES == 16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}

// ---- K x packed-N weights ----------------------------------------------------
// One unit = 32 k: rows k0 .. k0 + 31 of the CTA's 128 columns (64 bytes a
// row) and the activation rows' 32 k, in the ring.  Thread (g, t) computes on rows
// k0 + 8t + i (i < 8), 16 columns each: x[i].x = columns 0-7 of its group,
// x[i].y = 8-15 (byte b = columns 2b, 2b + 1).

constexpr int kKnW = 32 * 64;           // weight bytes of a unit
constexpr int kKnSlot = kKnW + 8 * 32;  // + 8 activation rows x 32 k
constexpr int kKnDepth = 4;

struct KnStep {
  uint2 x[8];
  uint2 a;  // activation row g, k0 + 8t .. + 7
};

// Row r of the unit sits at slot row (r % 8) * 4 + r / 8, so the 32 lanes'
// reads of one i (rows 8t + i) are 256 contiguous bytes.  CHUNK: 16 when the
// weight rows are 16-byte aligned (N % 32 == 0), else 8.
// A copy instruction covers whole 64-byte row segments (64 / CHUNK lanes a
// row), so it touches few cache lines.
template <int CHUNK>
__device__ __forceinline__ void kn_issue(uint32_t slot, const Params& p, int unit, int n0, int lane) {
  constexpr int kLanesPerRow = 64 / CHUNK, kRowsPerCopy = 32 / kLanesPerRow;
  const size_t row_bytes = static_cast<size_t>(p.N) / 2;
  const int q = lane % kLanesPerRow;  // this lane's chunk of each row segment
  const int left = (p.N - n0) / 2 - q * CHUNK;  // bytes of the chunk inside the row
  const uint32_t n = left >= CHUNK ? CHUNK : (left > 0 ? static_cast<uint32_t>(left) : 0u);
#pragma unroll
  for (int c = 0; c < 32 / kRowsPerCopy; ++c) {
    const int r = c * kRowsPerCopy + lane / kLanesPerRow;
    const uint8_t* src = p.qweight + static_cast<size_t>(unit * 32 + r) * row_bytes + n0 / 2 + q * CHUNK;
    cp_async<CHUNK>(slot + ((r & 7) * 4 + (r >> 3)) * 64 + q * CHUNK, n ? static_cast<const void*>(src) : p.qweight,
                    n);
  }
}

// the unit's activation rows (zero past M): lanes 0-15, 16 bytes each
__device__ __forceinline__ void kn_issue_act(uint32_t slot, const Params& p, int unit, int lane) {
  if (lane < 16) {
    const int r = lane >> 1, h = lane & 1;
    const bool ok = r < p.M;
    cp_async<16>(slot + kKnW + r * 32 + h * 16,
                 ok ? static_cast<const void*>(p.act + static_cast<size_t>(r) * p.K + unit * 32 + h * 16) : p.act,
                 ok ? 16u : 0u);
  }
}

__device__ __forceinline__ void kn_read(KnStep& s, uint32_t slot, int g, int t) {
#pragma unroll
  for (int i = 0; i < 8; ++i) s.x[i] = lds64(slot + (i * 4 + t) * 64 + 8 * g);
  s.a = lds64(slot + kKnW + g * 32 + 8 * t);
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
// One unit = 128 k: 64 bytes of each of the CTA's 64 columns and the
// activation rows' 128 k, in the ring.  Thread (g, t) computes, for MMA j, on 32 k (16
// bytes) at k0 + 32t of columns 16j + g and 16j + g + 8.

constexpr int kNkW = 64 * 64;
constexpr int kNkActStride = 144;  // 128 k + 16 bytes, so rows g and g + 1 fall on other banks
constexpr int kNkSlot = kNkW + 8 * kNkActStride;
constexpr int kNkDepth = 3;

struct NkStep {
  uint4 wa[4], wb[4];
  uint4 a0, a1;  // activation row g, k0 + 32t .. + 31
};

__device__ __forceinline__ void nk_issue(uint32_t slot, const Params& p, int unit, int n0, int lane) {
  const size_t row_bytes = static_cast<size_t>(p.K) / 2;
  const int kb = unit * 64;                               // the unit's byte offset in a weight row
  const int kvalid = static_cast<int>(row_bytes) - kb;    // > 0, a multiple of 16
  const int q = lane & 3;  // this lane's 16 bytes of each column's 64 (4 lanes a column, 8 columns a copy)
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int col = c * 8 + (lane >> 2);
    const bool ok = n0 + col < p.N && q * 16 < kvalid;
    const uint8_t* src = p.qweight + static_cast<size_t>(n0 + col) * row_bytes + kb + q * 16;
    cp_async<16>(slot + col * 64 + q * 16, ok ? static_cast<const void*>(src) : p.qweight, ok ? 16u : 0u);
  }
}

// the unit's activation rows (zero past M or K): 64 chunks of 16 bytes
__device__ __forceinline__ void nk_issue_act(uint32_t slot, const Params& p, int unit, int lane) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int id = lane + 32 * h, r = id >> 3, part = id & 7;
    const bool ok = r < p.M && unit * 128 + part * 16 < p.K;
    cp_async<16>(slot + kNkW + r * kNkActStride + part * 16,
                 ok ? static_cast<const void*>(p.act + static_cast<size_t>(r) * p.K + unit * 128 + part * 16)
                    : p.act,
                 ok ? 16u : 0u);
  }
}

__device__ __forceinline__ void nk_read(NkStep& s, uint32_t slot, int g, int t) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    s.wa[j] = lds128(slot + (16 * j + g) * 64 + 16 * t);
    s.wb[j] = lds128(slot + (16 * j + g + 8) * 64 + 16 * t);
  }
  s.a0 = lds128(slot + kNkW + g * kNkActStride + 32 * t);
  s.a1 = lds128(slot + kNkW + g * kNkActStride + 32 * t + 16);
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

template <int LAYOUT>
__host__ __device__ constexpr int ring_bytes() {
  return LAYOUT == CONVROT_LAYOUT_KN ? kWarps * kKnDepth * kKnSlot : kWarps * kNkDepth * kNkSlot;
}

template <int LAYOUT, int CHUNK, typename TOut>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const Params p) {
  constexpr bool kKN = LAYOUT == CONVROT_LAYOUT_KN;
  constexpr int CB = kKN ? kCbKN : kCbNK;
  constexpr int SLOT = kKN ? kKnSlot : kNkSlot;
  constexpr int DEPTH = kKN ? kKnDepth : kNkDepth;
  static_assert(kWarps * kMaxRows * CB * 4 <= ring_bytes<LAYOUT>(), "partial sums overlay the rings");
  static_assert(kThreads % CB == 0, "a thread's epilogue items share one column");
  // the warps' rings; after the K loop the same memory holds the per-warp
  // partial sums red[warp][row * CB + column]
  extern __shared__ __align__(128) uint8_t smem[];
  int32_t* red = reinterpret_cast<int32_t*>(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int rank = p.cluster > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int n0 = static_cast<int>(blockIdx.x) / p.cluster * CB;
  const uint32_t ring = smem_u32(smem) + static_cast<uint32_t>(warp * DEPTH * SLOT);

  int lo, hi;
  k_range(kKN ? p.K / 32 : (p.K + 127) / 128, rank, p.cluster, warp, lo, hi);
  const int units = hi - lo;
  auto issue_w = [&](int i) {
    if constexpr (kKN) kn_issue<CHUNK>(ring + (i % DEPTH) * SLOT, p, lo + i, n0, lane);
    else nk_issue(ring + (i % DEPTH) * SLOT, p, lo + i, n0, lane);
  };
  auto issue_a = [&](int i) {
    if constexpr (kKN) kn_issue_act(ring + (i % DEPTH) * SLOT, p, lo + i, lane);
    else nk_issue_act(ring + (i % DEPTH) * SLOT, p, lo + i, lane);
  };
  // The packed weights do not come from the previous kernel of the stream
  // (no kernel of this library that lets its dependents start early writes
  // packed weights), so the first units' weight copies start before waiting
  // for it; their activation rows follow after the wait, as one more group.
  // Commit groups: W0 .. W(D-2), A(0 .. D-2), then one per later unit.
#pragma unroll
  for (int i = 0; i < DEPTH - 1; ++i) {
    if (i < units) issue_w(i);
    cp_async_commit();
  }
  // The epilogue items of a thread (i = threadIdx.x + 256 j) share one
  // column, i % CB == threadIdx.x % CB, so its weight scale and bias, which
  // do not come from the previous kernel either, load now.
  __shared__ float row_scale[kMaxRows];
  const int my_n = n0 + static_cast<int>(threadIdx.x) % CB;
  const float my_ws = (rank == 0 && my_n < p.N) ? __ldg(p.wscales + my_n) : 0.0f;
  const float my_b = (rank == 0 && my_n < p.N && p.bias) ? __ldg(p.bias + my_n) : 0.0f;
  grid_dependency_wait();  // the activation codes may come from the previous kernel of the stream
  grid_dependents_launch();
#pragma unroll
  for (int i = 0; i < DEPTH - 1; ++i)
    if (i < units) issue_a(i);
  cp_async_commit();
  if (rank == 0 && threadIdx.x < p.M) row_scale[threadIdx.x] = __ldg(p.xscales + threadIdx.x);

  int32_t* mine = red + warp * kMaxRows * CB;
  // unit i and its activations have landed (this lane's copies): all but
  // the min(i + 1, DEPTH - 1) most recent groups are complete
  auto wait_unit = [&](int i) {
    static_assert(DEPTH >= 2 && DEPTH <= 6, "wait_unit covers rings of 2-6 units");
    if (DEPTH >= 3 && i == 0) cp_async_wait<1>();
    else if (DEPTH >= 4 && i == 1) cp_async_wait<2>();
    else if (DEPTH >= 5 && i == 2) cp_async_wait<3>();
    else if (DEPTH >= 6 && i == 3) cp_async_wait<4>();
    else cp_async_wait<DEPTH - 1>();
  };
  auto refill = [&](int i) {
    if (i + DEPTH - 1 < units) {
      issue_w(i + DEPTH - 1);
      issue_a(i + DEPTH - 1);
    }
    cp_async_commit();
  };
  if constexpr (kKN) {
    int32_t acc[2][4][4] = {};
    for (int i = 0; i < units; ++i) {
      refill(i);
      wait_unit(i);
      __syncwarp();  // ... and every lane's
      KnStep s;
      kn_read(s, ring + (i % DEPTH) * SLOT, g, t);
      kn_mma(s, acc);
      __syncwarp();  // all reads of the slot done before it is refilled
    }
    cp_async_wait<0>();
    __syncthreads();  // every warp is out of its ring before the partial sums overlay it
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
    for (int i = 0; i < units; ++i) {
      refill(i);
      wait_unit(i);
      __syncwarp();
      NkStep s;
      nk_read(s, ring + (i % DEPTH) * SLOT, g, t);
      nk_mma(s, acc);
      __syncwarp();
    }
    cp_async_wait<0>();
    __syncthreads();
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

  // this CTA's partial of rows < M: the sum over its warps, into warp 0's slice
  const int items = p.M * CB;
  for (int i = threadIdx.x; i < items; i += kThreads) {
    int32_t v = red[i];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) v += red[w * kMaxRows * CB + i];
    red[i] = v;
  }
  if (p.cluster > 1) cluster_sync();
  else __syncthreads();

  if (rank == 0) {
    TOut* out = static_cast<TOut*>(p.out);
    for (int i = threadIdx.x; i < items; i += kThreads) {
      const int r = i / CB, n = n0 + i % CB;
      uint32_t v = static_cast<uint32_t>(red[i]);
      uint32_t rem[kMaxCluster];
#pragma unroll
      for (int q = 1; q < kMaxCluster; ++q)
        rem[q] = q < p.cluster ? dsmem_ld(mapa_shared(&red[i], static_cast<uint32_t>(q))) : 0u;
#pragma unroll
      for (int q = 1; q < kMaxCluster; ++q) v += rem[q];
      if (n < p.N) {  // n == my_n
        const int32_t dot = static_cast<int32_t>(v) >> 4;  // 16 * dot exactly
        const float y = __fadd_rn(__fmul_rn(__fmul_rn(__int2float_rn(dot), row_scale[r]), my_ws), my_b);
        out[static_cast<int64_t>(r) * p.N + n] = cvt_out<TOut>(y);
      }
    }
  }
  // no CTA leaves while the rank-0 CTA may still read its shared memory
  if (p.cluster > 1) cluster_sync();
}

template <int LAYOUT, int CHUNK, typename TOut>
static int launch_t(const Params& p, int col_blocks, cudaStream_t stream) {
  auto kernel = gemv_kernel<LAYOUT, CHUNK, TOut>;
  constexpr int smem = ring_bytes<LAYOUT>();
  CONVROT_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(col_blocks * p.cluster), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
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
  CONVROT_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, p));
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
  // split K over a cluster so that the CTAs make one wave, one per SM (a
  // second wave, or two CTAs per SM, measured slower on B200), with at least
  // one K unit per warp
  int c = device_sm_count() / col_blocks;
  if (c > kMaxCluster) c = kMaxCluster;
  if (c > units / kWarps) c = units / kWarps;
  p.cluster = c < 1 ? 1 : c;
  if (layout == CONVROT_LAYOUT_NK) {
    switch (out_dtype) {
      case CONVROT_BF16: return launch_t<CONVROT_LAYOUT_NK, 16, __nv_bfloat16>(p, col_blocks, stream);
      case CONVROT_F16: return launch_t<CONVROT_LAYOUT_NK, 16, __half>(p, col_blocks, stream);
      default: return launch_t<CONVROT_LAYOUT_NK, 16, float>(p, col_blocks, stream);
    }
  }
  if (n % 32 == 0) {  // weight rows 16-byte aligned
    switch (out_dtype) {
      case CONVROT_BF16: return launch_t<CONVROT_LAYOUT_KN, 16, __nv_bfloat16>(p, col_blocks, stream);
      case CONVROT_F16: return launch_t<CONVROT_LAYOUT_KN, 16, __half>(p, col_blocks, stream);
      default: return launch_t<CONVROT_LAYOUT_KN, 16, float>(p, col_blocks, stream);
    }
  }
  switch (out_dtype) {
    case CONVROT_BF16: return launch_t<CONVROT_LAYOUT_KN, 8, __nv_bfloat16>(p, col_blocks, stream);
    case CONVROT_F16: return launch_t<CONVROT_LAYOUT_KN, 8, __half>(p, col_blocks, stream);
    default: return launch_t<CONVROT_LAYOUT_KN, 8, float>(p, col_blocks, stream);
  }
}

}  // namespace convrot
