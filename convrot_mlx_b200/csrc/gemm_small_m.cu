// W4A4 GEMM for few activation rows (m <= 64) on sm_100a: swap-AB tcgen05.
//
// With m = batch (the modulation and embedding linears of a DiT, 1-8 rows)
// or BASELINE config 1 (m = 64), a 128- or 256-row activation tile would
// leave most of every MMA empty, and the work is bound by reading the
// packed weights from HBM.  This kernel puts the weights on the MMA's M
// side and the activations on its N side:
//
//   D[n, m] (TMEM, int32) += W8[n, k] (smem, expanded nibbles) x A[m, k]^T
//
// with MMA M = 128 weight rows, N = m rounded up to 16 (rows past m are TMA
// zero fill), K = 32 per instruction, kind::i8.  The packed weights stream
// through a TMA ring of their own, 6 or 7 deep (a slot is free again as
// soon as the transform warps have read it); the activation codes, reused
// by every CTA, through a 4-deep ring freed by the MMA.  Eight transform
// warps expand each stage's nibbles (x 16, exact) into the 128-byte-swizzled
// int8 tile the tensor core reads -- K-major for N x packed-K weights,
// MN-major (the A operand transposed) for K x packed-N weights -- into a
// ring of 2 or 3 slots.
//
// Parallelism comes from splitting K over a cluster of up to 8 CTAs per
// 128-row weight tile: each CTA accumulates its share of the K stages in its
// own TMEM, writes the int32 partial sums to its shared memory, and after a
// cluster barrier the tile's rank-0 CTA adds its peers' partials over
// distributed shared memory (exact integer sums) and runs the epilogue
// out[m, n] = T(fl(fl(float(dot) * xs[m]) * ws[n]) + bias[n]), the reference
// order (core.py:932-936).  No TMA load uses cluster multicast.
#include <cudaTypedefs.h>

#include "common.cuh"

namespace convrot {
namespace small_m {

constexpr int BN = 128;             // weight rows per tile (MMA M)
constexpr int KS = 256;             // K per stage
constexpr int kMaxSW = 8;           // packed-weight ring slots (at most)
constexpr int SA = 4;               // activation ring slots
constexpr int kMaxX = 4;            // expanded-weight slots (at most)
constexpr int kMaxRows = 64;        // activation rows handled (MMA N <= 64)
constexpr int kMaxCluster = 8;
constexpr int kBpBytes = BN * KS / 2;   // 16 KB packed weights per stage
constexpr int kW8Bytes = BN * KS;       // 32 KB expanded weights per stage
constexpr int kActMaxBytes = kMaxRows * KS;  // activations per stage (64 rows)
constexpr int kXWarps = 8;
constexpr int kXThreads = kXWarps * 32;
// warp 0 streams the packed weights, warp 1 issues the MMAs, warps 2-9
// transform (and 2-5 then read TMEM), warp 10 streams the activation codes
constexpr int kWarpTma = 0, kWarpMma = 1, kWarpX0 = 2, kWarpAct = kWarpX0 + kXWarps;
constexpr int kThreads = (kWarpAct + 1) * 32;  // 352
constexpr int kItems = kBpBytes / 16;                // 1024 transform items per stage
constexpr int kItemsPerThread = kItems / kXThreads;  // 4
constexpr uint64_t kTimeoutNs = 4000000000ull;

struct alignas(8) Bars {
  uint64_t wfull[kMaxSW];   // TMA: a stage's packed weights landed
  uint64_t wempty[kMaxSW];  // the 8 transform warps have read them
  uint64_t afull[SA];       // TMA: a stage's activation codes landed
  uint64_t aempty[SA];      // the stage's MMAs are done with them
  uint64_t w8_ready[kMaxX];
  uint64_t w8_empty[kMaxX];
  uint64_t mma_done;
  uint32_t tmem_base;
  int err;
  float xs[64];  // the activation row scales, staged once for the epilogue
};

constexpr size_t kSmemCap = 232448;
// Ring depths for np activation rows: the expanded-weight and activation
// rings first, then as many packed-weight slots as fit.
// (the MMA -> transform -> MMA round trip spans x_slots stages)
constexpr int x_slots(int np) { return np > 32 ? 2 : np > 16 ? 3 : kMaxX; }
constexpr size_t fixed_bytes(int np) {
  return 1024 + sizeof(Bars) + static_cast<size_t>(SA) * np * KS + static_cast<size_t>(x_slots(np)) * kW8Bytes;
}
constexpr int sw_slots(int np) {
  return (kSmemCap - fixed_bytes(np)) / kBpBytes > kMaxSW ? kMaxSW
                                                           : static_cast<int>((kSmemCap - fixed_bytes(np)) / kBpBytes);
}
constexpr size_t smem_bytes(int np) { return fixed_bytes(np) + static_cast<size_t>(sw_slots(np)) * kBpBytes; }
static_assert(sw_slots(kMaxRows) >= 4 && smem_bytes(kMaxRows) <= kSmemCap, "shared memory budget");

struct Params {
  const uint8_t* qweight;
  const float* xscales;
  const float* wscales;
  const float* bias;
  void* out;
  int M, N, K;
  int np;        // MMA N: M rounded up to 16
  int k_stages;  // ceil(K / KS)
  int cluster;   // CTAs splitting one tile's K stages
  int sw, x;     // packed-weight and expanded-weight ring depths
  int* err_word; // device error word (bounded waits that time out record here)
};

__device__ __noinline__ bool wait(uint64_t* bar, uint32_t parity, Bars* b, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 0) {
      if (*reinterpret_cast<volatile int*>(&b->err)) return false;
      if (globaltimer() - t0 > kTimeoutNs) {
        atomicCAS(&b->err, 0, code);
        return false;
      }
    }
  }
}

// 16 packed bytes -> 32 int8 values 16 * nibble, in element order (the
// nibble moved to the high half of its byte: no sign extension needed).
__device__ __forceinline__ void expand16(const uint4 w, uint32_t (&o)[8]) {
  const uint32_t s[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t even = (s[j] << 4) & 0xF0F0F0F0u;
    const uint32_t odd = s[j] & 0xF0F0F0F0u;
    o[2 * j] = __byte_perm(even, odd, 0x5140);
    o[2 * j + 1] = __byte_perm(even, odd, 0x7362);
  }
}

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ uint32_t ld_dsmem_u32(uint32_t cluster_addr) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(cluster_addr) : "memory");
  return v;
}

template <typename TOut>
__device__ __forceinline__ void store_out(TOut* p, float v) {
  *p = cvt_out<TOut>(v);
}

template <int LAYOUT, typename TOut>
__global__ void __launch_bounds__(kThreads, 1)
    small_m_kernel(const __grid_constant__ CUtensorMap tmap_act, const __grid_constant__ CUtensorMap tmap_w,
                   const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int np = p.np, SW = p.sw, X = p.x;
  const int act_bytes = np * KS;                 // activations per stage
  uint8_t* sW8 = smem;                           // X x 32 KB (also the partial sums at the end)
  uint8_t* sBp = sW8 + X * kW8Bytes;             // SW x 16 KB
  uint8_t* sAct = sBp + SW * kBpBytes;           // SA x np * 256
  Bars* bars = reinterpret_cast<Bars*>(sAct + SA * act_bytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster_ctarank());
  const int tile = blockIdx.x / p.cluster;
  const int g0 = static_cast<int>(static_cast<int64_t>(rank) * p.k_stages / p.cluster);  // this CTA's stages
  const int g1 = static_cast<int>(static_cast<int64_t>(rank + 1) * p.k_stages / p.cluster);
  const int nst = g1 - g0;
  const uint32_t tmem_cols = np > 32 ? 64 : 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SW; ++s) {
      mbar_init(&bars->wfull[s], 1);
      mbar_init(&bars->wempty[s], kXWarps);
    }
    for (int s = 0; s < SA; ++s) {
      mbar_init(&bars->afull[s], 1);
      mbar_init(&bars->aempty[s], 1);
    }
    for (int s = 0; s < X; ++s) {
      mbar_init(&bars->w8_ready[s], kXWarps);
      mbar_init(&bars->w8_empty[s], 1);
    }
    mbar_init(&bars->mma_done, 1);
    bars->err = 0;
    fence_mbar_init();
    prefetch_tensormap(&tmap_act);
    prefetch_tensormap(&tmap_w);
  }
  if (warp == kWarpMma) {
    tmem_alloc(&bars->tmem_base, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;
  grid_dependency_wait();  // the activation codes may come from the previous kernel of the stream
  grid_dependents_launch();
  if (warp == kWarpAct + 0 && rank == 0) {  // row scales for the epilogue (read after the cluster barrier)
    for (int m = lane; m < p.M; m += 32) bars->xs[m] = __ldg(p.xscales + m);
  }

  if (warp == kWarpTma || warp == kWarpAct) {
    // the two streams advance independently, each from a warp of its own
    if (lane == 0) {
      bool ok = true;
      for (int g = 0; g < nst; ++g) {
        const int ks = g0 + g;
        if (warp == kWarpTma) {
          const int slot = g % SW;
          if (!wait(&bars->wempty[slot], ((g / SW) & 1) ^ 1, bars, 51)) { ok = false; break; }
          mbar_arrive_expect_tx(&bars->wfull[slot], kBpBytes);
          if constexpr (LAYOUT == CONVROT_LAYOUT_NK)
            tma_load_2d(sBp + slot * kBpBytes, &tmap_w, &bars->wfull[slot], ks * (KS / 2), tile * BN);
          else
            tma_load_2d(sBp + slot * kBpBytes, &tmap_w, &bars->wfull[slot], tile * (BN / 2), ks * KS);
        } else {
          const int slot = g % SA;
          if (!wait(&bars->aempty[slot], ((g / SA) & 1) ^ 1, bars, 57)) { ok = false; break; }
          mbar_arrive_expect_tx(&bars->afull[slot], act_bytes);
          tma_load_3d(sAct + slot * act_bytes, &tmap_act, &bars->afull[slot], 0, 0, 2 * ks);
        }
      }
      if (!ok) {  // let a copy still in flight land before the CTA tears down
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 2000000ull) {
        }
      }
    }
  } else if (warp == kWarpMma) {
    if (lane == 0) {
      // D s32, A and B s8, A major = MN for K x packed-N weights, N = np, M = 128
      const uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) |
                             (static_cast<uint32_t>(LAYOUT == CONVROT_LAYOUT_KN) << 15) |
                             (static_cast<uint32_t>(np >> 3) << 17) | (static_cast<uint32_t>(BN >> 4) << 24);
      const uint32_t w_base = smem_u32(sW8), a_base = smem_u32(sAct);
      for (int g = 0; g < nst; ++g) {
        const int slot = g % SA, x = g % X, ks = g0 + g;
        if (!wait(&bars->afull[slot], (g / SA) & 1, bars, 52)) break;
        if (!wait(&bars->w8_ready[x], (g / X) & 1, bars, 53)) break;
        tc_fence_after();
        const int k_rem = p.K - ks * KS;
        const int steps = k_rem >= KS ? KS / 32 : k_rem / 32;
        const uint32_t w_addr = w_base + x * kW8Bytes, a_addr = a_base + slot * act_bytes;
        for (int j = 0; j < steps; ++j) {
          // weights: K-major (NK) -- two 16 KB K chunks of 128 rows; MN-major
          // (KN) -- K rows of 128 bytes, 32 rows per step
          const uint64_t wdesc = LAYOUT == CONVROT_LAYOUT_NK
                                     ? smem_desc(w_addr + (j >> 2) * 16384 + (j & 3) * 32, 16, 1024, 2)
                                     : smem_desc(w_addr + j * 4096, kW8Bytes, 1024, 2);
          const uint64_t adesc = smem_desc(a_addr + (j >> 2) * (np * 128) + (j & 3) * 32, 16, 1024, 2);
          mma_i8(tmem_base, wdesc, adesc, idesc, (g | j) != 0 ? 1u : 0u);
        }
        mma_commit(&bars->aempty[slot]);
        mma_commit(&bars->w8_empty[x]);
      }
      mma_commit(&bars->mma_done);
    }
  } else {
    // ---------------- transform: packed nibbles -> int8 (x 16) ----------------
    const int xt = (warp - kWarpX0) * 32 + lane;
    uint32_t src[kItemsPerThread], d0[kItemsPerThread], d1[kItemsPerThread];
#pragma unroll
    for (int i = 0; i < kItemsPerThread; ++i) {
      const int item = i * kXThreads + xt;
      if constexpr (LAYOUT == CONVROT_LAYOUT_NK) {
        // packed row n (128 bytes = 256 K), 16-byte chunk c (32 K) -> int8 K
        // chunk c / 4, 16-byte chunks 2j and 2j + 1 (j = c % 4) of row n; a
        // quarter-warp takes rows 2p, 2p + 1 with opposite K chunks so its
        // stores hit eight distinct bank groups
        const int qw = item >> 3, l = item & 7, h = qw & 1;
        const int n = 2 * (qw >> 1) + (l >> 2);
        const int c = (l & 3) + 4 * ((l >> 2) ^ h);
        const int kc = c >> 2, j = c & 3;
        src[i] = n * 128 + c * 16;
        const uint32_t row = kc * 16384 + n * 128;
        d0[i] = row + (((2 * j) ^ (n & 7)) << 4);
        d1[i] = row + (((2 * j + 1) ^ (n & 7)) << 4);
      } else {
        // packed row k (64 bytes = 128 N), chunk c -> MN-major int8 row k
        const int k = item >> 2, c = item & 3;
        src[i] = k * 64 + c * 16;
        const uint32_t row = (k >> 3) * 1024 + (k & 7) * 128;
        d0[i] = row + (((2 * c) ^ (k & 7)) << 4);
        d1[i] = row + (((2 * c + 1) ^ (k & 7)) << 4);
      }
    }
    for (int g = 0; g < nst; ++g) {
      const int slot = g % SW, x = g % X;
      if (!wait(&bars->wfull[slot], (g / SW) & 1, bars, 54)) break;
      uint4 w[kItemsPerThread];
      const uint8_t* bp = sBp + slot * kBpBytes;
#pragma unroll
      for (int i = 0; i < kItemsPerThread; ++i) w[i] = *reinterpret_cast<const uint4*>(bp + src[i]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->wempty[slot]);  // this warp has read the packed slot
      if (!wait(&bars->w8_empty[x], ((g / X) & 1) ^ 1, bars, 55)) break;
      const uint32_t dst = smem_u32(sW8 + x * kW8Bytes);
#pragma unroll
      for (int i = 0; i < kItemsPerThread; ++i) {
        uint32_t o[8];
        expand16(w[i], o);
        sts128(dst + d0[i], o[0], o[1], o[2], o[3]);
        sts128(dst + d1[i], o[4], o[5], o[6], o[7]);
      }
      fence_proxy_async_smem();  // generic stores -> the tensor core (async proxy)
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->w8_ready[x]);
    }

    // ---------------- partial sums (warps 2-5: TMEM lane quarters 2, 3, 0, 1) ----------------
    if (warp < kWarpX0 + 4) {
      const int quarter = warp & 3;
      const bool ok = wait(&bars->mma_done, 0, bars, 56);
      tc_fence_after();
      // the expanded-weight ring is idle now: partials as P[m][n_local] int32
      uint32_t* part = reinterpret_cast<uint32_t*>(sW8);
      const int nl = quarter * 32 + lane;
      for (int c = 0; c < np; c += 16) {
        uint32_t r[16];
        if (ok) {
          tmem_ld_32x32b_x16(tmem_base + ((static_cast<uint32_t>(quarter) * 32u) << 16) + c, r);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) r[i] = 0;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) part[(c + i) * BN + nl] = r[i];
      }
    }
  }

  // all partials written before any CTA of the cluster reads them
  tc_fence_before();
  __syncwarp();
  cluster_sync();
  tc_fence_after();

  if (rank == 0 && warp >= kWarpX0 && warp < kWarpX0 + 4) {
    const int quarter = warp & 3;
    const int nl = quarter * 32 + lane;
    const int n = tile * BN + nl;
    const uint32_t* part = reinterpret_cast<const uint32_t*>(sW8);
    const bool n_ok = n < p.N;
    const float ws = n_ok ? __ldg(p.wscales + n) : 0.0f;
    const float b = (n_ok && p.bias) ? __ldg(p.bias + n) : 0.0f;
    TOut* out = static_cast<TOut*>(p.out);
    uint32_t peer[kMaxCluster];
#pragma unroll
    for (int r = 1; r < kMaxCluster; ++r) peer[r] = r < p.cluster ? mapa_shared(part + nl, r) : 0u;
    for (int m0 = 0; m0 < p.M; m0 += 8) {
      // the peers' partials of 8 rows: all loads issued before any is summed
      uint32_t acc[8], rem[kMaxCluster][8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = m0 + i < p.M ? part[(m0 + i) * BN + nl] : 0u;
#pragma unroll
      for (int r = 1; r < kMaxCluster; ++r)
#pragma unroll
        for (int i = 0; i < 8; ++i)
          rem[r][i] = (r < p.cluster && m0 + i < p.M) ? ld_dsmem_u32(peer[r] + (m0 + i) * BN * 4) : 0u;
#pragma unroll
      for (int r = 1; r < kMaxCluster; ++r)
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += rem[r][i];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int m = m0 + i;
        if (m >= p.M) break;
        // the accumulator holds 16 * dot exactly (K * 56 * 16 < 2^31)
        const int32_t dot = static_cast<int32_t>(acc[i]) >> 4;
        const float v = __fadd_rn(__fmul_rn(__fmul_rn(__int2float_rn(dot), bars->xs[m]), ws), b);
        if (n_ok) store_out<TOut>(out + static_cast<int64_t>(m) * p.N + n, v);
      }
    }
  }

  // no CTA leaves while the rank-0 CTA may still read its shared memory
  __syncwarp();
  cluster_sync();
  if (warp == kWarpMma) {
    __syncwarp();
    tmem_dealloc(tmem_base, tmem_cols);
  }
  if (threadIdx.x == 0 && bars->err && p.err_word) atomicCAS(p.err_word, 0, bars->err);
}

}  // namespace small_m

namespace w4a4 {
int make_tmap_u8(CUtensorMap* map, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                 const uint32_t* box, CUtensorMapSwizzle swizzle, CUtensorMapDataType dtype);
}

bool small_m_supported(int layout, int64_t m, int64_t n, int64_t k) {
  return m >= 1 && m <= small_m::kMaxRows && k % 128 == 0 && (layout == CONVROT_LAYOUT_NK || n % 32 == 0);
}

// Rows up to which the default routing prefers this kernel to the CTA-pair
// one: measured on B200, it matches or beats the CTA-pair kernel at m <= 8
// (both are bound by per-stage hand-off latency there, and its K split fills
// more SMs), while from m = 16 the CTA-pair kernel is faster.  The default
// routing tries the GEMV kernel (gemv_w4a4.cu, 1.5-2.2x faster at m <= 8)
// before either, so this one serves route 3 and shapes the GEMV declines.
int small_m_auto_rows() { return 8; }

template <int LAYOUT, typename TOut>
static int launch_small_m_t(const int8_t* act, const small_m::Params& p0, cudaStream_t stream) {
  using namespace small_m;
  Params p = p0;
  CUtensorMap map_act, map_w;
  {
    // activations as (K / 128) x M rows x one 128-byte chunk; a box = 2 chunks x np rows
    const uint64_t dims[3] = {128, static_cast<uint64_t>(p.M), static_cast<uint64_t>(p.K) / 128};
    const uint64_t strides[2] = {static_cast<uint64_t>(p.K), 128};
    const uint32_t box[3] = {128, static_cast<uint32_t>(p.np), 2};
    int rc = w4a4::make_tmap_u8(&map_act, act, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_DATA_TYPE_UINT8);
    if (rc != CONVROT_OK) return rc;
  }
  {
    int rc;
    if (LAYOUT == CONVROT_LAYOUT_NK) {
      const uint64_t dims[2] = {static_cast<uint64_t>(p.K / 2), static_cast<uint64_t>(p.N)};
      const uint64_t strides[1] = {static_cast<uint64_t>(p.K / 2)};
      const uint32_t box[2] = {KS / 2, BN};
      rc = w4a4::make_tmap_u8(&map_w, p.qweight, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_DATA_TYPE_UINT8);
    } else {
      const uint64_t dims[2] = {static_cast<uint64_t>(p.N / 2), static_cast<uint64_t>(p.K)};
      const uint64_t strides[1] = {static_cast<uint64_t>(p.N / 2)};
      const uint32_t box[2] = {BN / 2, KS};
      rc = w4a4::make_tmap_u8(&map_w, p.qweight, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_DATA_TYPE_UINT8);
    }
    if (rc != CONVROT_OK) return rc;
  }
  auto kernel = small_m_kernel<LAYOUT, TOut>;
  p.sw = sw_slots(p.np);
  p.x = x_slots(p.np);
  const size_t smem = smem_bytes(p.np);
  CONVROT_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  const int n_tiles = (p.N + BN - 1) / BN;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(n_tiles * p.cluster), 1, 1);
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
  CONVROT_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, map_act, map_w, p));
  return check_launch("w4a4 small-m gemm");
}

// Called by convrot_w4a4_gemm after its argument checks, for shapes that
// small_m_supported accepts.
int launch_small_m(const int8_t* act, const uint8_t* qweight, int layout, const float* xscales, const float* wscales,
                   const float* bias, void* out, int out_dtype, int64_t m, int64_t n, int64_t k, cudaStream_t stream) {
  using namespace small_m;
  Params p;
  p.qweight = qweight;
  p.xscales = xscales;
  p.wscales = wscales;
  p.bias = bias;
  p.out = out;
  p.M = static_cast<int>(m);
  p.N = static_cast<int>(n);
  p.K = static_cast<int>(k);
  p.np = static_cast<int>((m + 15) / 16 * 16);
  p.k_stages = static_cast<int>((k + KS - 1) / KS);
  // split K over a cluster so that the tiles x ranks fill the SMs, at least
  // one K stage per rank
  const int n_tiles = static_cast<int>((n + BN - 1) / BN);
  int c = device_sm_count() / n_tiles;
  if (c > kMaxCluster) c = kMaxCluster;
  if (c > p.k_stages) c = p.k_stages;
  p.cluster = c < 1 ? 1 : c;
  p.err_word = device_error_word();
  CONVROT_REQUIRE(p.err_word != nullptr, CONVROT_ERR_CUDA, "device error word unavailable");
  if (layout == CONVROT_LAYOUT_NK) {
    switch (out_dtype) {
      case CONVROT_BF16: return launch_small_m_t<CONVROT_LAYOUT_NK, __nv_bfloat16>(act, p, stream);
      case CONVROT_F16: return launch_small_m_t<CONVROT_LAYOUT_NK, __half>(act, p, stream);
      default: return launch_small_m_t<CONVROT_LAYOUT_NK, float>(act, p, stream);
    }
  }
  switch (out_dtype) {
    case CONVROT_BF16: return launch_small_m_t<CONVROT_LAYOUT_KN, __nv_bfloat16>(act, p, stream);
    case CONVROT_F16: return launch_small_m_t<CONVROT_LAYOUT_KN, __half>(act, p, stream);
    default: return launch_small_m_t<CONVROT_LAYOUT_KN, float>(act, p, stream);
  }
}

}  // namespace convrot
