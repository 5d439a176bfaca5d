// W4A4 GEMM for sm_100a: int8 activation codes x packed signed-int4 weights on
// tcgen05 (kind::i8), int32 accumulators in TMEM, fused scale/bias epilogue.
//
// Replaces the reference's MPP TensorOp dot (core.py:839-874) plus its
// separate int32 -> scale/bias epilogue dispatch (core.py:925-937, 994-1011):
// here the int32 dots never leave the SM.
//
// Persistent kernel, one CTA per SM, tile 128 (M) x 256 (N) x 128 (K bytes):
//   warp 0      TMA producer: int8 activation tiles, 128-byte swizzle
//   warp 1      MMA issuer (one elected thread) + TMEM owner
//   warps 2-9   weight transform: 16-byte global loads of packed nibbles,
//               expanded to int8 in the canonical 128-byte-swizzled layout the
//               tensor core reads (K-major for the NK layout, MN-major for KN)
//   warps 10-13 epilogue: TMEM -> registers -> out = T(f32(dot) * xs * ws + b)
// Weight nibbles are expanded as 16 * w (the nibble moved to the high half of
// the byte: one AND, no sign extension), so the accumulator holds 16 * dot
// exactly; the epilogue shifts it back (|dot| <= 56 K stays far below 2^27).
// Two TMEM accumulators (2 x 256 columns) let the epilogue of tile i overlap
// the main loop of tile i + 1.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace convrot {

__device__ int g_convrot_device_error = 0;

int* device_error_word() {
  // per-device cache; host threads may race to fill a slot with the same
  // address, so the slots are atomic
  static std::atomic<int*> words[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  int* w = words[dev].load(std::memory_order_acquire);
  if (w == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_convrot_device_error) != cudaSuccess) return nullptr;
    w = static_cast<int*>(p);
    words[dev].store(w, std::memory_order_release);
  }
  return w;
}

namespace w4a4 {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;  // bytes of K per stage
constexpr int STAGES = 4;
constexpr int kWarpTma = 0;
constexpr int kWarpMma = 1;
constexpr int kWarpXform0 = 2;
constexpr int kXformWarps = 8;
constexpr int kWarpEpi0 = kWarpXform0 + kXformWarps;
constexpr int kEpiWarps = 4;
constexpr int kThreads = (kWarpEpi0 + kEpiWarps) * 32;  // 448
constexpr int kXformThreads = kXformWarps * 32;
constexpr int kItems = BN * BK / 32;  // 16 packed bytes -> 32 int8 per item
constexpr int kItemsPerThread = kItems / kXformThreads;  // 4
constexpr uint32_t kTmemCols = 2 * BN;
constexpr int kABytes = BM * BK;  // 16 KB
constexpr int kBBytes = BN * BK;  // 32 KB
constexpr uint64_t kTimeoutNs = 4000000000ull;  // a single wait never legitimately takes this long

struct alignas(8) Barriers {
  uint64_t a_full[STAGES];
  uint64_t b_full[STAGES];
  uint64_t empty[STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int err;
};

constexpr int kEpiBytes = kEpiWarps * 2 * BN * 4;  // ws and bias, one copy per epilogue warp
constexpr size_t kSmemBytes = 1024 /*alignment slack*/ + STAGES * (kABytes + kBBytes) + kEpiBytes + sizeof(Barriers);

constexpr int kMaxOuts = 8;

int forced_kernel();

struct Params {
  const uint8_t* qweight;
  const float* xscales;
  const float* wscales;
  const float* bias;
  void* out;
  int M, N, K;
  int m_tiles, n_tiles, k_blocks;
  int layout;
  // Extra destinations of the pair kernel's epilogue (tensor-parallel
  // all-gather): with n_outs > 0, element (m, n) goes to outs[i][m * ldc +
  // col_off + n] for every i (this GPU's buffer and peers' buffers mapped
  // into this GPU's address space), and `out` is unused.
  void* outs[kMaxOuts] = {};
  int n_outs = 0;
  int64_t ldc = 0;
  int64_t col_off = 0;
};

// Wait for the phase of `bar` with parity `parity` to complete, for at most
// kTimeoutNs.  On time-out record the error in shared memory and return false.
__device__ __noinline__ bool wait_bar(uint64_t* bar, uint32_t parity, Barriers* b, int code) {
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

// 16 packed bytes -> 32 int8 values of 16 * nibble, in element order.
__device__ __forceinline__ void expand16(const uint4 w, uint32_t (&o)[8]) {
  const uint32_t s[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t even = (s[j] << 4) & 0xF0F0F0F0u;  // elements 0,2,4,6 of this word
    const uint32_t odd = s[j] & 0xF0F0F0F0u;          // elements 1,3,5,7
    o[2 * j] = __byte_perm(even, odd, 0x5140);
    o[2 * j + 1] = __byte_perm(even, odd, 0x7362);
  }
}

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// Per-thread description of one transform item: 16 packed bytes (32 int4
// values) that become 32 int8 bytes in two 16-byte chunks of a B stage.
// Everything but the block origin (n0, k0) is fixed for the whole kernel.
struct Item {
  int a;          // NK: row n within the tile;   KN: row k within the block
  int b;          // NK: 32-k group q (0..3);     KN: 32-n group q (0..7)
  uint32_t s0;    // smem offsets of the two output chunks within a stage
  uint32_t s1;
};

template <int LAYOUT>
__device__ __forceinline__ Item make_item(int item) {
  Item it;
  if constexpr (LAYOUT == CONVROT_LAYOUT_NK) {
    // K-major 128-byte-swizzled tile: row n at n * 128, chunk c at (c ^ (n & 7)) * 16
    const int n = item >> 2, q = item & 3;
    it.a = n;
    it.b = q;
    const uint32_t row = n * 128;
    it.s0 = row + (((2 * q) ^ (n & 7)) << 4);
    it.s1 = row + (((2 * q + 1) ^ (n & 7)) << 4);
  } else {
    // MN-major 128-byte-swizzled tile: n-atoms of 128 columns (BK * 128 bytes
    // apart), each 8-row k-atoms of 1 KB; chunk c of row k at (c ^ (k & 7)) * 16.
    // Lanes 0-3 / 4-7 of a quarter-warp take two consecutive k rows so their
    // eight chunks fall on distinct banks.
    const int wi = item >> 5, lane = item & 31;
    const int kr = 4 * wi + ((lane >> 2) & 3);
    const int q = (lane & 3) + 4 * (lane >> 4);
    it.a = kr;
    it.b = q;
    const uint32_t base = (q >> 2) * (BK * 128) + (kr >> 3) * 1024 + (kr & 7) * 128;
    const int c = 2 * (q & 3);
    it.s0 = base + ((c ^ (kr & 7)) << 4);
    it.s1 = base + (((c + 1) ^ (kr & 7)) << 4);
  }
  return it;
}

// Load the 16 packed bytes of `it` for the block at (n0, k0); zero outside the weight.
template <int LAYOUT>
__device__ __forceinline__ uint4 load_item(const Params& p, const Item& it, int n0, int k0) {
  if constexpr (LAYOUT == CONVROT_LAYOUT_NK) {
    const int gn = n0 + it.a, gk = k0 + 32 * it.b;
    if (gn >= p.N || gk >= p.K) return make_uint4(0, 0, 0, 0);
    // K % 32 == 0: the row stride K / 2 and the offset gk / 2 are multiples of 16
    return __ldg(reinterpret_cast<const uint4*>(p.qweight + static_cast<int64_t>(gn) * (p.K >> 1) + (gk >> 1)));
  } else {
    const int gk = k0 + it.a, gn = n0 + 32 * it.b;
    if (gk >= p.K || gn >= p.N) return make_uint4(0, 0, 0, 0);
    const uint8_t* src = p.qweight + static_cast<int64_t>(gk) * (p.N >> 1) + (gn >> 1);
    // 16-byte loads need a row stride (N / 2 bytes) that is a multiple of 16;
    // then every item with gn < N also lies wholly inside the row.
    if ((p.N & 31) == 0) return __ldg(reinterpret_cast<const uint4*>(src));
    // ragged N: bytes one by one, zero past N (byte b holds columns gn + 2b, gn + 2b + 1)
    uint32_t w0 = 0, w1 = 0, w2 = 0, w3 = 0;
#pragma unroll
    for (int b = 0; b < 16; ++b) {
      const uint32_t v = (gn + 2 * b < p.N) ? static_cast<uint32_t>(src[b]) << (8 * (b & 3)) : 0u;
      if (b < 4) w0 |= v;
      else if (b < 8) w1 |= v;
      else if (b < 12) w2 |= v;
      else w3 |= v;
    }
    return make_uint4(w0, w1, w2, w3);
  }
}

template <int LAYOUT>
__device__ __forceinline__ void load_block(const Params& p, const Item (&it)[kItemsPerThread], int tile, int kb,
                                           uint4 (&dst)[kItemsPerThread]) {
  const int n0 = (tile / p.m_tiles) * BN, k0 = kb * BK;
#pragma unroll
  for (int i = 0; i < kItemsPerThread; ++i) dst[i] = load_item<LAYOUT>(p, it[i], n0, k0);
}

// 16 consecutive outputs with 16-byte stores (pointer 16-byte aligned).
__device__ __forceinline__ void store16(float* dst, const float (&v)[32], int o) {
#pragma unroll
  for (int q = 0; q < 4; ++q)
    reinterpret_cast<float4*>(dst)[q] = make_float4(v[o + 4 * q], v[o + 4 * q + 1], v[o + 4 * q + 2], v[o + 4 * q + 3]);
}

// Two outputs rounded to nearest even (as cvt_out) in one paired conversion,
// a in the low half.
template <typename T16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (std::is_same<T16, __nv_bfloat16>::value) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}

template <typename T16>
__device__ __forceinline__ void store16(T16* dst, const float (&v)[32], int o) {
#pragma unroll
  for (int q = 0; q < 2; ++q)
    reinterpret_cast<uint4*>(dst)[q] =
        make_uint4(pack2<T16>(v[o + 8 * q], v[o + 8 * q + 1]), pack2<T16>(v[o + 8 * q + 2], v[o + 8 * q + 3]),
                   pack2<T16>(v[o + 8 * q + 4], v[o + 8 * q + 5]), pack2<T16>(v[o + 8 * q + 6], v[o + 8 * q + 7]));
}

template <int LAYOUT, typename TOut>
__global__ void __launch_bounds__(kThreads, 1)
    w4a4_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * kABytes;
  float* epi_ws = reinterpret_cast<float*>(sB + STAGES * kBBytes);
  Barriers* bars = reinterpret_cast<Barriers*>(sB + STAGES * kBBytes + kEpiBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = p.m_tiles * p.n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->a_full[s], 1);
      mbar_init(&bars->b_full[s], kXformWarps);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->acc_full[b], 1);
      mbar_init(&bars->acc_empty[b], kEpiWarps);
    }
    mbar_init(&bars->mma_done, 1);
    bars->err = 0;
    fence_mbar_init();
    prefetch_tensormap(&tmap_a);
  }
  if (warp == kWarpMma) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp == kWarpTma) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m_blk = tile % p.m_tiles;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!wait_bar(&bars->empty[stage], phase ^ 1, bars, 1)) { ok = false; break; }
          mbar_arrive_expect_tx(&bars->a_full[stage], kABytes);
          tma_load_2d(sA + stage * kABytes, &tmap_a, &bars->a_full[stage], kb * BK, m_blk * BM);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        // error exit: let the (at most STAGES) copies still in flight land
        for (int j = 0; j < STAGES && j < issued; ++j) {
          if (--stage < 0) { stage = STAGES - 1; phase ^= 1; }
          wait_bar(&bars->a_full[stage], phase, bars, 1);
        }
      }
    }
  } else if (warp == kWarpMma) {
    if (lane == 0) {
      // idesc: D s32 (bits 4-5 = 2), A s8 (bits 7-9 = 1), B s8 (bits 10-12 = 1),
      // A K-major, B K-major (NK) or MN-major (KN), N >> 3 at bit 17, M >> 4 at bit 24.
      const uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) |
                             (static_cast<uint32_t>(LAYOUT == CONVROT_LAYOUT_KN) << 16) |
                             (static_cast<uint32_t>(BN >> 3) << 17) | (static_cast<uint32_t>(BM >> 4) << 24);
      const uint32_t a_base = smem_u32(sA), b_base = smem_u32(sB);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
        const int buf = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!wait_bar(&bars->acc_empty[buf], acc_phase ^ 1, bars, 2)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!wait_bar(&bars->a_full[stage], phase, bars, 3)) { ok = false; break; }
          if (!wait_bar(&bars->b_full[stage], phase, bars, 4)) { ok = false; break; }
          tc_fence_after();
          const int k_rem = p.K - kb * BK;
          const int ksteps = k_rem >= BK ? BK / 32 : k_rem / 32;
          const uint32_t a_addr = a_base + stage * kABytes;
          const uint32_t b_addr = b_base + stage * kBBytes;
          for (int ks = 0; ks < ksteps; ++ks) {
            const uint64_t adesc = smem_desc(a_addr + ks * 32, 16, 1024, 2);
            const uint64_t bdesc = LAYOUT == CONVROT_LAYOUT_NK ? smem_desc(b_addr + ks * 32, 16, 1024, 2)
                                                               : smem_desc(b_addr + ks * 4096, BK * 128, 1024, 2);
            mma_i8(d_tmem, adesc, bdesc, idesc, (kb | ks) != 0 ? 1u : 0u);
          }
          mma_commit(&bars->empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        mma_commit(&bars->acc_full[buf]);
      }
      // every MMA issued above must finish before TMEM is released
      mma_commit(&bars->mma_done);
      wait_bar(&bars->mma_done, 0, bars, 5);
    }
  } else if (warp < kWarpEpi0) {
    // ---------------- weight transform ----------------
    // Blocks (tile, kb) in this CTA's order; registers hold the packed bytes of
    // the current block and the two after it, so global latency is covered by
    // two blocks of tensor-core work.
    const int xt = threadIdx.x - kWarpXform0 * 32;
    Item it[kItemsPerThread];
#pragma unroll
    for (int i = 0; i < kItemsPerThread; ++i) it[i] = make_item<LAYOUT>(i * kXformThreads + xt);
    int stage = 0;
    uint32_t phase = 0;
    uint4 b0[kItemsPerThread], b1[kItemsPerThread], b2[kItemsPerThread];
    int t0 = blockIdx.x, k0 = 0;         // block being written
    int t1 = t0, k1 = 0, t2 = t0, k2 = 0;  // the next two blocks
    auto advance = [&](int& t, int& k) {
      if (++k == p.k_blocks) { k = 0; t += gridDim.x; }
    };
    t1 = t0; k1 = k0; advance(t1, k1);
    t2 = t1; k2 = k1; advance(t2, k2);
    if (t0 < num_tiles) load_block<LAYOUT>(p, it, t0, k0, b0);
    if (t1 < num_tiles) load_block<LAYOUT>(p, it, t1, k1, b1);
    while (t0 < num_tiles) {
      if (t2 < num_tiles) load_block<LAYOUT>(p, it, t2, k2, b2);
      if (!wait_bar(&bars->empty[stage], phase ^ 1, bars, 6)) break;
      const uint32_t b_addr = smem_u32(sB + stage * kBBytes);
#pragma unroll
      for (int i = 0; i < kItemsPerThread; ++i) {
        uint32_t o[8];
        expand16(b0[i], o);
        sts128(b_addr + it[i].s0, o[0], o[1], o[2], o[3]);
        sts128(b_addr + it[i].s1, o[4], o[5], o[6], o[7]);
      }
      fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->b_full[stage]);
      if (++stage == STAGES) { stage = 0; phase ^= 1; }
#pragma unroll
      for (int i = 0; i < kItemsPerThread; ++i) {
        b0[i] = b1[i];
        b1[i] = b2[i];
      }
      t0 = t1; k0 = k1;
      t1 = t2; k1 = k2;
      advance(t2, k2);
    }
  } else {
    // ---------------- epilogue ----------------
    // Each epilogue warp stages the tile columns' weight scales and bias in its
    // own shared-memory slice (only warp-level synchronization, so a warp that
    // stops early on an error can never strand the others); each thread owns
    // one output row and reads 32 accumulator columns per tcgen05.ld.
    const int ew = warp & 3;  // TMEM lane quarter this warp may access
    float* sws = epi_ws + ew * 2 * BN;
    float* sbias = sws + BN;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int buf = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      const int m_blk = tile % p.m_tiles, n_blk = tile / p.m_tiles;
      __syncwarp();  // the previous tile's reads of sws / sbias are done
      for (int j = lane; j < BN; j += 32) {
        const int col = n_blk * BN + j;
        sws[j] = col < p.N ? __ldg(p.wscales + col) : 0.0f;
        sbias[j] = (col < p.N && p.bias) ? __ldg(p.bias + col) : 0.0f;
      }
      __syncwarp();
      if (!wait_bar(&bars->acc_full[buf], acc_phase, bars, 7)) break;
      tc_fence_after();
      const int m = m_blk * BM + ew * 32 + lane;
      const bool row_ok = m < p.M;
      const float xs = row_ok ? __ldg(p.xscales + m) : 0.0f;
      TOut* orow = static_cast<TOut*>(p.out) + static_cast<int64_t>(row_ok ? m : 0) * p.N;
      const bool vec_store = (p.N % (16 / sizeof(TOut))) == 0;
      const uint32_t t_row = tmem_base + ((ew * 32u) << 16) + buf * BN;
      for (int c = 0; c < BN / 32; ++c) {
        const int n = n_blk * BN + c * 32;
        if (n >= p.N) break;  // uniform across the warp
        uint32_t r[32];
        __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp, converged
        tmem_ld_32x32b_x32(t_row + c * 32, r);
        tmem_ld_wait();
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 w4 = *reinterpret_cast<const float4*>(sws + c * 32 + j);
          const float4 b4 = *reinterpret_cast<const float4*>(sbias + c * 32 + j);
          const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
          const float bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            // accumulator = 16 * dot exactly; dot * xs * ws + bias, each step rounded
            const float dot = static_cast<float>(static_cast<int32_t>(r[j + u]) >> 4);
            v[j + u] = __fadd_rn(__fmul_rn(__fmul_rn(dot, xs), wv[u]), bv[u]);
          }
        }
        if (!row_ok) continue;
        if (vec_store && n + 32 <= p.N) {
          store16(orow + n, v, 0);
          store16(orow + n + 16, v, 16);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n + j < p.N) orow[n + j] = cvt_out<TOut>(v[j]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acc_empty[buf]);
    }
  }

  __syncwarp();  // roles above ran on single lanes: reconverge before the block barrier
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kWarpMma) {
    __syncwarp();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0 && bars->err) atomicCAS(&g_convrot_device_error, 0, bars->err);
}

// ===========================================================================
// CTA-pair kernel (cta_group::2): pair tile 256 (M) x 256 (N), 256 K-bytes per
// stage.  Each CTA of the pair owns 128 rows of A and 128 columns of B:
//   warp 0    A producer: lane s owns slot s of the 3-slot ring and issues
//             one 32 KB 3-D TMA box (two 128-byte K chunks) per stage into
//             this CTA, completing on the pair leader's a_full.  Copies
//             issued by one thread are served one after another, hence one
//             issuing lane per slot.
//   warp 1    leader: MMA issuer (tcgen05.mma.cta_group::2, M = 256); both
//             CTAs: TMEM allocation for the pair
//   warp 2    packed-weight producer: lane s owns slot s; one 16 KB TMA box
//             per stage (this CTA's 128 columns x 256 K) on this CTA's bp_full
//   warps 3, 4, 6, 7  transform: packed nibbles (shared) -> int8 x 16 in the
//             128-byte-swizzled layout the tensor core reads, into a 2-slot
//             ring.  The leader's warps arrive on its b8_ready; the peer's
//             warps each bulk-copy a 16-byte token into the leader, completing
//             bytes on that barrier (a copy-engine signal).
//   warp 5    idle, so that the MMA issuer has its scheduler to itself
//   warps 8-11 epilogue: this CTA's 128 accumulator rows x 256 columns
// The leader's commits are multicast to both CTAs (stage release, int8-slot
// release, accumulator ready); the peer's epilogue warps arrive on the
// leader's acc_empty through cluster addresses.  Per SM this halves the
// weight bytes and the transform work of the one-CTA kernel for the same
// tensor-core rate, and every operand arrives by TMA.
// ===========================================================================
// W4A4 epilogue of one 32-column chunk: v[j] = fl(fl(fl(dot_j) * xs) * ws_j)
// + bias_j (core.py:932-936).  The accumulator holds 16 * dot exactly.  With
// kDiv16 the caller passes xs / 16, exact because it is still a normal float
// (or zero, infinite, NaN): then fl(float(acc) * xs / 16) == fl(fl(dot) * xs)
// -- float(acc) = 16 * fl(dot) and the power-of-two factor cancels exactly --
// and the shift is saved.  The two products are paired fp32 multiplies
// (mul2_rn, rounded per component as __fmul_rn); the bias add stays scalar
// __fadd_rn, because a paired add right after a paired multiply was fused
// into one rounding by the compiler even with .rn spelled out.
template <bool kDiv16>
__device__ __forceinline__ void scale_chunk_i8(const uint32_t (&r)[32], const float* ws, const float* bias, float xs,
                                               float (&v)[32]) {
  const float2 xs2 = make_float2(xs, xs);
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    const float4 w4 = *reinterpret_cast<const float4*>(ws + j);
    const float4 b4 = *reinterpret_cast<const float4*>(bias + j);
    float2 d[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int32_t a0 = static_cast<int32_t>(r[j + 2 * h]), a1 = static_cast<int32_t>(r[j + 2 * h + 1]);
      d[h] = kDiv16 ? make_float2(__int2float_rn(a0), __int2float_rn(a1))
                    : make_float2(__int2float_rn(a0 >> 4), __int2float_rn(a1 >> 4));
    }
    const float2 p0 = mul2_rn(mul2_rn(d[0], xs2), make_float2(w4.x, w4.y));
    const float2 p1 = mul2_rn(mul2_rn(d[1], xs2), make_float2(w4.z, w4.w));
    v[j] = __fadd_rn(p0.x, b4.x);
    v[j + 1] = __fadd_rn(p0.y, b4.y);
    v[j + 2] = __fadd_rn(p1.x, b4.z);
    v[j + 3] = __fadd_rn(p1.y, b4.w);
  }
}

namespace pair {

constexpr int BM = 256;          // rows per pair tile (128 per CTA)
constexpr int BN = 256;          // columns per pair tile (128 per CTA)
constexpr int BK = 256;          // K bytes per stage
constexpr int S = 3;             // TMA stages (A + packed B)
constexpr int B8 = 2;            // int8 weight slots
// Warp w runs on scheduler w % 4.  The MMA issuer (warp 1) shares its
// scheduler with no transform warp: warp 5 idles, the transform warps are
// 3, 4, 6 and 7, the epilogue warps 8-11 (warp w reads TMEM lanes
// 32 * (w % 4) .. + 31).
constexpr int kWarpA = 0, kWarpMma = 1, kWarpBp = 2, kWarpX0 = 3, kXWarps = 4, kWarpIdle = 5, kWarpE0 = 8,
              kEWarps = 4;
constexpr int kThreads = (kWarpE0 + kEWarps) * 32;  // 384
constexpr int kXThreads = kXWarps * 32;
constexpr int kABytes = 128 * BK;         // 32 KB per CTA per stage
constexpr int kBpBytes = 128 * BK / 2;    // 16 KB
constexpr int kB8Bytes = 128 * BK;        // 32 KB
constexpr int kItems = kBpBytes / 16;     // 1024 transform items per stage
constexpr int kItemsPerThread = kItems / kXThreads;  // 8
constexpr int kEpiBytes = kEWarps * 2 * BN * 4;
constexpr int kStageOutBytes = kEWarps * 32 * 64;  // per epilogue warp: 32 rows x 32 16-bit columns
constexpr uint32_t kTmemCols = 2 * BN;

// Operand kinds.  KIND_I8: A4 int8 codes x nibbles expanded to int8 x 16
// (kind::i8, int32 accumulate; W4A4).  KIND_BF16 / KIND_F16: rotated 16-bit
// activations x nibbles expanded to exact 16-bit integers (kind::f16, fp32
// accumulate; W4A16).  A stage is 256 bytes of A's K extent either way.
constexpr int KIND_I8 = 0, KIND_BF16 = 1, KIND_F16 = 2;
template <int KIND> constexpr int kKStage = KIND == KIND_I8 ? 256 : 128;  // K per stage
template <int KIND> constexpr int kKStep = KIND == KIND_I8 ? 32 : 16;     // K per MMA
template <int KIND> constexpr int kBpStage = 128 * kKStage<KIND> / 2;     // packed bytes per CTA per stage

struct alignas(16) Bars {
  // The peer's transform warps signal the leader's b8_ready by copying a
  // 16-byte token each into tok (a bulk copy completing bytes on b8_ready):
  // copy-engine signals reach the leader much sooner than remote arrives.
  uint8_t tok[B8][kXWarps][16];
  uint8_t tok_src[16];
  uint64_t a_full[S];
  uint64_t bp_full[S];
  uint64_t tma_empty[S];
  uint64_t b8_ready[B8];
  uint64_t b8_empty[B8];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int err;
};

constexpr size_t kSmemBytes =
    1024 + S * (kABytes + kBpBytes) + B8 * kB8Bytes + kEpiBytes + kStageOutBytes + sizeof(Bars);
static_assert(kSmemBytes <= 232448, "shared memory budget");

// Named barriers 1-4: the epilogue warp of TMEM lane quarter q hands the last
// tile's staged scales to helper warp 4 + q (64 threads each).
constexpr int kHelpBar0 = 1;
__device__ __forceinline__ void named_bar_arrive(int id, int threads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Waits use cluster-scope acquire: most barriers of the pair kernel receive
// arrivals from the other CTA.
__device__ __noinline__ bool wait(uint64_t* bar, uint32_t parity, Bars* b, int code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & 255) == 0) {
      if (*reinterpret_cast<volatile int*>(&b->err)) return false;
      if (globaltimer() - t0 > kTimeoutNs) {
        atomicCAS(&b->err, 0, code);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void settle_after_error(bool ok) {
  // after an error, give an asynchronous copy still in flight 2 ms to land
  if (!ok) {
    const uint64_t t0 = globaltimer();
    while (globaltimer() - t0 < 2000000ull) {
    }
  }
}

// Four packed words (32 nibbles) -> 32 exact 16-bit integers in 4 chunks of
// 16 bytes.  The biased nibble u = nibble ^ 8 goes into the low mantissa bits
// of 128.0 (bf16, 0x4300) or 1024.0 (fp16, 0x6400), whose ulp is 1; one
// packed subtraction of 136 / 1032 then leaves the signed value exactly.
template <int KIND>
__device__ __forceinline__ void expand16_to_16bit(const uint4 w, uint32_t (&o)[16]) {
  const uint32_t in[4] = {w.x, w.y, w.z, w.w};
  constexpr uint32_t kBase = KIND == KIND_BF16 ? 0x43004300u : 0x64006400u;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t y = in[q] ^ 0x88888888u;
    const uint32_t lo = y & 0x0F0F0F0Fu, hi = (y >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const uint32_t v = (__byte_perm(lo, hi, t | ((4 + t) << 8)) & 0x00FF00FFu) | kBase;
      if constexpr (KIND == KIND_BF16) {
        const __nv_bfloat162 r = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&v), __float2bfloat162_rn(136.0f));
        o[4 * q + t] = *reinterpret_cast<const uint32_t*>(&r);
      } else {
        const __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&v), __float2half2_rn(1032.0f));
        o[4 * q + t] = *reinterpret_cast<const uint32_t*>(&r);
      }
    }
  }
}

template <int LAYOUT, typename TOut, int KIND = KIND_I8>
__global__ void __launch_bounds__(kThreads, 1)
    pair_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                     const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                                   // S x 32 KB
  uint8_t* sB8 = sA + S * kABytes;                      // B8 x 32 KB
  uint8_t* sBp = sB8 + B8 * kB8Bytes;                   // S x 16 KB
  float* epi = reinterpret_cast<float*>(sBp + S * kBpBytes);
  uint8_t* stage_out = reinterpret_cast<uint8_t*>(epi) + kEpiBytes;  // gather path: row-major restaging
  Bars* bars = reinterpret_cast<Bars*>(stage_out + kStageOutBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = leader
  const int pair_id = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  const int num_tiles = p.m_tiles * p.n_tiles;
  constexpr int KS = kKStage<KIND>;
  const int k_stages = (p.K + KS - 1) / KS;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&bars->a_full[s], 1);
      mbar_init(&bars->bp_full[s], 1);
      mbar_init(&bars->tma_empty[s], 1);
    }
    for (int s = 0; s < B8; ++s) {
      mbar_init(&bars->b8_ready[s], kXWarps);  // the leader's warps; the peer's arrive as bytes
      mbar_init(&bars->b8_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->acc_full[b], 1);
      mbar_init(&bars->acc_empty[b], 2 * kEWarps);
    }
    mbar_init(&bars->mma_done, 1);
    bars->err = 0;
    fence_mbar_init();
    prefetch_tensormap(&tmap_a);
    prefetch_tensormap(&tmap_b);
  }
  if (warp == kWarpMma) {
    tmem_alloc_pair(&bars->tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialized before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;
  // Everything above touches only shared memory, TMEM and kernel parameters,
  // so it overlaps the previous kernel's tail; global memory comes after.
  grid_dependency_wait();
  grid_dependents_launch();

  // Epilogue of one tile for TMEM lane quarter `quarter` (rows quarter * 32 ..
  // + 31 of this CTA's half), 32-column chunks [c_begin, c_end): waits for
  // the accumulator, then scales, converts and stores.  sws / sbias: the
  // tile's column scales and bias; stage_base: this warp's 2 KB of shared
  // memory for restaging 16-bit outputs.  False when the wait failed.
  auto epi_chunks = [&](int tile, int local, int quarter, int c_begin, int c_end, const float* sws,
                        const float* sbias, uint32_t stage_base) -> bool {
      const int buf = local & 1;
      const int m_blk = tile % p.m_tiles, n_blk = tile / p.m_tiles;
      const int m = m_blk * BM + 128 * rank + quarter * 32 + lane;
      const bool row_ok = m < p.M;
      // the row scale is loaded before the wait, off the tile's critical path
      const float xs = (KIND == KIND_I8 && row_ok) ? __ldg(p.xscales + m) : 0.0f;
      const bool xs_div16 = __all_sync(0xFFFFFFFFu, !(fabsf(xs) < 0x1p-122f) || xs == 0.0f);  // xs / 16 exact
      __syncwarp();
      if (!wait(&bars->acc_full[buf], (local >> 1) & 1, bars, 19)) return false;
      tc_fence_after();
      const bool gather = p.n_outs > 0;
      const int64_t ldc = gather ? p.ldc : p.N;
      const int64_t row_off = static_cast<int64_t>(row_ok ? m : 0) * ldc + (gather ? p.col_off : 0);
      TOut* orow = static_cast<TOut*>(p.out) + row_off;
      const bool vec_store = ((gather ? (ldc | p.col_off) : p.N) % (16 / sizeof(TOut))) == 0;
      const uint32_t t_row = tmem_base + ((static_cast<uint32_t>(quarter) * 32u) << 16) + buf * BN;
      for (int c = c_begin; c < c_end; ++c) {
        const int n = n_blk * BN + c * 32;
        if (n >= p.N) break;  // uniform across the warp
        uint32_t r[32];
        __syncwarp();
        tmem_ld_32x32b_x32(t_row + c * 32, r);
        tmem_ld_wait();
        float v[32];
        if constexpr (KIND == KIND_I8) {
          if (xs_div16) scale_chunk_i8<true>(r, sws + c * 32, sbias + c * 32, xs * 0.0625f, v);
          else scale_chunk_i8<false>(r, sws + c * 32, sbias + c * 32, xs, v);
        } else {
#pragma unroll
          for (int j = 0; j < 32; j += 4) {  // core.py:1145-1152: fl(dots * ws) + bias, fp32 dots
            const float4 w4 = *reinterpret_cast<const float4*>(sws + c * 32 + j);
            const float4 b4 = *reinterpret_cast<const float4*>(sbias + c * 32 + j);
            const float2 p0 = mul2_rn(make_float2(__uint_as_float(r[j]), __uint_as_float(r[j + 1])), make_float2(w4.x, w4.y));
            const float2 p1 = mul2_rn(make_float2(__uint_as_float(r[j + 2]), __uint_as_float(r[j + 3])), make_float2(w4.z, w4.w));
            v[j] = __fadd_rn(p0.x, b4.x);  // scalar add: see scale_chunk_i8
            v[j + 1] = __fadd_rn(p0.y, b4.y);
            v[j + 2] = __fadd_rn(p1.x, b4.z);
            v[j + 3] = __fadd_rn(p1.y, b4.w);
          }
        }
        if constexpr (sizeof(TOut) == 2) {
          if (vec_store && n + 32 <= p.N) {  // warp-uniform; every lane takes part
            // lane = row would give 32 scattered 16-byte pieces per store
            // instruction (NVLink carries those badly, L2 merges them at a
            // cost).  Restage the warp's
            // 32 x 32 chunk in shared memory (16-byte chunk q of row r at
            // ((q + r / 2) % 4) -- conflict-free both ways) and store it with
            // four lanes per row: 64 contiguous bytes per row, 8 rows per
            // instruction.
            const uint32_t sb = stage_base;
            __syncwarp();
#pragma unroll
            for (int q = 0; q < 4; ++q)
              sts128(sb + lane * 64 + (((q + (lane >> 1)) & 3) << 4), pack2<TOut>(v[8 * q], v[8 * q + 1]),
                     pack2<TOut>(v[8 * q + 2], v[8 * q + 3]), pack2<TOut>(v[8 * q + 4], v[8 * q + 5]),
                     pack2<TOut>(v[8 * q + 6], v[8 * q + 7]));
            __syncwarp();
            uint4 piece[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int r = i * 8 + (lane >> 2), q = lane & 3;
              const uint32_t a = sb + r * 64 + (((q + (r >> 1)) & 3) << 4);
              asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                           : "=r"(piece[i].x), "=r"(piece[i].y), "=r"(piece[i].z), "=r"(piece[i].w)
                           : "r"(a));
            }
            const int64_t row0 = static_cast<int64_t>(m_blk * BM + 128 * rank + quarter * 32);
            const int n_dst = gather ? p.n_outs : 1;
#pragma unroll 1
            for (int d = 0; d < n_dst; ++d) {
              TOut* base = static_cast<TOut*>(gather ? p.outs[d] : p.out) + (gather ? p.col_off : 0) + n +
                           (lane & 3) * 8;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int64_t r = row0 + i * 8 + (lane >> 2);
                if (r < p.M) *reinterpret_cast<uint4*>(base + r * ldc) = piece[i];
              }
            }
            continue;
          }
        }
        if (!row_ok) continue;
        if (gather) {
          // this tile's columns into every destination (peers over NVLink)
#pragma unroll 1
          for (int d = 0; d < p.n_outs; ++d) {
            TOut* drow = static_cast<TOut*>(p.outs[d]) + row_off;
            if (vec_store && n + 32 <= p.N) {
              store16(drow + n, v, 0);
              store16(drow + n + 16, v, 16);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (n + j < p.N) drow[n + j] = cvt_out<TOut>(v[j]);
            }
          }
        } else if (vec_store && n + 32 <= p.N) {
          store16(orow + n, v, 0);
          store16(orow + n + 16, v, 16);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n + j < p.N) orow[n + j] = cvt_out<TOut>(v[j]);
        }
      }
      return true;
  };


  if (warp == kWarpA) {
    // Lane s issues the copies of slot s: copies issued by one thread are
    // served one after another, so one issuing lane per slot keeps S copies
    // in flight.
    if (lane < S) {
      const uint32_t lead_a_full0 = mapa_shared(&bars->a_full[0], 0);
      int g = 0;
      bool ok = true;
      for (int tile = pair_id; tile < num_tiles && ok; tile += num_pairs) {
        const int m_row = (tile % p.m_tiles) * BM + 128 * rank;
        for (int ks = 0; ks < k_stages; ++ks, ++g) {
          const int slot = g % S;
          if (slot != lane) continue;
          if (!wait(&bars->tma_empty[slot], ((g / S) & 1) ^ 1, bars, 11)) { ok = false; break; }
          if (rank == 0) mbar_arrive_expect_tx(&bars->a_full[slot], 2 * kABytes);
          tma_load_3d_pair(sA + slot * kABytes, &tmap_a, lead_a_full0 + slot * 8, 0, m_row, 2 * ks);
        }
      }
      // Copies complete on the leader's barrier, which this thread cannot poll
      // in the peer CTA: after an error, give any copy still in flight 2 ms to
      // land before the pair tears down.
      if (!ok) {
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 2000000ull) {
        }
      }
    }
  } else if (warp == kWarpBp) {
    if (lane < S) {  // one issuing lane per slot, as for A
      int g = 0;
      bool ok = true;
      for (int tile = pair_id; tile < num_tiles && ok; tile += num_pairs) {
        const int n_col = (tile / p.m_tiles) * BN + 128 * rank;
        for (int ks = 0; ks < k_stages; ++ks, ++g) {
          const int slot = g % S;
          if (slot != lane) continue;
          if (!wait(&bars->tma_empty[slot], ((g / S) & 1) ^ 1, bars, 12)) { ok = false; break; }
          mbar_arrive_expect_tx(&bars->bp_full[slot], kBpStage<KIND>);
          if constexpr (LAYOUT == CONVROT_LAYOUT_NK)
            tma_load_2d(sBp + slot * kBpBytes, &tmap_b, &bars->bp_full[slot], ks * (KS / 2), n_col);
          else
            tma_load_2d(sBp + slot * kBpBytes, &tmap_b, &bars->bp_full[slot], n_col / 2, ks * KS);
        }
      }
      // after an error, give a copy still in flight 2 ms to land before teardown
      if (!ok) {
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 2000000ull) {
        }
      }
    }
  } else if (warp == kWarpMma) {
    if (rank == 0 && lane == 0) {
      // D format (s32 / f32), A and B formats (s8 / bf16 / f16), B major, N, M
      constexpr uint32_t kFormats = KIND == KIND_I8     ? (2u << 4) | (1u << 7) | (1u << 10)
                                    : KIND == KIND_BF16 ? (1u << 4) | (1u << 7) | (1u << 10)
                                                        : (1u << 4);
      const uint32_t idesc = kFormats | (static_cast<uint32_t>(LAYOUT == CONVROT_LAYOUT_KN) << 16) |
                             (static_cast<uint32_t>(BN >> 3) << 17) | (static_cast<uint32_t>(BM >> 4) << 24);
      const uint32_t a_base = smem_u32(sA), b_base = smem_u32(sB8);
      int g = 0, local = 0;
      bool ok = true;
      for (int tile = pair_id; tile < num_tiles && ok; tile += num_pairs, ++local) {
        const int buf = local & 1;
        if (!wait(&bars->acc_empty[buf], ((local >> 1) & 1) ^ 1, bars, 13)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int ks = 0; ks < k_stages; ++ks, ++g) {
          const int slot = g % S, b8 = g % B8;
          if (!wait(&bars->a_full[slot], (g / S) & 1, bars, 14)) { ok = false; break; }
          if (!wait(&bars->b8_ready[b8], (g / B8) & 1, bars, 15)) { ok = false; break; }
          tc_fence_after();
          const int k_rem = p.K - ks * KS;
          const int steps = k_rem >= KS ? KS / kKStep<KIND> : k_rem / kKStep<KIND>;
          const uint32_t a_addr = a_base + slot * kABytes;
          const uint32_t b_addr = b_base + b8 * kB8Bytes;
          for (int j = 0; j < steps; ++j) {
            const uint32_t a_off = (j >> 2) * 16384 + (j & 3) * 32;
            const uint64_t adesc = smem_desc(a_addr + a_off, 16, 1024, 2);
            // B: K-major (NK) like A; MN-major (KN): K step = 32 (int8) or 16
            // (16-bit) rows of 128 bytes; 16-bit tiles hold two 64-column
            // atoms 16 KB apart (the leading byte offset)
            const uint64_t bdesc = LAYOUT == CONVROT_LAYOUT_NK
                                       ? smem_desc(b_addr + a_off, 16, 1024, 2)
                                       : (KIND == KIND_I8 ? smem_desc(b_addr + j * 4096, kB8Bytes, 1024, 2)
                                                          : smem_desc(b_addr + j * 2048, 16384, 1024, 2));
            if constexpr (KIND == KIND_I8)
              mma_i8_pair(d_tmem, adesc, bdesc, idesc, (ks | j) != 0 ? 1u : 0u);
            else
              mma_f16_pair(d_tmem, adesc, bdesc, idesc, (ks | j) != 0 ? 1u : 0u);
          }
          mma_commit_pair_multicast(&bars->tma_empty[slot], 0x3);
          mma_commit_pair_multicast(&bars->b8_empty[b8], 0x3);
        }
        if (!ok) break;
        mma_commit_pair_multicast(&bars->acc_full[buf], 0x3);
      }
      // every MMA issued above finishes before the pair's TMEM is released
      mma_commit_pair_multicast(&bars->mma_done, 0x1);
      wait(&bars->mma_done, 0, bars, 16);
    }
  } else if (warp == kWarpIdle) {
  } else if (warp < kWarpE0) {
    // ---------------- transform ----------------
    const int xw = warp < kWarpIdle ? warp - kWarpX0 : warp - kWarpX0 - 1;  // 0..3
    const int xt = xw * 32 + lane;
    const uint32_t lead_ready0 = mapa_shared(&bars->b8_ready[0], 0);
    const uint32_t lead_tok0 = mapa_shared(&bars->tok[0][0][0], 0);
    auto publish = [&](int b8) {
      fence_proxy_async_smem();  // generic stores -> the pair MMA (async proxy)
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) {
          // the leader's warp 0 also announces the peer's token bytes
          if (xw == 0) mbar_arrive_expect_tx(&bars->b8_ready[b8], kXWarps * 16);
          else mbar_arrive(&bars->b8_ready[b8]);
        } else {
          bulk_copy_to_peer(lead_tok0 + (b8 * kXWarps + xw) * 16, bars->tok_src, 16, lead_ready0 + b8 * 8);
        }
      }
    };
    bool ok = true;
    if constexpr (KIND == KIND_I8) {
    // per-item fixed geometry: packed source offset and the two int8 chunks
    uint32_t src[kItemsPerThread], d0[kItemsPerThread], d1[kItemsPerThread];
#pragma unroll
    for (int i = 0; i < kItemsPerThread; ++i) {
      const int item = i * kXThreads + xt;
      if constexpr (LAYOUT == CONVROT_LAYOUT_NK) {
        // packed row n (128 bytes = 256 K values), chunk c (32 K values) ->
        // int8 K-chunk kc = c / 4, chunks 2j and 2j + 1 (j = c % 4) of row n.
        // A quarter-warp takes rows 2p and 2p + 1 with opposite K-chunks: its
        // loads cover both halves of the bank space and its stores land on
        // chunk sets of opposite row parity -- eight distinct bank groups.
        const int qw = item >> 3, l = item & 7, h = qw & 1;
        const int n = 2 * (qw >> 1) + (l >> 2);
        const int c = (l & 3) + 4 * ((l >> 2) ^ h);
        const int kc = c >> 2, j = c & 3;
        src[i] = n * 128 + c * 16;
        const uint32_t row = kc * 16384 + n * 128;
        d0[i] = row + (((2 * j) ^ (n & 7)) << 4);
        d1[i] = row + (((2 * j + 1) ^ (n & 7)) << 4);
      } else {
        // packed row k (64 bytes = 128 N values), chunk c -> MN-major int8 row k
        const int k = item >> 2, c = item & 3;
        src[i] = k * 64 + c * 16;
        const uint32_t row = (k >> 3) * 1024 + (k & 7) * 128;
        d0[i] = row + (((2 * c) ^ (k & 7)) << 4);
        d1[i] = row + (((2 * c + 1) ^ (k & 7)) << 4);
      }
    }
    int g = 0;
    for (int tile = pair_id; tile < num_tiles && ok; tile += num_pairs) {
      for (int ks = 0; ks < k_stages; ++ks, ++g) {
        const int slot = g % S, b8 = g % B8;
        if (!wait(&bars->bp_full[slot], (g / S) & 1, bars, 17)) { ok = false; break; }
        uint4 w[kItemsPerThread];
        const uint8_t* bp = sBp + slot * kBpBytes;
#pragma unroll
        for (int i = 0; i < kItemsPerThread; ++i) w[i] = *reinterpret_cast<const uint4*>(bp + src[i]);
        if (!wait(&bars->b8_empty[b8], ((g / B8) & 1) ^ 1, bars, 18)) { ok = false; break; }
        const uint32_t dst = smem_u32(sB8 + b8 * kB8Bytes);
#pragma unroll
        for (int i = 0; i < kItemsPerThread; ++i) {
          uint32_t o[8];
          expand16(w[i], o);
          sts128(dst + d0[i], o[0], o[1], o[2], o[3]);
          sts128(dst + d1[i], o[4], o[5], o[6], o[7]);
        }
        publish(b8);
      }
    }
    } else {
      // W4A16: packed row r (64 bytes = 128 values), 16-byte chunk c (32
      // values) -> 32 16-bit values in 64-value atom c / 2, 16-byte chunks
      // 4 (c % 2) .. + 3 of row r (row r at (r / 8) * 1024 + (r % 8) * 128 of
      // the atom, chunk index XOR r % 8).  NK: r = column n, K-major atoms of
      // 64 K.  KN: r = k, MN-major atoms of 64 columns.  A quarter-warp takes
      // rows 4q .. 4q + 3 with c in {0, 1} or {2, 3}: each of its stores hits
      // 8 distinct chunk positions.
      constexpr int kIt = kBpStage<KIND> / 16 / kXThreads;  // 4
      uint32_t src[kIt], rowoff[kIt], cbase[kIt], rsw[kIt];
#pragma unroll
      for (int i = 0; i < kIt; ++i) {
        const int item = i * kXThreads + xt;
        const int qw = item >> 3, l = item & 7;
        const int r = 4 * (qw >> 1) + (l >> 1), c = ((qw & 1) << 1) | (l & 1);
        src[i] = r * 64 + c * 16;
        rowoff[i] = (c >> 1) * 16384 + (r >> 3) * 1024 + (r & 7) * 128;
        cbase[i] = (c & 1) * 4;
        rsw[i] = r & 7;
      }
      int g = 0;
      for (int tile = pair_id; tile < num_tiles && ok; tile += num_pairs) {
        for (int ks = 0; ks < k_stages; ++ks, ++g) {
          const int slot = g % S, b8 = g % B8;
          if (!wait(&bars->bp_full[slot], (g / S) & 1, bars, 17)) { ok = false; break; }
          uint4 w[kIt];
          const uint8_t* bp = sBp + slot * kBpBytes;
#pragma unroll
          for (int i = 0; i < kIt; ++i) w[i] = *reinterpret_cast<const uint4*>(bp + src[i]);
          if (!wait(&bars->b8_empty[b8], ((g / B8) & 1) ^ 1, bars, 18)) { ok = false; break; }
          const uint32_t dst = smem_u32(sB8 + b8 * kB8Bytes);
#pragma unroll
          for (int i = 0; i < kIt; ++i) {
            uint32_t o[16];
            expand16_to_16bit<KIND>(w[i], o);
#pragma unroll
            for (int q = 0; q < 4; ++q)
              sts128(dst + rowoff[i] + (((cbase[i] + q) ^ rsw[i]) << 4), o[4 * q], o[4 * q + 1], o[4 * q + 2],
                     o[4 * q + 3]);
          }
          publish(b8);
        }
      }
    }
    if (lane == 0) settle_after_error(ok);  // a token copy may still be in flight
  } else {
    // ---------------- epilogue ----------------
    const int ew = warp & 3;
    float* sws = epi + ew * 2 * BN;
    float* sbias = sws + BN;
    const uint32_t lead_empty0 = mapa_shared(&bars->acc_empty[0], 0);
    // this CTA's last tile: columns 128.. go to the helper warp of this quarter
    const int last_local = pair_id < num_tiles ? (num_tiles - 1 - pair_id) / num_pairs : -1;
    bool helper_released = false;
    int local = 0;
    for (int tile = pair_id; tile < num_tiles; tile += num_pairs, ++local) {
      const int buf = local & 1;
      const int n_blk = tile / p.m_tiles;
      __syncwarp();
      for (int j = lane; j < BN; j += 32) {
        const int col = n_blk * BN + j;
        sws[j] = col < p.N ? __ldg(p.wscales + col) : 0.0f;
        sbias[j] = (col < p.N && p.bias) ? __ldg(p.bias + col) : 0.0f;
      }
      __syncwarp();
      const bool last = local == last_local;
      if (last) {
        named_bar_arrive(kHelpBar0 + ew, 64);  // scales staged: the helper may read them
        helper_released = true;
      }
      if (!epi_chunks(tile, local, ew, 0, last ? BN / 64 : BN / 32, sws, sbias, smem_u32(stage_out) + ew * 2048))
        break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(lead_empty0 + buf * 8);
    }
    // after an error before the last tile: still release the helper (its own
    // accumulator wait then fails at once on the recorded error)
    if (!helper_released && last_local >= 0) named_bar_arrive(kHelpBar0 + ew, 64);
    // peers read the gathered output after a flag barrier that follows this
    // kernel: make this thread's stores to their memory visible system-wide
    if (p.n_outs > 0) __threadfence_system();
  }

  // Helpers: once their own work is done, warps 4-7 (TMEM lane quarters 0-3)
  // take columns 128..255 of the CTA's last tile, whose epilogue is otherwise
  // exposed after the last MMA.  They restage through the int8 weight ring,
  // idle once the last accumulator is complete.
  if (warp >= 4 && warp < 8 && pair_id < num_tiles) {
    const int q = warp & 3;
    const int last_local = (num_tiles - 1 - pair_id) / num_pairs;
    named_bar_sync(kHelpBar0 + q, 64);  // the quarter's epilogue warp has staged the scales
    const float* hws = epi + q * 2 * BN;
    epi_chunks(pair_id + last_local * num_pairs, last_local, q, BN / 64, BN / 32, hws, hws + BN,
               smem_u32(sB8) + (warp - 4) * 2048);
    if (p.n_outs > 0) __threadfence_system();
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync();  // no CTA leaves while its partner may still touch its shared memory or TMEM
  tc_fence_after();
  if (warp == kWarpMma) {
    __syncwarp();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0 && bars->err) atomicCAS(&g_convrot_device_error, 0, bars->err);
}

}  // namespace pair

// ---------------------------------------------------------------------------
// host side

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

int make_tmap_2d_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                    uint32_t box_inner, uint32_t box_outer) {
  auto encode = get_encode_fn();
  CONVROT_REQUIRE(encode != nullptr, CONVROT_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t elem_strides[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, elem_strides,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  CONVROT_REQUIRE(r == CUDA_SUCCESS, CONVROT_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return CONVROT_OK;
}

// Tiled uint8 tensor map of rank 2 or 3 (dims / strides in bytes, innermost first).
int make_tmap_u8(CUtensorMap* map, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                 const uint32_t* box, CUtensorMapSwizzle swizzle,
                 CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_UINT8) {
  auto encode = get_encode_fn();
  CONVROT_REQUIRE(encode != nullptr, CONVROT_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t d[3];
  cuuint64_t st[2];
  cuuint32_t b[3];
  cuuint32_t es[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
  }
  for (int i = 0; i + 1 < rank; ++i) st[i] = strides[i];
  CUresult r = encode(map, dtype, rank, const_cast<void*>(base), d, st, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  CONVROT_REQUIRE(r == CUDA_SUCCESS, CONVROT_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return CONVROT_OK;
}

// The CTA-pair kernel needs K % 128 == 0 (A is read as 128-byte K chunks) and
// a weight row stride that TMA can describe (K x packed-N: N % 32 == 0).
bool pair_supported(int layout, int64_t n, int64_t k) {
  return k % 128 == 0 && (layout == CONVROT_LAYOUT_NK || n % 32 == 0);
}

template <int LAYOUT, typename TOut, int KIND = pair::KIND_I8>
static int launch_pair(const void* act, const Params& p0, cudaStream_t stream) {
  Params p = p0;
  p.m_tiles = (p.M + pair::BM - 1) / pair::BM;
  p.n_tiles = (p.N + pair::BN - 1) / pair::BN;
  CONVROT_REQUIRE(static_cast<int64_t>(p.m_tiles) * p.n_tiles < (1LL << 31), CONVROT_ERR_UNSUPPORTED,
                  "too many output tiles");
  constexpr bool k16 = KIND != pair::KIND_I8;
  constexpr int KS = pair::kKStage<KIND>;
  CUtensorMap map_a, map_b;
  {
    // A viewed as (K / chunk) x M rows x one 128-byte chunk; one box = 2 chunks x 128 rows
    const uint64_t chunk = k16 ? 64 : 128;  // elements per 128 bytes
    const uint64_t dims[3] = {chunk, static_cast<uint64_t>(p.M), static_cast<uint64_t>(p.K) / chunk};
    const uint64_t strides[2] = {static_cast<uint64_t>(p.K) * (k16 ? 2 : 1), 128};
    const uint32_t box[3] = {static_cast<uint32_t>(chunk), 128, 2};
    int rc = make_tmap_u8(&map_a, act, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                          k16 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8);
    if (rc != CONVROT_OK) return rc;
  }
  {
    int rc;
    if (LAYOUT == CONVROT_LAYOUT_NK) {
      const uint64_t dims[2] = {static_cast<uint64_t>(p.K / 2), static_cast<uint64_t>(p.N)};
      const uint64_t strides[1] = {static_cast<uint64_t>(p.K / 2)};
      const uint32_t box[2] = {KS / 2, 128};
      rc = make_tmap_u8(&map_b, p.qweight, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    } else {
      const uint64_t dims[2] = {static_cast<uint64_t>(p.N / 2), static_cast<uint64_t>(p.K)};
      const uint64_t strides[1] = {static_cast<uint64_t>(p.N / 2)};
      const uint32_t box[2] = {64, KS};
      rc = make_tmap_u8(&map_b, p.qweight, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    if (rc != CONVROT_OK) return rc;
  }
  auto kernel = pair::pair_gemm_kernel<LAYOUT, TOut, KIND>;
  CONVROT_CUDA_CHECK(
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(pair::kSmemBytes)));
  const int tiles = p.m_tiles * p.n_tiles;
  const int max_pairs = device_sm_count() / 2;
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(pair::kThreads, 1, 1);
  cfg.dynamicSmemBytes = pair::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see grid_dependency_wait
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  CONVROT_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, map_a, map_b, p));
  return check_launch("w4a4 pair gemm");
}

template <int LAYOUT, typename TOut>
static int launch(const CUtensorMap& map, const Params& p, cudaStream_t stream) {
  auto kernel = w4a4_gemm_kernel<LAYOUT, TOut>;
  CONVROT_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes)));
  const int tiles = p.m_tiles * p.n_tiles;
  const int grid = tiles < device_sm_count() ? tiles : device_sm_count();
  kernel<<<grid, kThreads, kSmemBytes, stream>>>(map, p);
  return check_launch("w4a4 gemm");
}

// Kernel routing of convrot_w4a4_gemm: 0 automatic, 1 every shape to the
// one-CTA kernel, 2 every shape the CTA-pair kernel takes to it, 3 every
// shape the swap-AB kernel takes (m <= 64) to it, 4 every shape the GEMV
// kernel takes (m <= 8) to it (set by convrot_set_gemm_route, for tests and
// A/B measurements).
std::atomic<int> g_gemm_route{0};

int forced_kernel() { return g_gemm_route.load(std::memory_order_relaxed); }

}  // namespace w4a4

// Argument checks of convrot_w4a4_gemm, also run by callers that enqueue
// other work before the GEMM (the allocation-free linear), so that a call the
// GEMM would reject enqueues nothing.  With need_act false the activation
// pointer (not yet produced) is not checked.
int w4a4::check_gemm_args(const int8_t* act, const uint8_t* qweight, int layout, const float* xscales,
                          const float* wscales, const void* out, int out_dtype, int64_t m, int64_t n, int64_t k,
                          bool need_act) {
  CONVROT_REQUIRE(layout == CONVROT_LAYOUT_NK || layout == CONVROT_LAYOUT_KN, CONVROT_ERR_INVALID, "unknown layout %d",
                  layout);
  CONVROT_REQUIRE(valid_dtype(out_dtype), CONVROT_ERR_INVALID, "unknown output dtype %d", out_dtype);
  CONVROT_REQUIRE(m >= 0 && n > 0 && k > 0, CONVROT_ERR_INVALID, "invalid shape m=%lld n=%lld k=%lld",
                  static_cast<long long>(m), static_cast<long long>(n), static_cast<long long>(k));
  CONVROT_REQUIRE(k % 32 == 0, CONVROT_ERR_INVALID, "W4A4 GEMM requires K divisible by 32, got %lld",
                  static_cast<long long>(k));
  CONVROT_REQUIRE(layout == CONVROT_LAYOUT_NK || n % 2 == 0, CONVROT_ERR_INVALID,
                  "K x packed-N weights require even N, got %lld", static_cast<long long>(n));
  CONVROT_REQUIRE(m < (1LL << 31) && n < (1LL << 31) && k < (1LL << 31), CONVROT_ERR_UNSUPPORTED, "shape too large");
  if (m == 0) return CONVROT_OK;
  CONVROT_REQUIRE((act || !need_act) && qweight && (xscales || !need_act) && wscales && out, CONVROT_ERR_INVALID,
                  "null pointer");
  CONVROT_REQUIRE((!need_act || aligned_to(act, 16)) && aligned_to(qweight, 16) && aligned_to(out, 16),
                  CONVROT_ERR_INVALID, "activation, weight and output must be 16-byte aligned");
  return CONVROT_OK;
}

}  // namespace convrot

extern "C" {

int convrot_w4a4_gemm(const int8_t* act, const uint8_t* qweight, int layout, const float* xscales,
                      const float* wscales, const float* bias, void* out, int out_dtype, int64_t m, int64_t n,
                      int64_t k, void* stream) {
  using namespace convrot;
  const int args_rc = w4a4::check_gemm_args(act, qweight, layout, xscales, wscales, out, out_dtype, m, n, k,
                                            /*need_act=*/true);
  if (args_rc != CONVROT_OK || m == 0) return args_rc;
  w4a4::Params p;
  p.qweight = qweight;
  p.xscales = xscales;
  p.wscales = wscales;
  p.bias = bias;
  p.out = out;
  p.M = static_cast<int>(m);
  p.N = static_cast<int>(n);
  p.K = static_cast<int>(k);
  p.m_tiles = static_cast<int>((m + w4a4::BM - 1) / w4a4::BM);
  p.n_tiles = static_cast<int>((n + w4a4::BN - 1) / w4a4::BN);
  p.k_blocks = static_cast<int>((k + w4a4::BK - 1) / w4a4::BK);
  CONVROT_REQUIRE(static_cast<int64_t>(p.m_tiles) * p.n_tiles < (1LL << 31), CONVROT_ERR_UNSUPPORTED,
                  "too many output tiles");
  p.layout = layout;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int forced = w4a4::forced_kernel();
  if ((forced == 0 || forced == 4) && gemv_supported(layout, m, n, k))
    return launch_gemv(act, qweight, layout, xscales, wscales, bias, out, out_dtype, m, n, k, s);
  if (((forced == 0 && m <= small_m_auto_rows()) || forced == 3) && small_m_supported(layout, m, n, k))
    return launch_small_m(act, qweight, layout, xscales, wscales, bias, out, out_dtype, m, n, k, s);
  const bool use_pair = w4a4::pair_supported(layout, n, k) && forced != 1;
  if (use_pair) {
    if (layout == CONVROT_LAYOUT_NK) {
      switch (out_dtype) {
        case CONVROT_BF16: return w4a4::launch_pair<CONVROT_LAYOUT_NK, __nv_bfloat16>(act, p, s);
        case CONVROT_F16: return w4a4::launch_pair<CONVROT_LAYOUT_NK, __half>(act, p, s);
        default: return w4a4::launch_pair<CONVROT_LAYOUT_NK, float>(act, p, s);
      }
    }
    switch (out_dtype) {
      case CONVROT_BF16: return w4a4::launch_pair<CONVROT_LAYOUT_KN, __nv_bfloat16>(act, p, s);
      case CONVROT_F16: return w4a4::launch_pair<CONVROT_LAYOUT_KN, __half>(act, p, s);
      default: return w4a4::launch_pair<CONVROT_LAYOUT_KN, float>(act, p, s);
    }
  }
  CUtensorMap map;
  int rc = w4a4::make_tmap_2d_u8(&map, act, static_cast<uint64_t>(k), static_cast<uint64_t>(m),
                                 static_cast<uint64_t>(k), w4a4::BK, w4a4::BM);
  if (rc != CONVROT_OK) return rc;
  if (layout == CONVROT_LAYOUT_NK) {
    switch (out_dtype) {
      case CONVROT_BF16: return w4a4::launch<CONVROT_LAYOUT_NK, __nv_bfloat16>(map, p, s);
      case CONVROT_F16: return w4a4::launch<CONVROT_LAYOUT_NK, __half>(map, p, s);
      default: return w4a4::launch<CONVROT_LAYOUT_NK, float>(map, p, s);
    }
  }
  switch (out_dtype) {
    case CONVROT_BF16: return w4a4::launch<CONVROT_LAYOUT_KN, __nv_bfloat16>(map, p, s);
    case CONVROT_F16: return w4a4::launch<CONVROT_LAYOUT_KN, __half>(map, p, s);
    default: return w4a4::launch<CONVROT_LAYOUT_KN, float>(map, p, s);
  }
}

// Tensor-parallel W4A4: this rank's column shard, all-gathered by the epilogue.
int convrot_w4a4_gemm_gather(const int8_t* act, const uint8_t* qweight, int layout, const float* xscales,
                             const float* wscales, const float* bias, void* const* outs, int n_outs, int64_t ldc,
                             int64_t col_offset, int out_dtype, int64_t m, int64_t n, int64_t k, void* stream) {
  using namespace convrot;
  CONVROT_REQUIRE(layout == CONVROT_LAYOUT_NK || layout == CONVROT_LAYOUT_KN, CONVROT_ERR_INVALID, "unknown layout %d",
                  layout);
  CONVROT_REQUIRE(valid_dtype(out_dtype), CONVROT_ERR_INVALID, "unknown output dtype %d", out_dtype);
  CONVROT_REQUIRE(m >= 0 && n > 0 && k > 0, CONVROT_ERR_INVALID, "invalid shape m=%lld n=%lld k=%lld",
                  static_cast<long long>(m), static_cast<long long>(n), static_cast<long long>(k));
  CONVROT_REQUIRE(outs != nullptr && n_outs >= 1 && n_outs <= w4a4::kMaxOuts, CONVROT_ERR_INVALID,
                  "n_outs must be in [1, %d], got %d", w4a4::kMaxOuts, n_outs);
  CONVROT_REQUIRE(col_offset >= 0 && ldc >= col_offset + n, CONVROT_ERR_INVALID,
                  "ldc %lld too small for column offset %lld + n %lld", static_cast<long long>(ldc),
                  static_cast<long long>(col_offset), static_cast<long long>(n));
  CONVROT_REQUIRE(m < (1LL << 31) && n < (1LL << 31) && k < (1LL << 31), CONVROT_ERR_UNSUPPORTED, "shape too large");
  CONVROT_REQUIRE(w4a4::pair_supported(layout, n, k), CONVROT_ERR_UNSUPPORTED,
                  "the gathering GEMM needs K %% 128 == 0 and, for K x packed-N, N %% 32 == 0 (m=%lld n=%lld k=%lld)",
                  static_cast<long long>(m), static_cast<long long>(n), static_cast<long long>(k));
  if (m == 0) return CONVROT_OK;
  CONVROT_REQUIRE(act && qweight && xscales && wscales, CONVROT_ERR_INVALID, "null pointer");
  CONVROT_REQUIRE(aligned_to(act, 16) && aligned_to(qweight, 16), CONVROT_ERR_INVALID,
                  "activation and weight must be 16-byte aligned");
  w4a4::Params p;
  p.qweight = qweight;
  p.xscales = xscales;
  p.wscales = wscales;
  p.bias = bias;
  p.M = static_cast<int>(m);
  p.N = static_cast<int>(n);
  p.K = static_cast<int>(k);
  p.layout = layout;
  for (int d = 0; d < n_outs; ++d) {
    CONVROT_REQUIRE(outs[d] != nullptr, CONVROT_ERR_INVALID, "null destination %d", d);
    p.outs[d] = outs[d];
  }
  p.out = outs[0];
  p.n_outs = n_outs;
  p.ldc = ldc;
  p.col_off = col_offset;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  using namespace w4a4;
  if (layout == CONVROT_LAYOUT_NK) {
    switch (out_dtype) {
      case CONVROT_BF16: return launch_pair<CONVROT_LAYOUT_NK, __nv_bfloat16>(act, p, s);
      case CONVROT_F16: return launch_pair<CONVROT_LAYOUT_NK, __half>(act, p, s);
      default: return launch_pair<CONVROT_LAYOUT_NK, float>(act, p, s);
    }
  }
  switch (out_dtype) {
    case CONVROT_BF16: return launch_pair<CONVROT_LAYOUT_KN, __nv_bfloat16>(act, p, s);
    case CONVROT_F16: return launch_pair<CONVROT_LAYOUT_KN, __half>(act, p, s);
    default: return launch_pair<CONVROT_LAYOUT_KN, float>(act, p, s);
  }
}

// W4A16: rotated bf16 / fp16 activations x packed int4 weights (core.py:1123-1152).
int convrot_w4a16_gemm(const void* act, int act_dtype, const uint8_t* qweight, int layout, const float* wscales,
                       const float* bias, void* out, int out_dtype, int64_t m, int64_t n, int64_t k, void* stream) {
  using namespace convrot;
  CONVROT_REQUIRE(layout == CONVROT_LAYOUT_NK || layout == CONVROT_LAYOUT_KN, CONVROT_ERR_INVALID, "unknown layout %d",
                  layout);
  CONVROT_REQUIRE(act_dtype == CONVROT_BF16 || act_dtype == CONVROT_F16, CONVROT_ERR_INVALID,
                  "W4A16 activations must be bfloat16 or float16 (dtype %d)", act_dtype);
  CONVROT_REQUIRE(valid_dtype(out_dtype), CONVROT_ERR_INVALID, "unknown output dtype %d", out_dtype);
  CONVROT_REQUIRE(m >= 0 && n > 0 && k > 0, CONVROT_ERR_INVALID, "invalid shape m=%lld n=%lld k=%lld",
                  static_cast<long long>(m), static_cast<long long>(n), static_cast<long long>(k));
  CONVROT_REQUIRE(m < (1LL << 31) && n < (1LL << 31) && k < (1LL << 31), CONVROT_ERR_UNSUPPORTED, "shape too large");
  CONVROT_REQUIRE(k % 64 == 0, CONVROT_ERR_UNSUPPORTED,
                  "the W4A16 kernel needs K divisible by 64 (TMA chunks of 64 16-bit values), got %lld",
                  static_cast<long long>(k));
  CONVROT_REQUIRE(layout == CONVROT_LAYOUT_NK || n % 32 == 0, CONVROT_ERR_UNSUPPORTED,
                  "the W4A16 kernel needs N divisible by 32 for K x packed-N weights (16-byte rows), got %lld",
                  static_cast<long long>(n));
  if (m == 0) return CONVROT_OK;
  CONVROT_REQUIRE(act && qweight && wscales && out, CONVROT_ERR_INVALID, "null pointer");
  CONVROT_REQUIRE(aligned_to(act, 16) && aligned_to(qweight, 16) && aligned_to(out, 16), CONVROT_ERR_INVALID,
                  "activation, weight and output must be 16-byte aligned");
  w4a4::Params p;
  p.qweight = qweight;
  p.xscales = nullptr;
  p.wscales = wscales;
  p.bias = bias;
  p.out = out;
  p.M = static_cast<int>(m);
  p.N = static_cast<int>(n);
  p.K = static_cast<int>(k);
  p.layout = layout;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  using namespace w4a4;
#define CONVROT_W4A16_OUT(L, KIND)                                                    \
  switch (out_dtype) {                                                                \
    case CONVROT_BF16: return launch_pair<L, __nv_bfloat16, pair::KIND>(act, p, s);   \
    case CONVROT_F16: return launch_pair<L, __half, pair::KIND>(act, p, s);           \
    default: return launch_pair<L, float, pair::KIND>(act, p, s);                     \
  }
  if (layout == CONVROT_LAYOUT_NK) {
    if (act_dtype == CONVROT_BF16) { CONVROT_W4A16_OUT(CONVROT_LAYOUT_NK, KIND_BF16) }
    CONVROT_W4A16_OUT(CONVROT_LAYOUT_NK, KIND_F16)
  }
  if (act_dtype == CONVROT_BF16) { CONVROT_W4A16_OUT(CONVROT_LAYOUT_KN, KIND_BF16) }
  CONVROT_W4A16_OUT(CONVROT_LAYOUT_KN, KIND_F16)
#undef CONVROT_W4A16_OUT
}

int convrot_set_gemm_route(int route) {
  using namespace convrot;
  CONVROT_REQUIRE(route >= 0 && route <= 4, CONVROT_ERR_INVALID, "GEMM route must be 0-4, got %d", route);
  w4a4::g_gemm_route.store(route, std::memory_order_relaxed);
  return CONVROT_OK;
}

// Read and clear the device-side error word set by a kernel whose bounded
// wait timed out (0 = none).  Synchronizes the device.
int convrot_take_device_error(int* code) {
  int v = 0, zero = 0;
  CONVROT_CUDA_CHECK(cudaDeviceSynchronize());
  CONVROT_CUDA_CHECK(cudaMemcpyFromSymbol(&v, convrot::g_convrot_device_error, sizeof(int)));
  CONVROT_CUDA_CHECK(cudaMemcpyToSymbol(convrot::g_convrot_device_error, &zero, sizeof(int)));
  if (code) *code = v;
  return CONVROT_OK;
}

}  // extern "C"
