// Shared helpers for libconvrot_b200.so: status handling, dtype traits and
// the inline-PTX wrappers (mbarrier, TMA, tcgen05) used by the kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/convrot_b200.h"

namespace convrot {

// ---------------------------------------------------------------------------
// status handling (host)

void set_error(const char* fmt, ...);

#define CONVROT_REQUIRE(cond, code, ...)      \
  do {                                        \
    if (!(cond)) {                            \
      ::convrot::set_error(__VA_ARGS__);      \
      return (code);                          \
    }                                         \
  } while (0)

#define CONVROT_CUDA_CHECK(expr)                                                       \
  do {                                                                                 \
    cudaError_t err__ = (expr);                                                        \
    if (err__ != cudaSuccess) {                                                        \
      ::convrot::set_error("%s failed: %s", #expr, cudaGetErrorString(err__));         \
      return CONVROT_ERR_CUDA;                                                         \
    }                                                                                  \
  } while (0)

// Check the launch that was just enqueued.
int check_launch(const char* what);

inline bool aligned_to(const void* p, uintptr_t bytes) {
  return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}

int device_sm_count();

// Device address of the library's device-side error word (set by a kernel
// whose bounded wait timed out) on the current device.
int* device_error_word();

// Swap-AB W4A4 GEMM for few activation rows (gemm_small_m.cu): the shapes it
// takes, and its launch after convrot_w4a4_gemm's argument checks.
bool small_m_supported(int layout, int64_t m, int64_t n, int64_t k);
int small_m_auto_rows();
int launch_small_m(const int8_t* act, const uint8_t* qweight, int layout, const float* xscales, const float* wscales,
                   const float* bias, void* out, int out_dtype, int64_t m, int64_t n, int64_t k, cudaStream_t stream);

// Register-fragment W4A4 GEMV for at most 8 activation rows (gemv_w4a4.cu):
// the shapes it takes, and its launch after convrot_w4a4_gemm's argument
// checks.
bool gemv_supported(int layout, int64_t m, int64_t n, int64_t k);
int launch_gemv(const int8_t* act, const uint8_t* qweight, int layout, const float* xscales, const float* wscales,
                const float* bias, void* out, int out_dtype, int64_t m, int64_t n, int64_t k, cudaStream_t stream);

namespace w4a4 {
// Argument checks of convrot_w4a4_gemm (gemm_w4a4.cu); need_act false skips
// the activation and row-scale pointers (for callers that produce them).
int check_gemm_args(const int8_t* act, const uint8_t* qweight, int layout, const float* xscales,
                    const float* wscales, const void* out, int out_dtype, int64_t m, int64_t n, int64_t k,
                    bool need_act);
}  // namespace w4a4

// ---------------------------------------------------------------------------
// element types

template <typename T> struct Elem;

template <> struct Elem<__nv_bfloat16> {
  using Pair = __nv_bfloat162;
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ Pair add(Pair a, Pair b) { return __hadd2(a, b); }
  static __device__ __forceinline__ Pair sub(Pair a, Pair b) { return __hsub2(a, b); }
  static __device__ __forceinline__ Pair mul(Pair a, Pair b) { return __hmul2(a, b); }
  static __device__ __forceinline__ Pair make(__nv_bfloat16 lo, __nv_bfloat16 hi) { return __halves2bfloat162(lo, hi); }
  static __device__ __forceinline__ Pair splat(float v) { return __float2bfloat162_rn(v); }
  static __device__ __forceinline__ __nv_bfloat16 lo(Pair p) { return __low2bfloat16(p); }
  static __device__ __forceinline__ __nv_bfloat16 hi(Pair p) { return __high2bfloat16(p); }
};

template <> struct Elem<__half> {
  using Pair = __half2;
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ Pair add(Pair a, Pair b) { return __hadd2(a, b); }
  static __device__ __forceinline__ Pair sub(Pair a, Pair b) { return __hsub2(a, b); }
  static __device__ __forceinline__ Pair mul(Pair a, Pair b) { return __hmul2(a, b); }
  static __device__ __forceinline__ Pair make(__half lo, __half hi) { return __halves2half2(lo, hi); }
  static __device__ __forceinline__ Pair splat(float v) { return __float2half2_rn(v); }
  static __device__ __forceinline__ __half lo(Pair p) { return __low2half(p); }
  static __device__ __forceinline__ __half hi(Pair p) { return __high2half(p); }
};

template <> struct Elem<float> {
  using Pair = float2;
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
  static __device__ __forceinline__ Pair add(Pair a, Pair b) { return make_float2(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y)); }
  static __device__ __forceinline__ Pair sub(Pair a, Pair b) { return make_float2(__fsub_rn(a.x, b.x), __fsub_rn(a.y, b.y)); }
  static __device__ __forceinline__ Pair mul(Pair a, Pair b) { return make_float2(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y)); }
  static __device__ __forceinline__ Pair make(float lo, float hi) { return make_float2(lo, hi); }
  static __device__ __forceinline__ Pair splat(float v) { return make_float2(v, v); }
  static __device__ __forceinline__ float lo(Pair p) { return p.x; }
  static __device__ __forceinline__ float hi(Pair p) { return p.y; }
};

// Store float -> output element type with round-to-nearest-even.
template <typename T> __device__ __forceinline__ T cvt_out(float v);
template <> __device__ __forceinline__ float cvt_out<float>(float v) { return v; }
template <> __device__ __forceinline__ __half cvt_out<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 cvt_out<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

inline size_t dtype_size(int dtype) {
  return dtype == CONVROT_F32 ? 4 : 2;
}

inline bool valid_dtype(int dtype) {
  return dtype == CONVROT_F32 || dtype == CONVROT_F16 || dtype == CONVROT_BF16;
}

// ---------------------------------------------------------------------------
// PTX wrappers: shared-memory addresses, mbarriers, TMA, tcgen05

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialization may start while the previous kernel of its stream is still
// running.  grid_dependency_wait() returns once that kernel has completed
// and its writes are visible, so a thread calls it before its first global
// load or store; grid_dependents_launch() lets the next kernel of the stream
// start early (it still waits in its own grid_dependency_wait()).  Without
// the launch attribute both are no-ops.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dependents_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Cluster-scope acquire: for barriers that receive arrivals from the other
// CTA of a pair.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: spins at most `limit` polls (each try_wait itself blocks for a
// hardware-defined time slice).  On time-out it records `code` in *err and
// returns false; callers then skip the remaining work so the kernel ends.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t limit,
                                                  volatile int* err, int code) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*err) return false;
  }
  *err = code;
  return false;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// 1-D bulk copy global -> this CTA's shared memory (16-byte aligned, size a
// multiple of 16), completing transaction bytes on `bar`.
__device__ __forceinline__ void bulk_load_1d(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Pair-MMA form: the copy lands in this CTA's shared memory and completes
// transaction bytes on an mbarrier given as a cluster address (the pair
// leader's barrier).  No multicast.
__device__ __forceinline__ void tma_load_3d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster_addr, int x,
                                                 int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// ---- clusters --------------------------------------------------------------

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Cluster-window address of the same shared-memory location in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}

// Publishes this thread's earlier shared::cta writes to a cluster peer that
// acquires the barrier: a release fence restricted to shared::cta (much
// cheaper than a full cluster-scope release) followed by a relaxed remote
// arrive.  The writer fences its generic stores for the async proxy first
// when the tensor core is the reader.
__device__ __forceinline__ void mbar_arrive_cluster_publish_smem(uint32_t bar_cluster_addr) {
  asm volatile("fence.release.sync_restrict::shared::cta.cluster;" ::: "memory");
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}

// Bulk copy of `bytes` (multiple of 16) from this CTA's shared memory into a
// cluster peer's, completing transaction bytes on the peer's mbarrier (both
// given as cluster addresses).  Runs on the async proxy, like TMA.
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst_cluster, const void* src, uint32_t bytes,
                                                  uint32_t bar_cluster) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst_cluster),
               "r"(smem_u32(src)), "r"(bytes), "r"(bar_cluster)
               : "memory");
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// tcgen05 ------------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D(tmem) (+)= A(smem desc) x B(smem desc); kind::i8, one CTA.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D(tmem) (+)= A x B; kind::f16 (bf16 or fp16 operands, fp32 accumulate).
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// ---- CTA-pair (cta_group::2) forms ----
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the mbarrier at the same shared-memory offset in every CTA of
// `cta_mask` once all pair MMAs issued before by this thread are complete.
__device__ __forceinline__ void mma_commit_pair_multicast(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// Arrive on an mbarrier once every tcgen05.mma issued before by this thread
// has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// 32 lanes x 32 bit, 32 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Paired fp32 multiply (sm_100 f32x2), each component rounded to nearest
// even exactly as mul.rn.f32.
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor (tcgen05 form, version 1).
//   start address >> 4 in bits [0,14), leading byte offset >> 4 in [16,30),
//   stride byte offset >> 4 in [32,46), version 1 in [46,48), base offset 0,
//   swizzle mode in [61,64) (2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t swizzle_mode) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(swizzle_mode & 0x7u) << 61;
  return d;
}

}  // namespace convrot
