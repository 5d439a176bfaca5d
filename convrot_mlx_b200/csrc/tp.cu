// Tensor-parallel plumbing: a flag barrier between the GPUs of one node.
//
// Each rank owns a flag array (one 32-bit word per rank) in memory that every
// peer has mapped (symmetric memory).  After a rank's gathering GEMM has
// stored its column shard into every rank's output buffer (and fenced those
// stores system-wide), the barrier kernel writes the call's epoch into slot
// `rank` of every rank's array with a system-scope release store, then waits
// with acquire loads until every slot of its own array holds the epoch.  The
// wait is bounded: after kBarrierTimeoutNs the kernel records an error in
// the device error word and returns, so a missing peer never hangs the GPU.
#include "common.cuh"

namespace convrot {

constexpr int kMaxPeers = 8;
constexpr uint64_t kBarrierTimeoutNs = 2000000000ull;

struct PeerFlags {
  uint32_t* flags[kMaxPeers];
};

__global__ void peer_barrier_kernel(const __grid_constant__ PeerFlags pf, int world, int rank, uint32_t epoch,
                                    int* err_word) {
  const int t = threadIdx.x;
  if (t < world) {
    uint32_t* dst = pf.flags[t] + rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(dst), "r"(epoch) : "memory");
    const uint32_t* src = pf.flags[rank] + t;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 0;; ++i) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(src) : "memory");
      if (v == epoch) break;
      if ((i & 63) == 63 && globaltimer() - t0 > kBarrierTimeoutNs) {
        if (err_word) atomicCAS(err_word, 0, 31);
        break;
      }
    }
  }
}

}  // namespace convrot

extern "C" {

int convrot_peer_barrier(uint32_t* const* flag_arrays, int world, int rank, uint32_t epoch, void* stream) {
  using namespace convrot;
  CONVROT_REQUIRE(flag_arrays != nullptr && world >= 1 && world <= kMaxPeers, CONVROT_ERR_INVALID,
                  "world must be in [1, %d], got %d", kMaxPeers, world);
  CONVROT_REQUIRE(rank >= 0 && rank < world, CONVROT_ERR_INVALID, "rank %d outside [0, %d)", rank, world);
  CONVROT_REQUIRE(epoch != 0, CONVROT_ERR_INVALID, "epoch 0 is reserved (flags start at 0)");
  PeerFlags pf = {};
  for (int r = 0; r < world; ++r) {
    CONVROT_REQUIRE(flag_arrays[r] != nullptr && aligned_to(flag_arrays[r], 4), CONVROT_ERR_INVALID,
                    "flag array %d is null or misaligned", r);
    pf.flags[r] = flag_arrays[r];
  }
  peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(pf, world, rank, epoch, device_error_word());
  return check_launch("convrot peer barrier");
}

// One strided block copy on a copy engine: `rows` rows of `width_bytes`,
// source rows `src_pitch` bytes apart, destination rows `dst_pitch` apart.
// The tensor-parallel layer pushes each M-chunk of its column shard into
// every peer's output with it (peer memory mapped into this GPU), so the
// gather runs on the copy engines while the SMs compute the next chunk.
int convrot_copy_2d(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch, int64_t width_bytes,
                    int64_t rows, void* stream) {
  using namespace convrot;
  CONVROT_REQUIRE(rows >= 0 && width_bytes >= 0 && dst_pitch >= width_bytes && src_pitch >= width_bytes,
                  CONVROT_ERR_INVALID, "invalid 2-D copy: %lld rows of %lld bytes, pitches %lld / %lld",
                  static_cast<long long>(rows), static_cast<long long>(width_bytes),
                  static_cast<long long>(dst_pitch), static_cast<long long>(src_pitch));
  if (rows == 0 || width_bytes == 0) return CONVROT_OK;
  CONVROT_REQUIRE(dst && src, CONVROT_ERR_INVALID, "null pointer");
  CONVROT_CUDA_CHECK(cudaMemcpy2DAsync(dst, static_cast<size_t>(dst_pitch), src, static_cast<size_t>(src_pitch),
                                       static_cast<size_t>(width_bytes), static_cast<size_t>(rows),
                                       cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream)));
  return CONVROT_OK;
}

}  // extern "C"
