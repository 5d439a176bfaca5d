// The whole W4A4 linear (rotate + A4-quantize, then the int4 GEMM with its
// fused epilogue) in one call that allocates no device memory.
//
// Between its two kernels the linear needs an intermediate: the int8 codes
// (M x K bytes) and the row scales (M floats).  convrot_prepare_i8 +
// convrot_w4a4_gemm leave that buffer to the caller.  Some callers have no
// way to provide it: a plugin that a host engine invokes with nothing but
// its input and output buffers, or a caller whose host framework reserves
// the device's memory for its own allocator and allows no cudaMalloc on the
// side.  For them this entry point keeps the intermediate in a file-scope
// device array of fixed size, created when the library is loaded.
//
// Host code cannot use that array's name as a device address (in host code
// it names a host-side stand-in), so its device address is looked up once
// per device with cudaGetSymbolAddress, with that device current, on the
// first call made on the device.  That lookup may load the module on the
// device, which a stream capture does not allow: a first call made while its
// stream is capturing is refused with a message instead.
#include <mutex>
#include <vector>

#include "common.cuh"

namespace convrot {
namespace {

// 64 MiB: int8 codes of M x K (rounded up to 256 bytes) followed by M float
// row scales.  Enough for M x K up to about 67 million, e.g. 4096 x 16384.
constexpr int64_t kStaticScratchBytes = CONVROT_LINEAR_STATIC_SCRATCH_BYTES;
static __device__ __align__(256) uint8_t g_linear_scratch[kStaticScratchBytes];

std::mutex g_scratch_mu;
std::vector<uint8_t*> g_scratch_addr;  // device address of g_linear_scratch, per device

// Device address of the scratch array on the current device (nullptr with
// *status and an error message on failure).
uint8_t* scratch_on_current_device(cudaStream_t stream, int* status) {
  *status = CONVROT_ERR_CUDA;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) {
    set_error("no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (static_cast<int>(g_scratch_addr.size()) <= dev) g_scratch_addr.resize(dev + 1, nullptr);
  if (g_scratch_addr[dev] == nullptr) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
      set_error("convrot_w4a4_linear_static: the first call on device %d looks up the scratch array's address, "
                "which cannot happen inside a stream capture; make one call outside capture first", dev);
      *status = CONVROT_ERR_UNSUPPORTED;
      return nullptr;
    }
    void* p = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress(&p, g_linear_scratch);
    if (rc != cudaSuccess || p == nullptr) {
      set_error("cudaGetSymbolAddress of the linear scratch array failed on device %d: %s", dev,
                cudaGetErrorString(rc));
      return nullptr;
    }
    g_scratch_addr[dev] = static_cast<uint8_t*>(p);
  }
  return g_scratch_addr[dev];
}

}  // namespace
}  // namespace convrot

extern "C" {

int convrot_w4a4_linear_static(const void* x, int x_dtype, int group_size, const uint8_t* qweight, int layout,
                               const float* wscales, const float* bias, void* out, int out_dtype, int64_t m,
                               int64_t n, int64_t k, void* stream) {
  using namespace convrot;
  CONVROT_REQUIRE(m >= 0 && n > 0 && k > 0, CONVROT_ERR_INVALID, "invalid shape m=%lld n=%lld k=%lld",
                  static_cast<long long>(m), static_cast<long long>(n), static_cast<long long>(k));
  CONVROT_REQUIRE(m < (1LL << 31) && k < (1LL << 31), CONVROT_ERR_UNSUPPORTED, "shape too large");
  const int64_t codes_bytes = (m * k + 255) / 256 * 256;
  const int64_t need = codes_bytes + 4 * m;
  CONVROT_REQUIRE(need <= kStaticScratchBytes, CONVROT_ERR_UNSUPPORTED,
                  "convrot_w4a4_linear_static: m=%lld x k=%lld needs %lld bytes of scratch, more than its fixed "
                  "%lld; use convrot_prepare_i8 + convrot_w4a4_gemm with a caller-provided buffer",
                  static_cast<long long>(m), static_cast<long long>(k), static_cast<long long>(need),
                  static_cast<long long>(kStaticScratchBytes));
  // every check the GEMM would make, before the prep kernel is enqueued: a
  // rejected call enqueues nothing
  const int args_rc = w4a4::check_gemm_args(nullptr, qweight, layout, nullptr, wscales, out, out_dtype, m, n, k,
                                            /*need_act=*/false);
  if (args_rc != CONVROT_OK) return args_rc;
  if (m == 0) return CONVROT_OK;
  int status = CONVROT_OK;
  uint8_t* scratch = scratch_on_current_device(static_cast<cudaStream_t>(stream), &status);
  if (scratch == nullptr) return status;
  int8_t* codes = reinterpret_cast<int8_t*>(scratch);
  float* xscales = reinterpret_cast<float*>(scratch + codes_bytes);
  // Prep writes every code and every scale that the GEMM then reads, so the
  // array's contents from an earlier call never leak into this one.
  int rc = convrot_prepare_i8(x, x_dtype, m, k, group_size, codes, xscales, stream);
  if (rc != CONVROT_OK) return rc;
  return convrot_w4a4_gemm(codes, qweight, layout, xscales, wscales, bias, out, out_dtype, m, n, k, stream);
}

}  // extern "C"
