// Status handling shared by every entry point of libconvrot_b200.so.
#include <mutex>
#include <vector>

#include "common.cuh"

namespace convrot {

static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    set_error("%s: kernel launch failed: %s", what, cudaGetErrorString(err));
    return CONVROT_ERR_CUDA;
  }
  return CONVROT_OK;
}

int device_sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace convrot

extern "C" {

int convrot_abi_version(void) { return CONVROT_ABI_VERSION; }

const char* convrot_last_error(void) { return convrot::g_last_error; }

}  // extern "C"
