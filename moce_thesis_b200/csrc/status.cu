// Status strings and small host utilities of the C ABI.
#include <cstdarg>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace moce {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess)
    return set_error(MOCE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
  return MOCE_OK;
}

int num_sms() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace moce

extern "C" const char* moce_last_error(void) { return moce::g_last_error; }

extern "C" const char* moce_version(void) { return "moce_b200 0.1.0 (sm_100a)"; }
