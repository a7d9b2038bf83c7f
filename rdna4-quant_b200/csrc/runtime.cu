// Host runtime pieces shared by every entry point: error reporting, device
// queries, version.
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <vector>

#include "r4q_common.cuh"

namespace r4q {

static thread_local char g_err[512] = "";

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return status;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(R4Q_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return R4Q_OK;
}

int num_sms() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
  if (!cache[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 1;
  }
  return cache[dev];
}

}  // namespace r4q

extern "C" const char* r4q_last_error(void) { return r4q::g_err; }
extern "C" int r4q_version(void) { return 100; }
