// Host runtime pieces shared by every entry point: error reporting, device
// queries, version.
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <vector>

#include "gemv.cuh"
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

// Status word 0 of a GEMV / GEMM / attention workspace (NULL: the static
// scratch of r4q_gemv_int4_noalloc on the current device).
extern "C" int r4q_ws_status(const void* ws, int clear, void* stream) {
  using namespace r4q;
  void* w = const_cast<void*>(ws);
  if (!w) {
    const int st = noalloc_scratch(&w);
    if (st) return st;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, w, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && v && clear) {
    e = cudaMemsetAsync(w, 0, sizeof(int), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(R4Q_ERR_CUDA, "ws_status: %s", cudaGetErrorString(e));
  }
  if (v) return set_error(R4Q_ERR_TIMEOUT, "a bounded device-side wait gave up (status word %d): "
                          "the outputs of the kernels since the last check are not valid", v);
  return R4Q_OK;
}

extern "C" long r4q_debug_spin_limit(long polls) { return r4q::gemv_set_spin_limit(polls); }
extern "C" int r4q_version(void) { return 100; }
