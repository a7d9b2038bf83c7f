// INT4 GEMV entry point that allocates no device memory.
//
// Some callers cannot call cudaMalloc at all: code running inside a CUDA
// stream capture that must not allocate, plugins loaded into a host process
// whose allocator owns all device memory (and forbids others from taking
// more), and callers that must have a fixed, known device footprint.  For
// them, r4q_gemv_int4_noalloc uses the split-K scratch held in the file-scope
// array below instead of a caller-provided workspace.  Everything else is the
// same kernel as r4q_gemv_int4.
#include <mutex>

#include "gemv.cuh"
#include "r4q_common.cuh"

namespace r4q {

// Scratch: the GEMV workspace layout — a 256-byte header (status word), 64 KiB
// of tile counters, then fp32 split-K partials.  Every GPU that loads the
// library holds this array until exit.
constexpr size_t kNoAllocCounterBytes = kGemvHdrBytes + 64 * 1024;
constexpr size_t kNoAllocPartialBytes = 4 * 1024 * 1024;
constexpr size_t kNoAllocBytes = kNoAllocCounterBytes + kNoAllocPartialBytes;
// Largest B * N accepted: a two-way K split of one call must fit the partials.
constexpr long kNoAllocMaxBN = (long)(kNoAllocPartialBytes / (2 * sizeof(float)));

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

// Device address of the scratch on the current device.  Host code may not use
// the symbol g_noalloc_scratch as a pointer (it names a host-side shadow), so
// the address is looked up once per device with that device current.
int noalloc_scratch(void** out) {
  static std::mutex mu;
  static void* addr[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(R4Q_ERR_CUDA, "gemv_int4_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(R4Q_ERR_ARG, "gemv_int4_noalloc: device %d unsupported", dev);
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      return set_error(R4Q_ERR_CUDA, "gemv_int4_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    }
    addr[dev] = p;
  }
  *out = addr[dev];
  return R4Q_OK;
}

}  // namespace r4q

using namespace r4q;

extern "C" int r4q_gemv_int4_noalloc(const void* x, long ldx, const void* w, const void* sz,
                                     void* y, long ldy, int B, int N, int K, int prologue,
                                     void* stream) {
  if ((long)B * N > kNoAllocMaxBN)
    return set_error(R4Q_ERR_CAPACITY,
                     "gemv_int4_noalloc: B*N = %ld exceeds the static scratch limit %ld "
                     "(use r4q_gemv_int4 with a workspace)", (long)B * N, kNoAllocMaxBN);
  void* ws = nullptr;
  int st = noalloc_scratch(&ws);
  if (st) return st;
  // Calls share the array and it keeps the previous call's contents: the tile
  // counters must start at zero, so clear them on the stream.  The status word
  // is left alone: a timeout stays recorded until r4q_ws_status(NULL, 1, ...)
  // reads and clears it.
  cudaError_t e = cudaMemsetAsync(static_cast<unsigned char*>(ws) + kGemvHdrBytes, 0,
                                  kNoAllocCounterBytes - kGemvHdrBytes, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(R4Q_ERR_CUDA, "gemv_int4_noalloc: clearing scratch: %s", cudaGetErrorString(e));
  }
  GemvArgs a{};
  a.x = x; a.ldx = ldx; a.w = w; a.s = sz; a.y = y; a.ldy = ldy;
  a.B = B; a.N = N; a.K = K; a.prologue = prologue;
  a.ws = ws;
  a.ws_bytes = kNoAllocBytes;
  a.stream = reinterpret_cast<cudaStream_t>(stream);
  return launch_gemv(a, W_INT4);
}
