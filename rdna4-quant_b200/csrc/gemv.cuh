// Internal GEMV launcher interface shared by the C ABI and the decode step.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>

#include "tp_exchange.cuh"

namespace r4q {

enum WFmt { W_INT4 = 0, W_INT8 = 1, W_FP16 = 2 };

struct GemvArgs {
  const void* x;
  long ldx;
  const void* w;
  const void* s;
  void* y;
  long ldy;
  int B, N, K;
  int prologue;
  void* ws;
  size_t ws_bytes;
  cudaStream_t stream;
  // fused RMSNorm prologue / residual epilogue (all optional)
  const void* norm_w;
  float eps;
  const float* ss_in;
  int ss_in_parts;
  const void* res;
  long ldres;
  float* ss_out;
  // fp32 sums to npush arrays (local or peer memory) instead of fp16 y
  float* y32p[8];
  int npush;
  // tensor-parallel exchange: signal after the pushes / reduce-on-read prologue
  TpExchange tpx;
};

// GEMV workspace: status word in a 256-byte header, tile counters, partials.
constexpr size_t kGemvHdrBytes = 256;
size_t gemv_cnt_bytes(int N);  // offset of the partials (header + counters)
unsigned* gemv_counters(void* ws);
// Polls before a bounded mbarrier wait of the TMA GEMV gives up (test hook:
// gemv_set_spin_limit lowers it; <= 0 restores the default).  Returns the old value.
long gemv_spin_limit();
long gemv_set_spin_limit(long polls);
// 2-D byte tensor map [rows, row_bytes] with box [box_rows, box_bytes] (TMA).
int make_map(CUtensorMap* m, const void* base, long rows, long row_bytes, int box_bytes, int box_rows,
             CUtensorMapSwizzle sw);
// Device address of r4q_gemv_int4_noalloc's static scratch on the current device.
int noalloc_scratch(void** out);
size_t gemv_ws_bytes_for(int B, int N, int ksplit);
int gemv_validate(const GemvArgs& a, int fmt);
int launch_gemv(const GemvArgs& a, int fmt);
bool gemv_tma_supported(const GemvArgs& a, int fmt);
int launch_gemv_tma(const GemvArgs& a, int fmt);
// tcgen05 GEMV for INT4 at B = 3..16 (gemv_tc.cu): eligibility, launch
// (R4Q_ERR_CAPACITY without an error message when the workspace is too small),
// and the workspace bytes it needs beyond the split-K partials.
bool gemv_tc_eligible(const GemvArgs& a, int fmt);
int launch_gemv_tc(const GemvArgs& a);
size_t gemv_tc_extra_bytes(int B, int K);

}  // namespace r4q
