// Tensor-parallel exchange over NVLink peer memory (internal interface).
//
// Each rank owns one peer-visible allocation (cudaMalloc + CUDA IPC handle);
// every rank maps every other rank's allocation.  Producers (the GEMV
// epilogues) push their fp32 partial outputs straight into the destination
// ranks' buffers; a small sync kernel then signals the peers, waits for their
// signals (bounded) and reduces/gathers from local memory only.
//
// Allocation layout (offsets 256-byte aligned):
//   flags   u64 [8]                       flags[src] = last epoch src signalled
//   red     f32 [2][world][max_batch*hidden]   all-reduce slots, double-buffered
//   gat     f32 [max_batch][vocab]         lm_head gather
//   sa      f32 [2][world][sa_cap]          standalone all-reduce slots
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/r4q.h"
#include "tp_exchange.cuh"

namespace r4q {

// Base of rank `rank`'s all-reduce slot inside peer `peer`'s buffer (parity 0/1):
// [max_batch * hidden] elements, row stride `hidden` — floats, or with `ll`
// 64-bit tagged words (the pointer is then indexed as unsigned long long).
float* comm_reduce_slot(r4q_comm* c, int peer, int parity, bool ll = false);
// Base of peer `peer`'s gather buffer [max_batch][vocab].
float* comm_gather_base(r4q_comm* c, int peer);
int comm_rank(const r4q_comm* c);
int comm_world(const r4q_comm* c);
int comm_vocab(const r4q_comm* c);
int comm_max_batch(const r4q_comm* c);
int comm_hidden(const r4q_comm* c);

// Decode-step exchanges use static epochs (step counter * 256 + index + 1);
// the producer GEMVs signal (comm_fill_signal), consumers wait.
void comm_fill_signal(r4q_comm* c, TpExchange& x, int idx);
// Consumer GEMV prologue: wait for exchange idx, read reduce slots of `parity`,
// r = fp16(fp16(sum) + res) (res [B][hidden]); CTA 0 stores r to out.
// ll: the producer pushed tagged words (no flag to wait for).
void comm_fill_wait(r4q_comm* c, TpExchange& x, int idx, int parity, const __half* res, __half* out,
                    bool ll = false);
// Advance the step counter (once at the start of every decode step).
int comm_tick(r4q_comm* c, cudaStream_t st);
// Stand-alone consumer of exchange idx: out[b, d] = fp16(fp16(sum_src
// red[parity][src][b, d]) + res[b, d]) (res may alias out), ss_out[d/16][b] =
// sum of squares of the unrounded values.
int comm_reduce_residual(r4q_comm* c, int idx, int parity, const __half* res, __half* out, float* ss_out,
                         int B, int D, cudaStream_t st);
// logits[b, v] = fp16(gat[b, v]) once exchange idx (every rank's vocabulary
// slice) has arrived.
int comm_gather_logits(r4q_comm* c, int idx, __half* logits, int B, cudaStream_t st);

}  // namespace r4q
