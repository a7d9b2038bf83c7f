// Tensor-parallel exchange fused into the GEMVs (device side).
//
// Producer GEMV (o_proj, down_proj, lm_head under TP): its epilogue pushes the
// fp32 partial sums into every rank's exchange buffer (GemvParams::y32p); at
// kernel exit every CTA fences its pushes at system scope and the last CTA to
// finish stores the exchange's epoch into flags[rank] of every rank.
//
// Consumer GEMV (gate_up after o_proj, the next layer's qkv or the lm_head
// after down_proj): after griddepcontrol.wait — i.e. while its producer warp
// already streams weights — it waits (bounded) until flags[src] >= epoch for
// every src, then builds its RMSNorm+FWHT input straight from the exchange
// buffer: r = fp16(fp16(sum over src in rank order) + residual), every CTA
// computing the sum of squares itself; CTA 0 also stores r (the residual
// stream).  The separate all-reduce kernel disappears from the step.
//
// Epochs are static: epoch = step_counter * 256 + exchange index + 1, where
// the step counter (one per comm, shared by every context on it) is ticked
// once at the start of each step, so epochs only grow and a stale flag can
// never satisfy a wait.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace r4q {

constexpr int kTpMaxWorld = 8;
constexpr int kTpExchangesPerStep = 256;

struct TpExchange {
  // producer side
  unsigned long long* sig[kTpMaxWorld];  // &flags[rank] inside every rank's buffer
  unsigned* sig_done;                    // CTA-completion counter of this exchange (left zero)
  int nsig;                              // ranks to signal (0: no signal)
  int sig_idx;
  int ll_sig;                            // pushes are tagged words (epoch << 32 | fp32): no fence, no flag
  // consumer side
  const unsigned long long* wait_flags;  // this rank's flags[world]
  int nwait;                             // ranks to wait for (0: not a TP consumer)
  int wait_idx;
  int ll_wait;                           // the slots hold tagged words: poll them instead of the flags
  const float* red;                      // reduce slots of this parity: [world][red_slot]
  long red_slot;                         // floats per slot; row b of a slot at b * K
  const __half* red_res;                 // residual added to the reduced sum ([B][K])
  __half* red_out;                       // fp16(sum) + residual, written by CTA 0 (or null)
  // both
  const unsigned long long* ep_ctr;      // step counter
  unsigned long long* status;            // timeout bits (one per rank waited for)
  // optional timeline (R4Q_TP_TRACE): u64 [8][256] global-timer stamps per
  // exchange index: 0 producer compute start, 1 producer signal, 2 consumer
  // wait start, 3 consumer wait end, 4 consumer input staged, 5 producer
  // entry, 6 producer CTA 0 done, 7 producer's last CTA arrived
  unsigned long long* trace;
};

#ifdef __CUDACC__
__device__ __forceinline__ unsigned long long tp_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void tp_stamp(const TpExchange& x, int ev, int idx) {
  if (x.trace && idx >= 0 && idx < kTpExchangesPerStep) x.trace[ev * kTpExchangesPerStep + idx] = tp_now();
}

__device__ __forceinline__ unsigned long long tp_epoch(const TpExchange& x, int idx) {
  const unsigned long long c = *reinterpret_cast<const volatile unsigned long long*>(x.ep_ctr);
  return c * (unsigned long long)kTpExchangesPerStep + (unsigned long long)idx + 1ull;
}

// Tagged exchange words (ll_sig / ll_wait): each pushed element is one 64-bit
// word, epoch << 32 | fp32 bits, stored with a single-copy-atomic 64-bit
// store; the reader knows an element has arrived from its own tag, so the
// producer needs neither a fence nor a flag (each system-scope fence or
// release store cost ~5 us on B200).
__device__ __forceinline__ unsigned long long tp_word(unsigned tag, float v) {
  return ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(v);
}
// element i of a tagged slot whose base is given as float* (the push table's type)
__device__ __forceinline__ void tp_push_word(float* base, long i, unsigned tag, float v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(reinterpret_cast<unsigned long long*>(base) + i),
               "l"(tp_word(tag, v))
               : "memory");
}
// Element i of a tagged slot (unsigned long long words), waited for until its
// tag matches (bounded by ~2 s, then the rank's status bit and 0).
__device__ __forceinline__ float tp_read_word(const TpExchange& x, const float* slot_base, long i, unsigned tag,
                                              int src) {
  const unsigned long long* a = reinterpret_cast<const unsigned long long*>(slot_base) + i;
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(a) : "memory");
  if ((unsigned)(w >> 32) != tag) {
    unsigned long long t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    unsigned it = 0;
    for (;;) {
      if ((*reinterpret_cast<volatile const unsigned long long*>(x.status) >> src) & 1ull) break;
      __nanosleep(32);
      asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(a) : "memory");
      if ((unsigned)(w >> 32) == tag) break;
      if ((++it & 63) == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        if (t - t0 > 2000000000ull) {
          atomicOr(x.status, 1ull << src);
          break;
        }
      }
    }
    if ((unsigned)(w >> 32) != tag) w = 0;
  }
  return __uint_as_float((unsigned)w);
}

// Lanes 0..nwait-1 of one warp each wait for one rank; bounded by ~2 s of
// wall time, after which the missing rank is recorded in `status`.
__device__ __forceinline__ void tp_wait_lane(const TpExchange& x, int lane) {
  if (lane >= x.nwait) return;
  const unsigned long long e = tp_epoch(x, x.wait_idx);
  unsigned long long t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  unsigned it = 0;
  for (;;) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(x.wait_flags + lane) : "memory");
    if (v >= e) break;
    if ((++it & 63) == 0) {
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > 2000000000ull) {
        atomicOr(x.status, 1ull << lane);
        break;
      }
    }
    __nanosleep(32);
  }
}

// One thread per CTA, after a CTA-wide barrier that follows every thread's
// pushes: a system-scope acq_rel fence (cumulative over the writes the
// barrier made visible to this thread; it completes once those pushes are
// performed at system scope), then the gpu-scope counter.  The last CTA to
// arrive therefore finds every CTA's pushes already performed system-wide and
// publishes the epoch to all ranks with plain system-scope stores.  Measured
// on B200 (2 GPUs): each fence.sc.sys, and each st.release.sys, cost ~5 us
// here — against an exchange whose data moves in ~1 us.
__device__ __forceinline__ void tp_signal_cta(const TpExchange& x) {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(x.sig_done) : "memory");
  if (old != gridDim.x * gridDim.y * gridDim.z - 1) return;
  tp_stamp(x, 7, x.sig_idx);
  *x.sig_done = 0u;
  // the other CTAs' pushes were released to this thread by the counter (gpu
  // scope); this fence makes them cumulative into the system-scope flag
  // stores below (one fence per exchange, in the last CTA only)
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  const unsigned long long e = tp_epoch(x, x.sig_idx);
  for (int q = 0; q < x.nsig; ++q)
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(x.sig[q]), "l"(e) : "memory");
  tp_stamp(x, 1, x.sig_idx);
}
#endif

}  // namespace r4q
