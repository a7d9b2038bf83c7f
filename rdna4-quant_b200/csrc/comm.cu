// Tensor-parallel exchange over NVLink peer memory: the collective steps of the
// TP decode (all-reduce after o_proj and down_proj, vocabulary gather after
// lm_head) and the standalone all-reduce of expert parallelism.  The
// reference runs on one GPU and has no collectives; the split is new here,
// and r4q/tp_nccl.py keeps an NCCL all-reduce arm of the same step for
// comparison.  Here the producer GEMV's epilogue
// pushes its fp32 partials into every rank's buffer and the consumer GEMV's
// prologue reduces them (tp_exchange.cuh, gemv_tma.cu); this file owns the
// buffers, the peer mappings, the step counter and the kernels for what the
// GEMVs do not fuse: the reduce kernel for consumers that cannot read the
// slots in their prologue, the vocabulary gather, the standalone all-reduce.
//
// Synchronisation.  Decode exchanges with a fused consumer carry tagged
// 64-bit words (epoch << 32 | fp32 bits): a reader polls each word until its
// tag is the exchange's epoch, so there is no fence and no flag.  The other
// exchanges use flags: flags[src] on every rank holds the last epoch rank src
// signalled, published with system-scope stores after a fence, and readers
// wait (acquire, bounded by time) until flags[src] >= e for all src.  Epochs
// only grow (static decode epochs: step counter * 256 + exchange index + 1;
// the standalone all-reduce: completed calls + 1), so a late reader is safe
// against a peer that has already moved on.  Buffers are double-buffered by
// exchange parity; a slot is rewritten by a producer only after that producer
// has consumed the next exchange, which needs every reader to have finished
// reading the slot.  Summation runs in rank order, so every rank computes
// bit-identical replicated activations.
//
// A wait that exceeds ~2 s records R4Q_ERR_TIMEOUT (with the missing ranks) in
// a local status word (r4q_comm_status) and continues, so the context stays
// usable; no kernel spins forever.
#include <cstdio>
#include <cstring>

#include "comm.cuh"
#include "tp_exchange.cuh"
#include "r4q_common.cuh"

struct r4q_comm {
  int rank, world, dev;
  int max_batch, hidden, vocab;
  long sa_cap;
  uint8_t* base;        // this rank's peer-visible allocation
  size_t bytes;
  uint8_t* peer[8];     // every rank's allocation as mapped here (peer[rank] = base)
  bool opened;
  // local control words: [0] standalone seq, [1] standalone done counter,
  // [2] status bits, [3] step counter; then u32 done counters [256] at byte 64
  unsigned long long* ctl;
  size_t off_red, off_gat, off_sa;
  size_t red_slot, sa_slot;  // floats per (parity, src) slot
  int sa_calls;
};

namespace r4q {

namespace {

constexpr int kMaxWorld = 8;

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct SyncArgs {
  unsigned long long* flags_local;         // flags[8] of this rank
  unsigned long long* flags_peer[kMaxWorld];  // flags[8] of each rank (mapped)
  unsigned long long* ctl;                 // local control words
  const unsigned long long* ep_ctr;        // static epochs (step counter) or null
  int ep_idx;
  bool signal;
  int rank, world;
};

constexpr size_t kFlagsX = 0;     // flags of the decode-step exchanges (static epochs)
constexpr size_t kFlagsSA = 64;   // flags of the standalone all-reduce (sequence epochs)

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Signal (block 0) and wait for every rank's signal of this epoch.  Static
// epochs (ep_ctr set): the epoch comes from the step counter and the exchange
// index, and the producers have already signalled (signal = false).
__device__ void comm_sync(const SyncArgs& a, unsigned long long& epoch) {
  __shared__ unsigned long long s_ep;
  if (threadIdx.x == 0)
    s_ep = a.ep_ctr ? *(volatile unsigned long long*)a.ep_ctr * kTpExchangesPerStep + a.ep_idx + 1
                    : *(volatile unsigned long long*)&a.ctl[0] + 1;
  __syncthreads();
  const unsigned long long e = s_ep;
  epoch = e;
  const int t = threadIdx.x;
  if (a.signal && blockIdx.x == 0 && t < a.world) {
    __threadfence_system();  // pushes of earlier kernels are complete; order them first
    st_release_sys(a.flags_peer[t] + a.rank, e);
  }
  if (t < a.world) {
    const unsigned long long t0 = globaltimer();
    unsigned it = 0;
    while (ld_acquire_sys(a.flags_local + t) < e) {
      if ((++it & 63) == 0 && globaltimer() - t0 > 2000000000ull) {
        atomicOr(&a.ctl[2], 1ull << t);
        break;
      }
      __nanosleep(32);
    }
  }
  __syncthreads();
}

// Last block to finish publishes the epoch as completed.
__device__ void comm_done(const SyncArgs& a, unsigned long long e) {
  if (a.ep_ctr) return;
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned long long d = atomicAdd(&a.ctl[1], 1ull);
    if (d == gridDim.x - 1) {
      a.ctl[0] = e;
      a.ctl[1] = 0;
      __threadfence();
    }
  }
}

__global__ void reduce_residual_kernel(const SyncArgs s, const float* __restrict__ red, long slot,
                                       const __half* res, __half* out, float* __restrict__ ss_out,
                                       int B, int D) {
  unsigned long long e;
  comm_sync(s, e);
  const long n = (long)B * D;
  const long i = ((long)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  const bool ok = i < n;
  float sq = 0.0f;
  if (ok) {
    float4 acc = __ldcg(reinterpret_cast<const float4*>(red + i));
    for (int r = 1; r < s.world; ++r) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(red + r * slot + i));
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    float a4[4] = {acc.x, acc.y, acc.z, acc.w};
    __half o4[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float v = __half2float(__float2half(a4[k]));
      if (res) v += __half2float(res[i + k]);
      sq += v * v;
      o4[k] = __float2half(v);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) out[i + k] = o4[k];
  }
  // four consecutive threads hold one 16-element tile (D % 16 == 0)
  sq += __shfl_xor_sync(0xffffffffu, sq, 1);
  sq += __shfl_xor_sync(0xffffffffu, sq, 2);
  if (ok && ss_out && (threadIdx.x & 3) == 0) {
    const int b = (int)(i / D), d = (int)(i - (long)b * D);
    ss_out[(long)(d >> 4) * B + b] = sq;
  }
  comm_done(s, e);
}

__global__ void gather_kernel(const SyncArgs s, const float* __restrict__ gat, __half* __restrict__ out,
                              long n) {
  unsigned long long e;
  comm_sync(s, e);
  for (long i = ((long)blockIdx.x * blockDim.x + threadIdx.x) * 4; i < n; i += (long)gridDim.x * blockDim.x * 4) {
    const float4 v = __ldcg(reinterpret_cast<const float4*>(gat + i));
    out[i] = __float2half(v.x);
    out[i + 1] = __float2half(v.y);
    out[i + 2] = __float2half(v.z);
    out[i + 3] = __float2half(v.w);
  }
  comm_done(s, e);
}

// Standalone all-reduce (the expert-parallel MoE sum), flag-free: every
// element travels as one 64-bit word (epoch << 32 | fp32 bits), so a reader
// knows an element has arrived from the element itself — no fence, no flag
// (each system-scope fence or release store cost ~5 us on B200).  The epoch
// is this rank's count of completed all-reduces + 1, the same on every rank.
// Step 1: push x into slot [rank] of every rank.
struct PushTable {
  unsigned long long* p[kMaxWorld];
};

__global__ void push_kernel_t(const float* __restrict__ x, const PushTable t, int world, long n,
                              const unsigned long long* ctl) {
  const unsigned long long e = (*(volatile const unsigned long long*)&ctl[0] + 1ull) & 0xffffffffull;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const unsigned long long w = (e << 32) | (unsigned long long)__float_as_uint(x[i]);
    for (int r = 0; r < world; ++r)
      asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(t.p[r] + i), "l"(w) : "memory");
  }
}

// Step 2: y = sum over src in rank order, each element waited for (bounded
// by ~2 s of wall time, then the missing rank is recorded and 0 used).
__global__ void sum_kernel(const SyncArgs s, const unsigned long long* sa, long slot, float* __restrict__ y,
                           long n) {
  __shared__ unsigned long long s_ep;
  if (threadIdx.x == 0) s_ep = *(volatile unsigned long long*)&s.ctl[0] + 1ull;
  __syncthreads();
  const unsigned long long e = s_ep;
  const unsigned long long tag = e & 0xffffffffull;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    float v = 0.0f;
    for (int r = 0; r < s.world; ++r) {
      unsigned long long w;
      const unsigned long long* a = sa + r * slot + i;
      asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(a) : "memory");
      if ((w >> 32) != tag && !((*(volatile unsigned long long*)&s.ctl[2] >> r) & 1ull)) {
        // (a rank that already timed out in this call is not waited for again)
        const unsigned long long t0 = globaltimer();
        unsigned it = 0;
        for (;;) {
          __nanosleep(32);
          asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(a) : "memory");
          if ((w >> 32) == tag) break;
          if ((++it & 63) == 0 && globaltimer() - t0 > 2000000000ull) {
            atomicOr(&s.ctl[2], 1ull << r);
            w = 0;
            break;
          }
        }
      }
      if ((w >> 32) != tag) w = 0;
      const float f = __uint_as_float((unsigned)(w & 0xffffffffull));
      v = r == 0 ? f : v + f;
    }
    y[i] = v;
  }
  comm_done(s, e);
}

SyncArgs sync_args(r4q_comm* c, size_t flags_off, int ep_idx, bool static_epoch) {
  SyncArgs a{};
  a.flags_local = reinterpret_cast<unsigned long long*>(c->base + flags_off);
  for (int r = 0; r < c->world; ++r)
    a.flags_peer[r] = reinterpret_cast<unsigned long long*>(c->peer[r] + flags_off);
  a.ctl = c->ctl;
  a.ep_ctr = static_epoch ? c->ctl + 3 : nullptr;
  a.ep_idx = ep_idx;
  a.signal = !static_epoch;
  a.rank = c->rank;
  a.world = c->world;
  return a;
}

__global__ void tick_kernel(unsigned long long* ctr) { *ctr += 1ull; }

}  // namespace

float* comm_reduce_slot(r4q_comm* c, int peer, int parity, bool ll) {
  const size_t i = ((size_t)(parity & 1) * c->world + c->rank) * c->red_slot;
  if (ll) return reinterpret_cast<float*>(reinterpret_cast<unsigned long long*>(c->peer[peer] + c->off_red) + i);
  return reinterpret_cast<float*>(c->peer[peer] + c->off_red) + i;
}
float* comm_gather_base(r4q_comm* c, int peer) {
  return reinterpret_cast<float*>(c->peer[peer] + c->off_gat);
}
int comm_rank(const r4q_comm* c) { return c->rank; }
int comm_world(const r4q_comm* c) { return c->world; }
int comm_vocab(const r4q_comm* c) { return c->vocab; }
int comm_max_batch(const r4q_comm* c) { return c->max_batch; }
int comm_hidden(const r4q_comm* c) { return c->hidden; }

void comm_fill_signal(r4q_comm* c, TpExchange& x, int idx) {
  for (int q = 0; q < c->world; ++q)
    x.sig[q] = reinterpret_cast<unsigned long long*>(c->peer[q] + kFlagsX) + c->rank;
  x.nsig = c->world;
  x.sig_idx = idx;
  x.sig_done = reinterpret_cast<unsigned*>(reinterpret_cast<uint8_t*>(c->ctl) + 64) + idx;
  x.ep_ctr = c->ctl + 3;
  x.status = c->ctl + 2;
}

void comm_fill_wait(r4q_comm* c, TpExchange& x, int idx, int parity, const __half* res, __half* out, bool ll) {
  x.wait_flags = reinterpret_cast<const unsigned long long*>(c->base + kFlagsX);
  x.nwait = c->world;
  x.wait_idx = idx;
  x.ll_wait = ll ? 1 : 0;
  const size_t i = (size_t)(parity & 1) * c->world * c->red_slot;
  x.red = ll ? reinterpret_cast<const float*>(reinterpret_cast<const unsigned long long*>(c->base + c->off_red) + i)
             : reinterpret_cast<const float*>(c->base + c->off_red) + i;
  x.red_slot = (long)c->red_slot;
  x.red_res = res;
  x.red_out = out;
  x.ep_ctr = c->ctl + 3;
  x.status = c->ctl + 2;
}

int comm_tick(r4q_comm* c, cudaStream_t st) {
  tick_kernel<<<1, 1, 0, st>>>(c->ctl + 3);
  return check_launch("tick_kernel");
}

int comm_reduce_residual(r4q_comm* c, int idx, int parity, const __half* res, __half* out, float* ss_out,
                         int B, int D, cudaStream_t st) {
  if (!c->opened) return set_error(R4Q_ERR_ARG, "comm: peers not opened");
  if (B > c->max_batch || D != c->hidden || D % 16)
    return set_error(R4Q_ERR_CAPACITY, "comm reduce: B=%d D=%d exceeds the comm (%d, %d)", B, D,
                     c->max_batch, c->hidden);
  const float* red = reinterpret_cast<const float*>(c->base + c->off_red) +
                     (size_t)(parity & 1) * c->world * c->red_slot;
  const long n = (long)B * D;
  const int thr = 256;
  const int grid = (int)((n / 4 + thr - 1) / thr);
  reduce_residual_kernel<<<grid, thr, 0, st>>>(sync_args(c, kFlagsX, idx, true), red, (long)c->red_slot,
                                                res, out, ss_out, B, D);
  return check_launch("reduce_residual_kernel");
}

int comm_gather_logits(r4q_comm* c, int idx, __half* logits, int B, cudaStream_t st) {
  if (!c->opened) return set_error(R4Q_ERR_ARG, "comm: peers not opened");
  if (B > c->max_batch) return set_error(R4Q_ERR_CAPACITY, "comm gather: B=%d > %d", B, c->max_batch);
  const long n = (long)B * c->vocab;
  int grid = (int)((n / 4 + 255) / 256);
  if (grid > 4 * num_sms()) grid = 4 * num_sms();
  gather_kernel<<<grid, 256, 0, st>>>(sync_args(c, kFlagsX, idx, true),
                                      reinterpret_cast<const float*>(c->base + c->off_gat), logits, n);
  return check_launch("gather_kernel");
}

}  // namespace r4q

using namespace r4q;

extern "C" int r4q_comm_create(int rank, int world, int max_batch, int hidden, int vocab, long sa_cap,
                               r4q_comm** out, void* handle_out) {
  if (!out || !handle_out || world < 1 || world > kMaxWorld || rank < 0 || rank >= world ||
      max_batch < 1 || hidden < 16 || hidden % 16 || vocab < 0 || vocab % 4 || sa_cap < 0)
    return set_error(R4Q_ERR_ARG, "comm_create: bad arguments (rank %d world %d B %d D %d V %d)", rank,
                     world, max_batch, hidden, vocab);
  r4q_comm* c = new r4q_comm();
  c->rank = rank;
  c->world = world;
  c->max_batch = max_batch;
  c->hidden = hidden;
  c->vocab = vocab;
  c->sa_cap = (sa_cap + 63) & ~63L;
  cudaGetDevice(&c->dev);
  c->red_slot = align256((size_t)max_batch * hidden * 4) / 4;
  c->sa_slot = (size_t)c->sa_cap;
  c->off_red = 256;
  c->off_gat = c->off_red + 2 * world * c->red_slot * 8;   // room for tagged 64-bit words
  c->off_sa = c->off_gat + align256((size_t)max_batch * vocab * 4);
  c->bytes = c->off_sa + 2 * world * c->sa_slot * 8 + 256;     // all-reduce words: epoch | fp32
  cudaError_t e = cudaMalloc(&c->base, c->bytes);
  if (e == cudaSuccess) e = cudaMemset(c->base, 0, c->bytes);
  if (e == cudaSuccess) e = cudaMalloc(&c->ctl, 64 + 4 * kTpExchangesPerStep);
  if (e == cudaSuccess) e = cudaMemset(c->ctl, 0, 64 + 4 * kTpExchangesPerStep);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->base);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (c->base) cudaFree(c->base);
    if (c->ctl) cudaFree(c->ctl);
    delete c;
    return set_error(R4Q_ERR_CUDA, "comm_create: %s", cudaGetErrorString(e));
  }
  static_assert(sizeof(cudaIpcMemHandle_t) <= R4Q_COMM_HANDLE_BYTES, "IPC handle size");
  memset(handle_out, 0, R4Q_COMM_HANDLE_BYTES);
  memcpy(handle_out, &h, sizeof(h));
  c->peer[rank] = c->base;
  if (world == 1) c->opened = true;
  *out = c;
  return R4Q_OK;
}

extern "C" int r4q_comm_open(r4q_comm* c, const void* handles) {
  if (!c || !handles) return set_error(R4Q_ERR_ARG, "comm_open: null argument");
  if (c->opened) return R4Q_OK;
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)r * R4Q_COMM_HANDLE_BYTES, sizeof(h));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (q != c->rank && c->peer[q]) {
          cudaIpcCloseMemHandle(c->peer[q]);
          c->peer[q] = nullptr;
        }
      return set_error(R4Q_ERR_CUDA, "comm_open: rank %d: %s", r, cudaGetErrorString(e));
    }
    c->peer[r] = static_cast<uint8_t*>(p);
  }
  c->opened = true;
  return R4Q_OK;
}

extern "C" int r4q_comm_status(r4q_comm* c) {
  if (!c) return set_error(R4Q_ERR_ARG, "comm_status: null comm");
  unsigned long long bits = 0;
  cudaError_t e = cudaMemcpy(&bits, c->ctl + 2, 8, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return set_error(R4Q_ERR_CUDA, "comm_status: %s", cudaGetErrorString(e));
  if (bits) {
    char who[64] = "";
    int n = 0;
    for (int r = 0; r < c->world && n < 60; ++r)
      if (bits >> r & 1) n += snprintf(who + n, sizeof(who) - n, "%s%d", n ? "," : "", r);
    return set_error(R4Q_ERR_TIMEOUT, "comm: timed out waiting for rank(s) %s", who);
  }
  return R4Q_OK;
}

extern "C" int r4q_comm_clear_status(r4q_comm* c) {
  if (!c) return set_error(R4Q_ERR_ARG, "comm_clear_status: null comm");
  cudaError_t e = cudaMemset(c->ctl + 2, 0, 8);
  return e == cudaSuccess ? R4Q_OK : set_error(R4Q_ERR_CUDA, "comm_clear_status: %s", cudaGetErrorString(e));
}

extern "C" int r4q_comm_allreduce_f32(r4q_comm* c, const float* x, float* y, long n, void* stream) {
  if (!c || !x || !y || n < 0) return set_error(R4Q_ERR_ARG, "comm_allreduce: bad arguments");
  if (!c->opened) return set_error(R4Q_ERR_ARG, "comm_allreduce: peers not opened");
  if (n > c->sa_cap)
    return set_error(R4Q_ERR_CAPACITY, "comm_allreduce: %ld elements > capacity %ld", n, c->sa_cap);
  cudaStream_t st = (cudaStream_t)stream;
  const int par = c->sa_calls & 1;
  c->sa_calls++;
  PushTable t{};
  for (int r = 0; r < c->world; ++r)
    t.p[r] = reinterpret_cast<unsigned long long*>(c->peer[r] + c->off_sa) +
             ((size_t)par * c->world + c->rank) * c->sa_slot;
  int grid = (int)((n + 255) / 256);
  if (grid > 2 * num_sms()) grid = 2 * num_sms();
  if (grid < 1) grid = 1;
  push_kernel_t<<<grid, 256, 0, st>>>(x, t, c->world, n, c->ctl);
  int rc = check_launch("push_kernel");
  if (rc) return rc;
  const unsigned long long* sa =
      reinterpret_cast<const unsigned long long*>(c->base + c->off_sa) + (size_t)par * c->world * c->sa_slot;
  sum_kernel<<<grid, 256, 0, st>>>(sync_args(c, kFlagsSA, 0, false), sa, (long)c->sa_slot, y, n);
  return check_launch("sum_kernel");
}

extern "C" void r4q_comm_destroy(r4q_comm* c) {
  if (!c) return;
  cudaDeviceSynchronize();
  for (int r = 0; r < c->world; ++r)
    if (r != c->rank && c->peer[r]) cudaIpcCloseMemHandle(c->peer[r]);
  if (c->base) cudaFree(c->base);
  if (c->ctl) cudaFree(c->ctl);
  delete c;
}
