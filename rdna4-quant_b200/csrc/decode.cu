// Decode-step runtime: the whole transformer decode step on one GPU.
//
// Replaces int4_decode_step / int4_decode_step_logits and the graph benchmark
// (int4_decode_step.hip:2325-2595, 2801-3041).  Per layer (B rows share pos):
//   1. qkv   = GEMV(in_norm, prologue RMSNorm+FWHT of h; rrms from the sums of
//              squares the previous down-proj wrote, or from h itself on layer 0)
//   2. q, k  <- per-head RMSNorm + RoPE(pos); K, V -> FP8 cache at pos
//   3. attn  = flash-decode over positions [0, pos] with the FWHT epilogue
//   4. r     = GEMV_o(attn) + h      (residual epilogue + sums of squares)
//   5. gu    = GEMV_gate_up(RMSNorm+FWHT of r with post_norm)
//   6. h     = GEMV_down(FWHT(silu(g) * u)) + r   (residual epilogue + ss)
// then logits = GEMV_lm(RMSNorm+FWHT of h with final_norm, rrms from the fp16
// h as the reference's final fused_rmsnorm_fwht does).
//
// The context owns every scratch buffer; one call enqueues the step on the
// caller's stream.  With use_graph the step is captured once into a CUDA graph
// (positions come from a device scalar, so one graph serves every token) and
// replayed.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "attention.cuh"
#include "comm.cuh"
#include "gemv.cuh"
#include "r4q_common.cuh"

struct r4q_decode_ctx {
  r4q_model_desc m;
  std::vector<r4q_layer_desc> layers;
  int dev;
  // scratch
  __half *h_in, *h, *r, *qkv, *attn, *gu, *logits, *h_out;
  float *ss_post, *ss_h;
  long long* pos_dev;   // [B] position of the token being decoded
  long long* seq_dev;   // [B] pos + 1
  void* gemv_ws;
  size_t gemv_ws_bytes;
  void* attn_ws;
  size_t attn_ws_bytes;
  // graph cache
  cudaStream_t cap_stream;
  cudaGraphExec_t graph[3];  // [without lm_head, with lm_head, greedy token (+ argmax, embedding)]
  // greedy loop state
  long long* tok_hist;       // [B][max_seq] token chosen at each position
  void* am_ws;               // argmax partials [B][kArgmaxBlocks] + counters
  const void* loop_embed;    // embedding table the token graph was captured with
  // decode_profile: events around kernel groups (cat 0 gemv, 1 attention, 2 norm)
  struct ProfEv {
    cudaEvent_t a, b;
    int cat;
  };
  bool prof;
  std::vector<ProfEv> prof_ev;
  unsigned long long* tp_trace;  // R4Q_TP_TRACE: exchange timeline u64 [8][256]
};

namespace r4q {

__global__ void set_positions(long long* pos, long long* seq, int B, int p) {
  const int i = threadIdx.x;
  if (i < B) {
    pos[i] = p;
    seq[i] = p + 1;
  }
}

static int gemv_call(r4q_decode_ctx* c, int fmt, const void* w, const void* s, const void* x, void* y,
                     int N, int K, int prologue, const void* norm_w, const float* ss_in, int ss_parts,
                     const void* res, float* ss_out, cudaStream_t st, float* const* push = nullptr,
                     int npush = 0, long ld_push = 0, const TpExchange* tpx = nullptr) {
  GemvArgs a{};
  a.x = x;
  a.ldx = (prologue == R4Q_PRO_SILU_FWHT) ? 2L * K : K;
  a.w = w;
  a.s = s;
  a.y = y;
  a.ldy = N;
  a.B = c->m.batch;
  a.N = N;
  a.K = K;
  a.prologue = prologue;
  a.ws = c->gemv_ws;
  a.ws_bytes = c->gemv_ws_bytes;
  a.stream = st;
  a.norm_w = norm_w;
  a.eps = c->m.rms_eps;
  a.ss_in = ss_in;
  a.ss_in_parts = ss_parts;
  a.res = res;
  a.ldres = N;
  a.ss_out = ss_out;
  if (npush) {  // fp32 partial sums straight into every rank's exchange buffer
    a.npush = npush;
    for (int q = 0; q < npush; ++q) a.y32p[q] = push[q];
    a.ldy = ld_push;
  }
  if (tpx) {
    a.tpx = *tpx;
    a.tpx.trace = c->tp_trace;

  }
  return launch_gemv(a, fmt);
}

// decode_profile: events around one kernel group when the context profiles
struct ProfScope {
  r4q_decode_ctx* c;
  cudaStream_t st;
  cudaEvent_t a = nullptr;
  int cat;
  ProfScope(r4q_decode_ctx* c_, int cat_, cudaStream_t st_) : c(c_), st(st_), cat(cat_) {
    if (!c->prof) return;
    cudaEventCreate(&a);
    cudaEventRecord(a, st);
  }
  ~ProfScope() {
    if (!a) return;
    cudaEvent_t b;
    cudaEventCreate(&b);
    cudaEventRecord(b, st);
    c->prof_ev.push_back({a, b, cat});
  }
};

// ------------------------------------------------------------ greedy loop
// argmax over fp16 logits [B][V] (first index of the maximum, NaN skipped —
// torch.argmax on the logits the reference's decode_loop takes), then the
// embedding row of the chosen token becomes the next step's input.
constexpr int kArgmaxBlocks = 64;

__device__ __forceinline__ bool am_better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

__global__ void argmax_kernel(const __half* __restrict__ logits, int V, float2* part, unsigned* cnt,
                              long long* tok_hist, int max_seq, const long long* pos_dev) {
  const int b = blockIdx.y;
  const __half* lr = logits + (long)b * V;
  const int per = (V + gridDim.x - 1) / gridDim.x;
  const int lo = blockIdx.x * per, hi = min(V, lo + per);
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const float v = __half2float(lr[i]);
    if (v == v && am_better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (am_better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ bool s_last;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sv[w] = bv;
    si[w] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < (int)(blockDim.x >> 5); ++k)
      if (am_better(sv[k], si[k], bv, bi)) {
        bv = sv[k];
        bi = si[k];
      }
    part[b * gridDim.x + blockIdx.x] = make_float2(bv, __int_as_float(bi));
    __threadfence();
    s_last = atomicAdd(&cnt[b], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last || threadIdx.x != 0) return;
  __threadfence();
  float gv = -INFINITY;
  int gi = 0x7fffffff;
  for (int k = 0; k < (int)gridDim.x; ++k) {
    const float2 pk = __ldcg(&part[b * gridDim.x + k]);
    if (am_better(pk.x, __float_as_int(pk.y), gv, gi)) {
      gv = pk.x;
      gi = __float_as_int(pk.y);
    }
  }
  if (gi == 0x7fffffff) gi = 0;  // every logit NaN
  const long long pos = pos_dev[b];
  tok_hist[(long)b * max_seq + pos] = gi;
  cnt[b] = 0u;
}

__global__ void embed_kernel(const __half* __restrict__ embed, int D, const long long* tok_hist, int max_seq,
                             const long long* pos_dev, __half* __restrict__ h) {
  const int b = blockIdx.x;
  const long long tok = tok_hist[(long)b * max_seq + pos_dev[b]];
  const uint4* src = reinterpret_cast<const uint4*>(embed + tok * D);
  uint4* dst = reinterpret_cast<uint4*>(h + (long)b * D);
  for (int i = threadIdx.x; i < D / 8; i += blockDim.x) dst[i] = src[i];
}

static bool getenv_ldg() {
  static const bool v = [] {
    const char* e = getenv("R4Q_GEMV_PATH");
    return e && e[0] == 'l';
  }();
  return v;
}

// Push targets of this rank's slot in every rank's all-reduce buffer.
struct PushSet {
  float* p[8];
  operator float* const*() const { return p; }
};
static PushSet push_slots(r4q_decode_ctx* c, int parity, bool ll) {
  PushSet s{};
  for (int q = 0; q < c->m.tp_size; ++q) s.p[q] = comm_reduce_slot(c->m.comm, q, parity, ll);
  return s;
}

// The consumer GEMV of an exchange reads the slots in its prologue (TMA path);
// otherwise a reduce kernel materialises r first.
// The consumer GEMV reads the exchange slots in its prologue (every CTA sums
// all ranks' partials) up to 4 ranks; with more, every CTA would re-read
// 8 x hidden tagged words per exchange, so one reduce kernel sums them once
// and the GEMV takes the materialised residual (measured on 8 x B200:
// decode fell below the 4-rank rate with the fused form).  R4Q_TP_FUSED=0 / 1
// forces either form (measurement).
static bool consumer_fused(r4q_decode_ctx* c, int fmt, const void* w, const void* s, int N) {
  GemvArgs probe{};
  probe.K = c->m.hidden; probe.N = N; probe.B = c->m.batch; probe.w = w; probe.s = s;
  static const int forced = [] {
    const char* e = getenv("R4Q_TP_FUSED");
    return e ? atoi(e) : -1;
  }();
  const bool by_size = forced >= 0 ? forced != 0 : c->m.tp_size <= 4;
  return by_size && gemv_tma_supported(probe, fmt) && !getenv_ldg();
}

// A producer whose consumer is fused pushes tagged words (no fence, no flag,
// the consumer polls the words); R4Q_TP_FLAGS=1 keeps the flag protocol
// (measurement only).
static bool exchange_ll(bool consumer_is_fused) {
  static const bool flags = [] {
    const char* e = getenv("R4Q_TP_FLAGS");
    return e && e[0] == '1';
  }();
  return consumer_is_fused && !flags;
}

static void producer_exchange(r4q_decode_ctx* c, TpExchange& x, int idx, bool ll) {
  comm_fill_signal(c->m.comm, x, idx);
  if (ll) {
    x.ll_sig = 1;
    x.nsig = 0;      // no flag: the words carry the epoch
  }
}

// Head norm + RoPE + KV write of the new token and attention over [0, pos]
// with the FWHT epilogue: one fused launch (R4Q_ATTN_FUSED=0: the two kernels).
static int attn_step(r4q_decode_ctx* c, const r4q_layer_desc& ly, cudaStream_t st) {
  const r4q_model_desc& m = c->m;
  const int B = m.batch, H = m.num_heads, Hk = m.num_kv_heads, hd = m.head_dim;
  const int qd = H * hd, kvd = Hk * hd, qkv_n = qd + 2 * kvd;
  static const bool fused = [] {
    const char* e = getenv("R4Q_ATTN_FUSED");
    return !(e && e[0] == '0');
  }();
  if (fused)
    return r4q_attn_decode_fused_ex(c->qkv, qkv_n, ly.q_norm, ly.k_norm, m.rope_cos, m.rope_sin, m.rope_stride,
                                    m.rms_eps, ly.k_cache, ly.v_cache, ly.k_scale, ly.v_scale, c->attn, qd, B, H,
                                    Hk, hd, m.max_seq, 0, c->seq_dev, R4Q_ATTN_FWHT, 1, c->attn_ws,
                                    c->attn_ws_bytes, st);
  int rc = r4q_head_norm_rope(c->qkv, c->qkv + qd, c->qkv + qd + kvd, ly.q_norm, ly.k_norm, m.rope_cos,
                              m.rope_sin, m.rope_stride, 0, c->pos_dev, c->qkv, c->qkv + qd, ly.k_cache,
                              ly.v_cache, ly.k_scale, ly.v_scale, B, H, Hk, hd, qkv_n, qkv_n, m.max_seq,
                              m.rms_eps, R4Q_HEAD_NORM | R4Q_HEAD_ROPE | R4Q_HEAD_KV, st);
  if (rc) return rc;
  return r4q_flash_decode(c->qkv, qkv_n, ly.k_cache, ly.v_cache, ly.k_scale, ly.v_scale, c->attn, qd, B, H, Hk,
                          hd, m.max_seq, 0, c->seq_dev, R4Q_ATTN_FWHT, c->attn_ws, c->attn_ws_bytes, st);
}

// One rank of a tensor-parallel step.  Exchange 2*li is layer li's o_proj,
// 2*li + 1 its down_proj (reduce slots of parity idx & 1), 2*L the lm_head
// vocabulary gather.  Producers push fp32 partials into every rank's slot and
// signal; the next GEMV (gate_up / next qkv / lm_head) waits and reduces in
// its RMSNorm+FWHT prologue, its CTA 0 storing the residual stream.  When
// that GEMV cannot take the TMA path, a reduce kernel materialises r and its
// sums of squares and the GEMV normalises from those.
static int consume(r4q_decode_ctx* c, int idx, const __half* res, __half* out, float* ss, int fmt,
                   const void* w, const void* s, void* y, int N, const void* norm_w, cudaStream_t st,
                   float* const* push = nullptr, int npush = 0, long ld_push = 0, int sig_idx = -1) {
  const r4q_model_desc& m = c->m;
  const int D = m.hidden;
  const bool fused = consumer_fused(c, fmt, w, s, N);
  TpExchange x{};
  int rc = 0;
  if (fused) {
    comm_fill_wait(m.comm, x, idx, idx & 1, res, out, exchange_ll(true));
  } else {
    rc = comm_reduce_residual(m.comm, idx, idx & 1, res, out, ss, m.batch, D, st);
    if (rc) return rc;
  }
  if (sig_idx >= 0) comm_fill_signal(m.comm, x, sig_idx);
  // x = out (fallback: the materialised r; fused: a valid dummy, the prologue
  // reads the exchange buffer)
  return gemv_call(c, fmt, w, s, fused ? res : out, y, N, D, R4Q_PRO_RMSNORM_FWHT, norm_w,
                   fused ? nullptr : ss, D / 16, nullptr, nullptr, st, push, npush, ld_push, &x);
}

static int enqueue_step_tp(r4q_decode_ctx* c, bool with_logits, cudaStream_t st) {
  const r4q_model_desc& m = c->m;
  const int B = m.batch, D = m.hidden, I = m.intermediate, H = m.num_heads, Hk = m.num_kv_heads,
            hd = m.head_dim;
  const int qd = H * hd, kvd = Hk * hd, qkv_n = qd + 2 * kvd;
  const int L = m.num_layers;
  int rc = comm_tick(m.comm, st);
  for (int li = 0; li < L && !rc; ++li) {
    const r4q_layer_desc& ly = c->layers[li];
    const int xo = 2 * li, xd = 2 * li + 1;
    // 1. qkv: layer 0 from the input; later layers consume the previous down exchange
    if (li == 0)
      rc = gemv_call(c, ly.qkv_fmt, ly.qkv_w, ly.qkv_s, c->h_in, c->qkv, qkv_n, D, R4Q_PRO_RMSNORM_FWHT,
                     ly.in_norm, nullptr, 0, nullptr, nullptr, st);
    else
      rc = consume(c, xd - 2, c->r, c->h, c->ss_h, ly.qkv_fmt, ly.qkv_w, ly.qkv_s, c->qkv, qkv_n,
                   ly.in_norm, st);
    if (rc) break;
    const __half* hin = (li == 0) ? c->h_in : c->h;
    rc = attn_step(c, ly, st);
    if (rc) break;
    // 4. o_proj over this rank's heads -> pushed + signalled (exchange xo)
    {
      const bool ll = exchange_ll(consumer_fused(c, ly.gate_up_fmt, ly.gate_up_w, ly.gate_up_s, 2 * I));
      TpExchange x{};
      producer_exchange(c, x, xo, ll);
      rc = gemv_call(c, ly.o_fmt, ly.o_w, ly.o_s, c->attn, nullptr, D, qd, R4Q_PRO_NONE, nullptr, nullptr,
                     0, nullptr, nullptr, st, push_slots(c, xo & 1, ll), m.tp_size, D, &x);
    }
    if (rc) break;
    // 5. gate_up consumes exchange xo: r = o + h
    rc = consume(c, xo, hin, c->r, c->ss_post, ly.gate_up_fmt, ly.gate_up_w, ly.gate_up_s, c->gu, 2 * I,
                 ly.post_norm, st);
    if (rc) break;
    // 6. down over this rank's intermediate slice -> pushed + signalled (xd);
    //    its consumer: the next layer's qkv, or the lm_head (or the final
    //    reduce kernel without logits)
    {
      bool ll;
      if (li + 1 < L) {
        const r4q_layer_desc& nx = c->layers[li + 1];
        ll = exchange_ll(consumer_fused(c, nx.qkv_fmt, nx.qkv_w, nx.qkv_s, qkv_n));
      } else {
        ll = with_logits && exchange_ll(consumer_fused(c, m.lm_fmt, m.lm_w, m.lm_s, m.lm_n));
      }
      TpExchange x{};
      producer_exchange(c, x, xd, ll);
      rc = gemv_call(c, ly.down_fmt, ly.down_w, ly.down_s, c->gu, nullptr, D, I, R4Q_PRO_SILU_FWHT,
                     nullptr, nullptr, 0, nullptr, nullptr, st, push_slots(c, xd & 1, ll), m.tp_size, D, &x);
    }
  }
  if (rc) return rc;
  const int xl = 2 * L - 1;
  if (!with_logits)  // final hidden h = down + r
    return comm_reduce_residual(m.comm, xl, xl & 1, c->r, c->h, nullptr, B, D, st);
  // lm_head: consumes the last down exchange (writes h), pushes its vocabulary
  // slice into every rank's gather buffer, signals exchange 2L
  float* gp[8];
  for (int q = 0; q < m.tp_size; ++q) gp[q] = comm_gather_base(m.comm, q) + (long)m.tp_rank * m.lm_n;
  rc = consume(c, xl, c->r, c->h, c->ss_h, m.lm_fmt, m.lm_w, m.lm_s, nullptr, m.lm_n, m.final_norm, st, gp,
               m.tp_size, (long)m.lm_n * m.tp_size, 2 * L);
  if (rc) return rc;
  return comm_gather_logits(m.comm, 2 * L, c->logits, B, st);
}

static int enqueue_step(r4q_decode_ctx* c, bool with_logits, cudaStream_t st) {
  if (c->m.tp_size > 1) return enqueue_step_tp(c, with_logits, st);
  const r4q_model_desc& m = c->m;
  const int B = m.batch, D = m.hidden, I = m.intermediate, H = m.num_heads, Hk = m.num_kv_heads,
            hd = m.head_dim;
  const int qd = H * hd, kvd = Hk * hd, qkv_n = qd + 2 * kvd;
  const int L = m.num_layers;
  int rc = 0;
  for (int li = 0; li < L && !rc; ++li) {
    const r4q_layer_desc& ly = c->layers[li];
    const __half* hin = (li == 0) ? c->h_in : c->h;
    // 1. qkv projection, RMSNorm + FWHT prologue
    {
    ProfScope ps(c, 0, st);
    rc = gemv_call(c, ly.qkv_fmt, ly.qkv_w, ly.qkv_s, hin, c->qkv, qkv_n, D, R4Q_PRO_RMSNORM_FWHT,
                   ly.in_norm, li == 0 ? nullptr : c->ss_h, D / 16, nullptr, nullptr, st);
    }
    if (rc) break;
    // 2-3. QK norm + RoPE, K/V to the FP8 cache, attention over [0, pos] with
    //      the FWHT on the output (feeds o_proj)
    {
    ProfScope ps(c, 1, st);
    rc = attn_step(c, ly, st);
    }
    if (rc) break;
    ProfScope ps(c, 0, st);  // o, gate_up, down
    // 4. o_proj + residual -> r, sums of squares for the post-attention norm
    rc = gemv_call(c, ly.o_fmt, ly.o_w, ly.o_s, c->attn, c->r, D, qd, R4Q_PRO_NONE, nullptr, nullptr, 0,
                   hin, c->ss_post, st);
    if (rc) break;
    // 5. gate_up with RMSNorm + FWHT of r
    rc = gemv_call(c, ly.gate_up_fmt, ly.gate_up_w, ly.gate_up_s, c->r, c->gu, 2 * I, D,
                   R4Q_PRO_RMSNORM_FWHT, ly.post_norm, c->ss_post, D / 16, nullptr, nullptr, st);
    if (rc) break;
    // 6. down with SiLU*up + FWHT, + residual r -> h, sums of squares for the next norm
    rc = gemv_call(c, ly.down_fmt, ly.down_w, ly.down_s, c->gu, c->h, D, I, R4Q_PRO_SILU_FWHT, nullptr,
                   nullptr, 0, c->r, c->ss_h, st);
  }
  if (rc || !with_logits) return rc;
  return gemv_call(c, m.lm_fmt, m.lm_w, m.lm_s, L > 0 ? c->h : c->h_in, c->logits, m.lm_n, D,
                   R4Q_PRO_RMSNORM_FWHT, m.final_norm, nullptr, 0, nullptr, nullptr, st);
}

static void free_ctx(r4q_decode_ctx* c) {
  for (int i = 0; i < 3; ++i)
    if (c->graph[i]) cudaGraphExecDestroy(c->graph[i]);
  if (c->cap_stream) cudaStreamDestroy(c->cap_stream);
  void* bufs[] = {c->h_in, c->h, c->r, c->qkv, c->attn, c->gu, c->logits, c->h_out, c->ss_post,
                  c->ss_h, c->pos_dev, c->seq_dev, c->gemv_ws, c->attn_ws, c->tp_trace, c->tok_hist,
                  c->am_ws};
  for (void* b : bufs)
    if (b) cudaFree(b);
  delete c;
}

}  // namespace r4q

using namespace r4q;

extern "C" int r4q_decode_ctx_create(const r4q_model_desc* md, const r4q_layer_desc* layers,
                                     r4q_decode_ctx** out) {
  if (!md || !out || (md->num_layers > 0 && !layers))
    return set_error(R4Q_ERR_ARG, "decode_ctx_create: null argument");
  const r4q_model_desc& m = *md;
  if (m.batch < 1 || m.batch > 16 || m.hidden % 128 || m.intermediate % 128 || m.head_dim != 128 ||
      m.num_heads % m.num_kv_heads || m.num_heads / m.num_kv_heads > 8 || m.max_seq < 1 ||
      (m.num_heads * m.head_dim) % 128)
    return set_error(R4Q_ERR_ARG, "decode_ctx_create: unsupported model shape");
  const int tps = m.tp_size < 1 ? 1 : m.tp_size;
  if (tps > 1) {
    if (tps > 8 || !m.comm || m.tp_rank < 0 || m.tp_rank >= tps || comm_world(m.comm) != tps ||
        comm_rank(m.comm) != m.tp_rank)
      return set_error(R4Q_ERR_ARG, "decode_ctx_create: tp_size %d / tp_rank %d do not match the comm",
                       m.tp_size, m.tp_rank);
    if (m.num_layers < 1 || 2 * m.num_layers + 1 > kTpExchangesPerStep || m.batch > comm_max_batch(m.comm) || m.hidden != comm_hidden(m.comm) ||
        (m.lm_w && (long)m.lm_n * tps != comm_vocab(m.comm)))
      return set_error(R4Q_ERR_ARG, "decode_ctx_create: comm sized for B %d D %d V %d",
                       comm_max_batch(m.comm), comm_hidden(m.comm), comm_vocab(m.comm));
  }
  r4q_decode_ctx* c = new r4q_decode_ctx();  // value-initialised: all pointers null
  c->m = m;
  c->m.tp_size = tps;
  c->layers.assign(layers, layers + m.num_layers);
  cudaGetDevice(&c->dev);
  const int B = m.batch, D = m.hidden, I = m.intermediate;
  const int qkv_n = (m.num_heads + 2 * m.num_kv_heads) * m.head_dim;
  const int qd = m.num_heads * m.head_dim;
  int nmax = qkv_n;
  if (2 * I > nmax) nmax = 2 * I;
  if (m.lm_n > nmax) nmax = m.lm_n;
  c->gemv_ws_bytes = r4q_gemv_workspace_bytes(B, nmax, D > I ? D : I);
  c->attn_ws_bytes = r4q_flash_decode_workspace_bytes(B, m.num_heads, m.num_kv_heads, m.max_seq);
  struct {
    void** p;
    size_t n;
  } al[] = {{(void**)&c->h_in, (size_t)B * D * 2},       {(void**)&c->h, (size_t)B * D * 2},
            {(void**)&c->r, (size_t)B * D * 2},          {(void**)&c->qkv, (size_t)B * qkv_n * 2},
            {(void**)&c->attn, (size_t)B * qd * 2},      {(void**)&c->gu, (size_t)B * 2 * I * 2},
            {(void**)&c->logits, (size_t)B * m.lm_n * tps * 2 + 16}, {(void**)&c->h_out, (size_t)B * D * 2},
            {(void**)&c->ss_post, (size_t)D / 16 * B * 4}, {(void**)&c->ss_h, (size_t)D / 16 * B * 4},
            {(void**)&c->pos_dev, (size_t)B * 8},         {(void**)&c->seq_dev, (size_t)B * 8},
            {&c->gemv_ws, c->gemv_ws_bytes},              {&c->attn_ws, c->attn_ws_bytes},
            {(void**)&c->tok_hist, (size_t)B * m.max_seq * 8},
            {&c->am_ws, (size_t)B * kArgmaxBlocks * 8 + (size_t)B * 4 + 16}};
  for (auto& a : al) {
    cudaError_t e = cudaMalloc(a.p, a.n);
    if (e == cudaSuccess) e = cudaMemset(*a.p, 0, a.n);
    if (e != cudaSuccess) {
      free_ctx(c);
      return set_error(R4Q_ERR_CUDA, "decode_ctx_create: %s", cudaGetErrorString(e));
    }
  }
  if (tps > 1 && getenv("R4Q_TP_TRACE")) {
    if (cudaMalloc(&c->tp_trace, 8 * kTpExchangesPerStep * 8) != cudaSuccess ||
        cudaMemset(c->tp_trace, 0, 8 * kTpExchangesPerStep * 8) != cudaSuccess) {
      free_ctx(c);
      return set_error(R4Q_ERR_CUDA, "decode_ctx_create: trace buffer");
    }
  }
  cudaError_t e = cudaStreamCreateWithFlags(&c->cap_stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    free_ctx(c);
    return set_error(R4Q_ERR_CUDA, "decode_ctx_create: stream: %s", cudaGetErrorString(e));
  }
  *out = c;
  return R4Q_OK;
}

extern "C" void r4q_decode_ctx_destroy(r4q_decode_ctx* c) {
  if (c) {
    cudaDeviceSynchronize();
    free_ctx(c);
  }
}

// kind 0: step without lm_head, 1: with logits, 2: greedy token (logits,
// argmax into tok_hist at pos, embedding of the token into h_in)
static int enqueue_kind(r4q_decode_ctx* c, int kind, cudaStream_t st) {
  int rc = enqueue_step(c, kind >= 1, st);
  if (rc || kind < 2) return rc;
  const int B = c->m.batch;
  const int V = c->m.lm_n * c->m.tp_size;
  float2* part = reinterpret_cast<float2*>(c->am_ws);
  unsigned* cnt = reinterpret_cast<unsigned*>(part + (size_t)B * kArgmaxBlocks);
  argmax_kernel<<<dim3(kArgmaxBlocks, B), 256, 0, st>>>(c->logits, V, part, cnt, c->tok_hist, c->m.max_seq,
                                                         c->pos_dev);
  rc = check_launch("argmax_kernel");
  if (rc) return rc;
  embed_kernel<<<B, 256, 0, st>>>(reinterpret_cast<const __half*>(c->loop_embed), c->m.hidden, c->tok_hist,
                                  c->m.max_seq, c->pos_dev, c->h_in);
  return check_launch("embed_kernel");
}

// Run one step of `kind` at the position already set on the device: eagerly,
// or through the context's CUDA graph for that kind (captured on first use).
static int run_kind(r4q_decode_ctx* c, int kind, bool use_graph, cudaStream_t st) {
  if (!use_graph) return enqueue_kind(c, kind, st);
  cudaGraphExec_t& ge = c->graph[kind];
  if (!ge) {
    // one eager step first: it initialises every per-kernel setting (shared
    // memory limits, tensor-map entry point) outside the capture; running the
    // step twice is harmless (same inputs, same cache bytes at pos).  The
    // token kind warms up without its argmax/embedding tail, which would
    // replace the step's input.
    int rc = enqueue_kind(c, kind < 2 ? kind : 1, st);
    if (rc) return rc;
    // capture on the context's stream, ordered after the caller's stream
    cudaEvent_t ev;
    cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    cudaEventRecord(ev, st);
    cudaStreamWaitEvent(c->cap_stream, ev, 0);
    cudaEventDestroy(ev);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamBeginCapture(c->cap_stream, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return set_error(R4Q_ERR_CUDA, "decode: begin capture: %s", cudaGetErrorString(e));
    rc = enqueue_kind(c, kind, c->cap_stream);
    e = cudaStreamEndCapture(c->cap_stream, &g);
    if (rc) {
      if (g) cudaGraphDestroy(g);
      return rc;
    }
    if (e != cudaSuccess) return set_error(R4Q_ERR_CUDA, "decode: end capture: %s", cudaGetErrorString(e));
    e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
      ge = nullptr;
      return set_error(R4Q_ERR_CUDA, "decode: instantiate: %s", cudaGetErrorString(e));
    }
  }
  cudaError_t e = cudaGraphLaunch(ge, st);
  if (e != cudaSuccess) return set_error(R4Q_ERR_CUDA, "decode: graph launch: %s", cudaGetErrorString(e));
  return R4Q_OK;
}

// Per-row positions (continuous batching: each row is its own sequence).
struct RowPositions {
  int p[16];
};
__global__ void set_positions_rows(long long* pos, long long* seq, int B, RowPositions rp) {
  const int i = threadIdx.x;
  if (i < B) {
    pos[i] = rp.p[i];
    seq[i] = rp.p[i] + 1;
  }
}

static int set_pos(r4q_decode_ctx* c, int pos, cudaStream_t st) {
  set_positions<<<1, 32, 0, st>>>(c->pos_dev, c->seq_dev, c->m.batch, pos);
  return check_launch("set_positions");
}

extern "C" int r4q_decode_step(r4q_decode_ctx* c, const void* hidden_in, int pos, void* hidden_out,
                               void* logits_out, int use_graph, void* stream) {
  if (!c || !hidden_in) return set_error(R4Q_ERR_ARG, "decode_step: null argument");
  if (pos < 0 || pos >= c->m.max_seq)
    return set_error(R4Q_ERR_CAPACITY, "decode_step: pos %d outside the KV cache (max_seq %d)", pos,
                     c->m.max_seq);
  cudaStream_t st = (cudaStream_t)stream;
  const int B = c->m.batch, D = c->m.hidden;
  const bool with_logits = logits_out != nullptr;
  cudaError_t e = cudaMemcpyAsync(c->h_in, hidden_in, (size_t)B * D * 2, cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) return set_error(R4Q_ERR_CUDA, "decode_step: copy in: %s", cudaGetErrorString(e));
  int rc = set_pos(c, pos, st);
  if (!rc) rc = run_kind(c, with_logits ? 1 : 0, use_graph != 0, st);
  if (rc) return rc;
  const __half* hfinal = c->m.num_layers > 0 ? c->h : c->h_in;
  if (hidden_out) {
    e = cudaMemcpyAsync(hidden_out, hfinal, (size_t)B * D * 2, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return set_error(R4Q_ERR_CUDA, "decode_step: copy out: %s", cudaGetErrorString(e));
  }
  if (logits_out) {
    e = cudaMemcpyAsync(logits_out, c->logits, (size_t)B * c->m.lm_n * c->m.tp_size * 2,
                        cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return set_error(R4Q_ERR_CUDA, "decode_step: copy logits: %s", cudaGetErrorString(e));
  }
  return R4Q_OK;
}

extern "C" int r4q_decode_step_rows(r4q_decode_ctx* c, const void* hidden_in, const int* pos,
                                    void* hidden_out, void* logits_out, int use_graph, void* stream) {
  if (!c || !hidden_in || !pos) return set_error(R4Q_ERR_ARG, "decode_step_rows: null argument");
  const int B = c->m.batch, D = c->m.hidden;
  RowPositions rp{};
  for (int b = 0; b < B; ++b) {
    if (pos[b] < 0 || pos[b] >= c->m.max_seq)
      return set_error(R4Q_ERR_CAPACITY, "decode_step_rows: row %d pos %d outside the KV cache (max_seq %d)", b,
                       pos[b], c->m.max_seq);
    rp.p[b] = pos[b];
  }
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaMemcpyAsync(c->h_in, hidden_in, (size_t)B * D * 2, cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) return set_error(R4Q_ERR_CUDA, "decode_step_rows: copy in: %s", cudaGetErrorString(e));
  set_positions_rows<<<1, 32, 0, st>>>(c->pos_dev, c->seq_dev, B, rp);
  int rc = check_launch("set_positions_rows");
  if (!rc) rc = run_kind(c, logits_out ? 1 : 0, use_graph != 0, st);
  if (rc) return rc;
  const __half* hfinal = c->m.num_layers > 0 ? c->h : c->h_in;
  if (hidden_out) {
    e = cudaMemcpyAsync(hidden_out, hfinal, (size_t)B * D * 2, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return set_error(R4Q_ERR_CUDA, "decode_step_rows: copy out: %s", cudaGetErrorString(e));
  }
  if (logits_out) {
    e = cudaMemcpyAsync(logits_out, c->logits, (size_t)B * c->m.lm_n * c->m.tp_size * 2,
                        cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess)
      return set_error(R4Q_ERR_CUDA, "decode_step_rows: copy logits: %s", cudaGetErrorString(e));
  }
  return R4Q_OK;
}

__global__ void gather_tokens(const long long* tok_hist, int max_seq, int B, int start, int n, long long* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n * B) return;
  const int t = i / B, b = i - t * B;
  out[i] = tok_hist[(long)b * max_seq + start + t];
}

extern "C" int r4q_decode_loop(r4q_decode_ctx* c, const void* embed, const void* hidden_first, int start_pos,
                               int num_tokens, long long* tokens_out, int use_graph, void* stream) {
  if (!c || !embed || !hidden_first || !tokens_out || num_tokens < 0)
    return set_error(R4Q_ERR_ARG, "decode_loop: bad arguments");
  if (!c->m.lm_w) return set_error(R4Q_ERR_ARG, "decode_loop: the context has no lm_head");
  if (start_pos < 0 || start_pos + num_tokens > c->m.max_seq)
    return set_error(R4Q_ERR_CAPACITY, "decode_loop: positions %d..%d outside the KV cache (max_seq %d)",
                     start_pos, start_pos + num_tokens - 1, c->m.max_seq);
  if (num_tokens == 0) return R4Q_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const int B = c->m.batch, D = c->m.hidden;
  if (c->loop_embed != embed && c->graph[2]) {  // the token graph holds the table pointer
    cudaGraphExecDestroy(c->graph[2]);
    c->graph[2] = nullptr;
  }
  c->loop_embed = embed;
  cudaError_t e = cudaMemcpyAsync(c->h_in, hidden_first, (size_t)B * D * 2, cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) return set_error(R4Q_ERR_CUDA, "decode_loop: copy in: %s", cudaGetErrorString(e));
  for (int t = 0; t < num_tokens; ++t) {
    int rc = set_pos(c, start_pos + t, st);
    if (!rc) rc = run_kind(c, 2, use_graph != 0, st);
    if (rc) return rc;
  }
  const int n = num_tokens * B;
  gather_tokens<<<(n + 255) / 256, 256, 0, st>>>(c->tok_hist, c->m.max_seq, B, start_pos, num_tokens, tokens_out);
  return check_launch("gather_tokens");
}

// One eager step of kind 1 with events between the kernel groups:
// [total, gemv, attention, norm (head norm/RoPE/KV write), rest] in ms
// (decode_profile, int4_decode_step.hip:3047-3281).  Synchronous.
extern "C" int r4q_decode_profile(r4q_decode_ctx* c, const void* hidden_in, int pos, float* out5, void* stream) {
  if (!c || !hidden_in || !out5) return set_error(R4Q_ERR_ARG, "decode_profile: null argument");
  if (pos < 0 || pos >= c->m.max_seq) return set_error(R4Q_ERR_CAPACITY, "decode_profile: pos %d", pos);
  cudaStream_t st = (cudaStream_t)stream;
  const int B = c->m.batch, D = c->m.hidden;
  cudaError_t e = cudaMemcpyAsync(c->h_in, hidden_in, (size_t)B * D * 2, cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) return set_error(R4Q_ERR_CUDA, "decode_profile: copy in: %s", cudaGetErrorString(e));
  int rc = set_pos(c, pos, st);
  if (rc) return rc;
  c->prof = true;
  c->prof_ev.clear();
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0, st);
  rc = enqueue_step(c, c->m.lm_w != nullptr, st);
  cudaEventRecord(e1, st);
  c->prof = false;
  if (!rc) e = cudaStreamSynchronize(st);
  float total = 0.f, cat[3] = {0.f, 0.f, 0.f};
  if (!rc && e == cudaSuccess) {
    cudaEventElapsedTime(&total, e0, e1);
    for (auto& pe : c->prof_ev) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, pe.a, pe.b);
      cat[pe.cat] += ms;
    }
  }
  for (auto& pe : c->prof_ev) {
    cudaEventDestroy(pe.a);
    cudaEventDestroy(pe.b);
  }
  c->prof_ev.clear();
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (rc) return rc;
  if (e != cudaSuccess) return set_error(R4Q_ERR_CUDA, "decode_profile: %s", cudaGetErrorString(e));
  out5[0] = total;
  out5[1] = cat[0];
  out5[2] = cat[1];
  out5[3] = cat[2];
  out5[4] = total - cat[0] - cat[1] - cat[2];
  return R4Q_OK;
}

extern "C" int r4q_decode_tp_trace(r4q_decode_ctx* c, unsigned long long* host) {
  if (!c || !host) return set_error(R4Q_ERR_ARG, "decode_tp_trace: null argument");
  if (!c->tp_trace) return set_error(R4Q_ERR_ARG, "decode_tp_trace: context built without R4Q_TP_TRACE");
  cudaError_t e = cudaMemcpy(host, c->tp_trace, 8 * kTpExchangesPerStep * 8, cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? R4Q_OK : set_error(R4Q_ERR_CUDA, "decode_tp_trace: %s", cudaGetErrorString(e));
}

// Timeouts of the context's GEMVs and attention kernels (their workspaces'
// status words).  Synchronous on the context's device.
extern "C" int r4q_decode_status(r4q_decode_ctx* c, int clear) {
  if (!c) return set_error(R4Q_ERR_ARG, "decode_status: null context");
  int cur = 0;
  cudaGetDevice(&cur);
  cudaSetDevice(c->dev);
  cudaError_t e = cudaDeviceSynchronize();
  int st = e == cudaSuccess ? R4Q_OK : set_error(R4Q_ERR_CUDA, "decode_status: %s", cudaGetErrorString(e));
  if (!st) st = r4q_ws_status(c->gemv_ws, clear, nullptr);
  const int st2 = (st == R4Q_ERR_CUDA) ? st : r4q_ws_status(c->attn_ws, clear, nullptr);
  cudaSetDevice(cur);
  return st ? st : st2;
}
