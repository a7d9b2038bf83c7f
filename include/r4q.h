/*
 * r4q — B200 (sm_100a) decode hot path of rdna4-quant, C ABI.
 *
 * Plain pointers and sizes only.  Every pointer argument is a CUDA device
 * pointer unless stated otherwise; `stream` is a cudaStream_t (NULL = legacy
 * default stream).  Every call only enqueues work on `stream` and returns a
 * status: 0 on success, a negative R4Q_ERR_* code otherwise (the message is
 * available from r4q_last_error()).  No call synchronises the device.
 *
 * Data layouts (the reference's runtime layouts, int4_engine_v5.py:95-102):
 *   INT4 weight   uint8 [N, K/2]   two nibbles per byte, low nibble = even k
 *   INT4 scales   fp16  [N, K/16]  (scale, zero-as-fp16) pair per 32-block
 *   INT8 weight   int8  [N, K]     scales fp16 [N, K/32]
 *   FP16 weight   fp16  [N, K]
 *   activations   fp16  [B, K] with row stride ldx (elements), outputs [B, N]
 *   KV cache      uint8 [Hk, max_seq, D] per batch row, FP8 E4M3 bytes of the
 *                 reference codec (int4_decode_step.hip:47-81)
 */
#ifndef R4Q_H
#define R4Q_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  R4Q_OK = 0,
  R4Q_ERR_ARG = -1,        /* bad shape / null pointer / unsupported option */
  R4Q_ERR_ALIGN = -2,      /* pointer or stride misaligned for vector access */
  R4Q_ERR_CAPACITY = -3,   /* workspace / scratch too small */
  R4Q_ERR_CUDA = -4,       /* a CUDA runtime call failed */
  R4Q_ERR_TIMEOUT = -5,    /* a bounded device-side wait gave up */
};

/* Activation prologue applied inside the GEMV before the dot products. */
enum {
  R4Q_PRO_NONE = 0,        /* x as given */
  R4Q_PRO_FWHT = 1,        /* x <- fp16(H32 x) per 32-block */
  R4Q_PRO_SILU_FWHT = 2,   /* x <- fp16(H32 (silu(g) * u)); g = x[:, :K], u = x[:, K:2K] */
  R4Q_PRO_RMSNORM_FWHT = 3,/* x <- fp16(H32 (x * rrms * norm_w)), rrms = rsqrt(ss/K + eps) */
};

/* Weight formats for r4q_gemv(). */
enum { R4Q_W_INT4 = 0, R4Q_W_INT8 = 1, R4Q_W_FP16 = 2 };

/* Optional fusions of r4q_gemv().  RMSNorm prologue: ss = sum of squares per
 * activation row, taken from `ss_in` ([ss_in_parts][B] partial sums, summed in
 * order) when given, else computed from the fp16 x.  Residual epilogue:
 * y = fp16(fp16(acc) + residual); when `ss_out` is given it receives, per
 * 16-row output tile and row b, the sum of squares of the unrounded sums
 * ([N/16][B]) — exactly the `ss_in` of a following RMSNorm prologue.  This is
 * fused_res_norm_fwht (int4_decode_step.hip:1143-1192) split across the two
 * GEMVs around it. */
typedef struct r4q_gemv_fused {
  const void* norm_w;     /* fp16 [K] */
  float eps;
  const float* ss_in;
  int ss_in_parts;
  const void* residual;   /* fp16 [B, ldres] or NULL; may alias y */
  long ldres;
  float* ss_out;          /* fp32 [N/16][B] or NULL */
  float* y32;             /* non-NULL: write the unrounded fp32 sums here,
                             [B, ldy] (y, residual and ss_out are then unused) */
} r4q_gemv_fused;

/* Status of the bounded device-side waits of the kernels that used the GEMV,
 * GEMM or attention workspace `ws` (NULL: the static scratch of
 * r4q_gemv_int4_noalloc on the current device).  Synchronises `stream`, then
 * returns R4Q_ERR_TIMEOUT if a wait gave up since the word was last cleared
 * (those kernels' outputs are not valid), else R4Q_OK; clear != 0 resets the
 * word after a timeout.  The reference has no bounded waits and no status. */
int r4q_ws_status(const void* ws, int clear, void* stream);

/* Test hook: polls before a bounded mbarrier wait of the GEMV kernels gives
 * up (default 2^26); polls <= 0 restores the default.  Returns the previous
 * limit.  Lowering it makes waits time out so that the error path (status
 * word, drain, R4Q_ERR_TIMEOUT) can be exercised without a hung kernel. */
long r4q_debug_spin_limit(long polls);

/* Message of the last failing call on this host thread ("" if none). */
const char* r4q_last_error(void);
/* Library version (major*10000 + minor*100 + patch). */
int r4q_version(void);

/* ---------------------------------------------------------------- GEMV --- */
/* Bytes of workspace the GEMV entry points need for (B, N, K).  The
 * workspace must be zero-filled once before its first use; the kernels leave
 * it zeroed again on exit, so it can be reused by later calls on the same
 * stream.  Calls that run concurrently need distinct workspaces. */
size_t r4q_gemv_workspace_bytes(int B, int N, int K);

/* y[b, n] = fp16( sum_k fp16((q[n,k] - z[n,k/32]) * s[n,k/32]) * x'[b, k] )
 * with fp32 accumulation, x' = prologue(x).  B in 1..16, K % 32 == 0,
 * N % 16 == 0.  Replaces `gemv_warp<4>`/`launch_gemv`
 * (int4_decode_step.hip:116-170,230-235) and `dbg_gemv`/`dbg_gemm`
 * (:3541-3563); the prologue replaces the separate FWHT / SiLU-FWHT kernels
 * (:1031-1051, :505-557).  ldx, ldy in elements. */
int r4q_gemv_int4(const void* x, long ldx, const void* w, const void* sz, void* y, long ldy,
                  int B, int N, int K, int prologue, void* workspace, size_t ws_bytes,
                  void* stream);

/* INT8 symmetric weights, y = x' @ fp16(q * s)^T.  No kernel in the reference;
 * its dequant is int8_quant.py:52-69 (dequantize_int8). */
int r4q_gemv_int8(const void* x, long ldx, const void* w, const void* s, void* y, long ldy,
                  int B, int N, int K, int prologue, void* workspace, size_t ws_bytes,
                  void* stream);

/* FP16 weights (fp16 lm_head option). */
int r4q_gemv_fp16(const void* x, long ldx, const void* w, void* y, long ldy, int B, int N,
                  int K, int prologue, void* workspace, size_t ws_bytes, void* stream);

/* Generic form: weight format R4Q_W_*, `s` = scales (NULL for FP16), any
 * prologue, optional fusions (may be NULL unless the prologue is RMSNorm). */
int r4q_gemv(int wfmt, const void* x, long ldx, const void* w, const void* s, void* y, long ldy,
             int B, int N, int K, int prologue, const r4q_gemv_fused* fused, void* workspace,
             size_t ws_bytes, void* stream);

/* Same as r4q_gemv_int4, but allocates nothing and takes no workspace: for
 * callers that cannot call cudaMalloc (inside a stream capture that must not
 * allocate, or a plugin whose host process owns all device memory).  No
 * counterpart in the reference.  Its split-K scratch is a fixed 4.06 MiB
 * static device array held by every GPU that loads the library; calls with
 * B * N > 524288 are rejected with R4Q_ERR_CAPACITY.  A timed-out wait is
 * reported by r4q_ws_status(NULL, ...).  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress), so make
 * it before any stream capture.  Every call clears the scratch's counters on
 * `stream`; all calls on one device share the array, so calls that overlap on
 * the GPU (e.g. on different streams) race and must be serialised by the
 * caller. */
int r4q_gemv_int4_noalloc(const void* x, long ldx, const void* w, const void* sz, void* y,
                          long ldy, int B, int N, int K, int prologue, void* stream);

/* ----------------------------------------------------- norms and heads --- */
/* y[r] = fp16(v * rsqrt(mean(v^2) + eps) * w) with v = x[r] (+ res[r]) in fp32;
 * res_out[r] = fp16(v) when given.  x/res rows are ldx apart, y/res_out are
 * contiguous [rows, D].  RMSNorm.forward (engine_utils.py:58-63), fused_rmsnorm
 * (fused_ops.py:12-41), rmsnorm_ds / fused_res_norm (int4_decode_step.hip:795-846). */
int r4q_rmsnorm(const void* x, const void* res, const void* w, void* y, void* res_out, int rows,
                int D, long ldx, float eps, void* stream);

enum { R4Q_HEAD_NORM = 1, R4Q_HEAD_ROPE = 2, R4Q_HEAD_KV = 4 };
/* Per-head RMSNorm (flag NORM), half-split RoPE at position `pos` (ROPE), and
 * the FP8 KV-cache write of K (after norm+RoPE) and V at `pos` (KV), in fp32
 * with one fp16 rounding.  q: [B][ld_in] with H heads of D, k and v likewise
 * with Hk heads; outputs q_out/k_out [B][ld_out] (may alias the inputs; NULL
 * skips); caches [B, Hk, max_seq, D] uint8; tables fp16 [rows][tab_stride],
 * row `pos`.  pos_dev (int64 [B], device) overrides `pos` per batch row (graph
 * replay).  k_scale/v_scale (fp32 [B, Hk], optional): the stored byte is
 * enc(x / scale).  Replaces head_rmsnorm_rope_kv (int4_decode_step.hip:1620-1683),
 * head_rmsnorm (:849), rope_ds (:888), fused_qknorm_rope_decode and
 * fused_rope_decode (fused_ops.py:155-215). */
int r4q_head_norm_rope(void* q, void* k, const void* v, const void* q_norm_w,
                       const void* k_norm_w, const void* cos_tab, const void* sin_tab,
                       long tab_stride, int pos, const long long* pos_dev, void* q_out,
                       void* k_out, void* k_cache, void* v_cache, const float* k_scale,
                       const float* v_scale, int B, int H, int Hk, int D, long ld_in,
                       long ld_out, int max_seq, float eps, int flags, void* stream);

/* --------------------------------------------------------------- attention --- */
enum { R4Q_ATTN_FWHT = 1 };
/* Bytes of workspace r4q_flash_decode needs (zero once before first use; left
 * zeroed by every call). */
size_t r4q_flash_decode_workspace_bytes(int B, int H, int Hk, int max_seq);
/* o[b, h, :] = softmax(q[b,h]·K^T / sqrt(D)) V over positions [0, seq) of the
 * FP8 cache of kv head h / (H / Hk), fp32 softmax/accumulate, fp16 out; with
 * R4Q_ATTN_FWHT the H32 FWHT is applied to every 32-element block of each head
 * (as the reference's reduce does before o_proj).  q: fp16 [B][ldq] with H
 * heads of D = 128; caches uint8 [B, Hk, max_seq, 128] (reference codec);
 * k_scale/v_scale fp32 [B, Hk] or NULL (stored byte = enc(x / scale)); seq =
 * seq_dev[b] (int64, device) when given, else seq_len.  Replaces
 * flash_decode_partial/_reduce/_fused and launch_flash_decode
 * (int4_decode_step.hip:1326-1593); Q is kept in full precision. */
int r4q_flash_decode(const void* q, long ldq, const void* k_cache, const void* v_cache,
                     const float* k_scale, const float* v_scale, void* o, long ldo, int B, int H,
                     int Hk, int D, int max_seq, int seq_len, const long long* seq_dev, int flags,
                     void* workspace, size_t ws_bytes, void* stream);

/* r4q_head_norm_rope (NORM | ROPE | KV) and r4q_flash_decode in one launch:
 * qkv fp16 [B, ld] holds the new token's raw q (H heads), k, v (Hk heads each)
 * side by side; q and k are RMS-normalised (q_norm_w / k_norm_w) and rotated
 * at pos = seq - 1, K and V are encoded to FP8 at cache row pos (divided by the
 * optional per-head scales), and o = attention over [0, seq) (R4Q_ATTN_FWHT as
 * in r4q_flash_decode).  The cache and o equal the two-call sequence.
 * Replaces head_rmsnorm_rope_kv + flash_decode (int4_decode_step.hip:
 * 1326-1593, 1620-1683) on the decode path. */
int r4q_attn_decode_fused(const void* qkv, long ld, const void* q_norm_w, const void* k_norm_w,
                          const void* cos_tab, const void* sin_tab, long tab_stride, float eps,
                          void* k_cache, void* v_cache, const float* k_scale, const float* v_scale,
                          void* o, long ldo, int B, int H, int Hk, int D, int max_seq, int seq_len,
                          const long long* seq_dev, int flags, void* workspace, size_t ws_bytes,
                          void* stream);

/* ------------------------------------------------------------ prefill GEMM --- */
/* y[M, N] fp16 = x[M, K] fp16 · w[N, K]ᵀ on the tcgen05 tensor cores (fp32
 * accumulation in tensor memory).  x row stride ldx, y row stride ldy
 * (elements); K % 8 == 0, 16-byte aligned x and w.  workspace: >= 4 bytes,
 * zeroed, receives 1 if a bounded wait gave up.  Replaces the rocBLAS GEMM of
 * the reference prefill (int4_decode_step.hip:2127-2320). */
int r4q_gemm_fp16(const void* x, long ldx, const void* w, void* y, long ldy, int M, int N, int K,
                  void* workspace, size_t ws_bytes, void* stream);
/* The same with INT4 weights in the runtime layout (nibbles [N, K/2], (scale,
 * zero) pairs [N, K/16]), dequantised in the kernel to the exact reference
 * value fp16((q - z) · s) (dequant_int4, :3568-3603) — dequant + GEMM of the
 * reference prefill (:1973-1988) in one pass over the weights.  K % 64 == 0. */
int r4q_gemm_int4(const void* x, long ldx, const void* w, const void* sz, void* y, long ldy, int M, int N,
                  int K, void* workspace, size_t ws_bytes, void* stream);
/* Workspace bytes for r4q_gemm_fp16 / r4q_gemm_int4 at this shape (16-byte
 * aligned, zeroed once; the kernels leave it zero).  Decode-sized M splits K
 * over the SMs and needs fp32 partials; with a smaller workspace the split
 * count drops (256 bytes: no split). */
size_t r4q_gemm_workspace_bytes(int M, int N, int K);

/* Row kernels of the batched prefill (int4_decode_step.hip:766-792, 2112-2124):
 * y = fp16(H32 x) on every 32-block of rows x K; y = fp16(silu(g) * u) with
 * g = x[:, :I], u = x[:, I:2I]; INT8 weights to fp16 (int8_quant.py:52-69). */
int r4q_fwht_rows(const void* x, long ldx, void* y, long ldy, int rows, int K, void* stream);
int r4q_silu_mul(const void* x, long ldx, void* y, long ldy, int rows, int I, void* stream);
int r4q_dequant_int8(const void* w, const void* s, void* out, int N, int K, void* stream);
/* Prompt K/V into the FP8 cache: rows m of k, v (fp16, row stride ld, Hk heads
 * of D = 128) to cache[batch_row][h][start_pos + m] with the reference encoder
 * (divided by the optional per-head scales).  The reference prefill writes no
 * cache; this lets a prefilled prompt feed the decode step. */
int r4q_kv_write_rows(const void* k, const void* v, long ld, void* k_cache, void* v_cache, int M, int Hk, int D,
                      int max_seq, int start_pos, int batch_row, const float* k_scale, const float* v_scale,
                      void* stream);

/* ------------------------------------------------- mixture-of-experts FFN --- */
/* No counterpart in the reference (its engine is dense); benchmark config 4.
 * Routing: per token softmax over router logits fp16 [B, E] (fp32), top-k
 * (ties to the lower expert), weights renormalised over the k -> ids int32
 * [B, topk], wts fp32 [B, topk]; entries t * topk + k grouped by expert in
 * token order: counts [E], offsets [E + 1], list [B * topk], active [E]
 * (experts with tokens in [e_lo, e_hi), ascending — this GPU's slice under
 * expert parallelism), n_active [1].  E <= 256, topk <= 16. */
int r4q_moe_route(const void* logits, int B, int E, int topk, int e_lo, int e_hi, int* ids, float* wts,
                  int* counts, int* offsets, int* list, int* active, int* n_active, void* stream);
/* Router of a decode layer in one launch: xn[b] = fp16(H32(x[b] * rrms *
 * norm_w)) with rrms from the ss_in partials [ss_parts][B] (norm_w null: xn
 * is an input, already normalised), logits[b][e] = fp16(router_w[e] · xn[b])
 * (router_w fp16 [E, D], H32-rotated), then the routing of r4q_moe_route by
 * the grid's last CTA.  done: one int, zero before the first call (the
 * kernel leaves it zero).  D % 256 == 0, D <= 2048, E <= 256. */
int r4q_moe_router(const void* x, const float* ss_in, int ss_parts, const void* norm_w, float eps, void* xn,
                   const void* router_w, void* logits, int B, int D, int E, int topk, int e_lo, int e_hi, int* ids,
                   float* wts, int* counts, int* offsets, int* list, int* active, int* n_active, int* done,
                   void* stream);
/* y[b] = fp16(H32(x[b] * rrms * w)) per 32-block, rrms from ss_in partials
 * ([ss_parts][rows]) or from x: the RMSNorm+FWHT prologue as its own pass. */
int r4q_norm_fwht_rows(const void* x, const float* ss_in, int ss_parts, const void* w, float eps, void* y,
                       int rows, int D, void* stream);
/* Grouped INT4 expert GEMV over the routed entries of experts [e_lo, e_hi)
 * (the active list of r4q_moe_route).  This GPU's experts stacked: w
 * [(e_hi - e_lo) * N, K/2], sz [(e_hi - e_lo) * N, K/16]; N % 64 == 0,
 * K % 128 == 0.  mode 0: y[j] = W_e · x[j / topk]; mode 1: y[j] = W_e · x[j];
 * mode 2 (gate_up, N = 2 Ie, rows [gate; up]): y[j] = fp16(H32(silu(g) u)),
 * g, u = fp16(W_e · x[j / topk]) halves — down_proj's input, Ie per row.
 * y rows fp16 (ldy), one per entry j.  status (nullable): set to 1 when a
 * bounded wait for the weight tile gives up. */
int r4q_moe_gemv(int mode, const void* w, const void* sz, const void* x, long ldx, void* y, long ldy, int N,
                 int K, int E, int e_lo, int e_hi, int B, int topk, const int* counts, const int* offsets,
                 const int* list, const int* active, const int* n_active, int* status, void* stream);
/* Over the entries of experts [e_lo, e_hi): h[b] = fp16(fp16(sum_k wts[b,k]
 * y[b*topk+k]) + res[b]) in slot order with ss_out [D/16][B] the sums of
 * squares of the unrounded h (res may alias h); or, with out32, the fp32
 * partial sum alone (expert parallelism: summed over GPUs, then
 * r4q_residual_f32). */
int r4q_moe_combine(const void* y, const float* wts, const int* ids, int e_lo, int e_hi, const void* res, void* h,
                    float* out32, float* ss_out, int B, int D, int topk, void* stream);
/* h = fp16(fp16(sum) + res) and its per-16-row sums of squares, sum fp32 [B, D]. */
int r4q_residual_f32(const float* sum, const void* res, void* h, float* ss_out, int B, int D, void* stream);
/* The same for an fp16 a: h = fp16(a + res) with the sums of squares of the
 * unrounded sum (the GEMV residual epilogue as its own pass, for batches the
 * tensor-core GEMM takes). */
int r4q_residual_f16(const void* a, const void* res, void* h, float* ss_out, int B, int D, void* stream);

/* ------------------------------------------------------------- decode step --- */
/* One transformer layer's weights and caches (device pointers).  *_fmt is
 * R4Q_W_INT4 (packed [N, K/2] + (scale, zero) pairs [N, K/16]) or R4Q_W_INT8
 * (int8 [N, K] + fp16 scales [N, K/32]).  qkv rows: q heads, k heads, v heads;
 * gate_up rows: gate then up (the reference's fused layouts). */
typedef struct r4q_comm r4q_comm;

typedef struct r4q_layer_desc {
  int qkv_fmt, o_fmt, gate_up_fmt, down_fmt;
  const void *qkv_w, *qkv_s, *o_w, *o_s, *gate_up_w, *gate_up_s, *down_w, *down_s;
  const void *in_norm, *post_norm, *q_norm, *k_norm;   /* fp16 [hidden] / [head_dim] */
  void *k_cache, *v_cache;                              /* uint8 [batch, Hk, max_seq, head_dim] */
  const float *k_scale, *v_scale;                       /* fp32 [batch, Hk] or NULL */
} r4q_layer_desc;

typedef struct r4q_model_desc {
  int num_layers, batch, hidden, intermediate, num_heads, num_kv_heads, head_dim, max_seq;
  float rms_eps;
  const void *rope_cos, *rope_sin;   /* fp16 [rows, head_dim/2] */
  long rope_stride;                  /* elements between table rows */
  const void* final_norm;            /* fp16 [hidden] */
  int lm_fmt;                        /* R4Q_W_INT4 / R4Q_W_INT8 / R4Q_W_FP16 */
  const void *lm_w, *lm_s;           /* lm_s NULL for fp16 */
  int lm_n;                          /* vocabulary rows (of this rank's shard) */
  /* Tensor parallelism (tp_size 1: single GPU, comm unused).  With tp_size > 1
   * the layer tensors are this rank's shards: qkv rows of its num_heads /
   * num_kv_heads (local counts), o_proj columns of those heads, gate_up rows of
   * its intermediate slice (gate slice then up slice), down columns of that
   * slice, KV caches of its kv heads, lm_head rows of its lm_n-row vocabulary
   * slice; hidden, norms and rope tables are whole.  logits are gathered to
   * [batch, lm_n * tp_size] on every rank; hidden states are replicated. */
  int tp_rank, tp_size;
  r4q_comm* comm;
} r4q_model_desc;

typedef struct r4q_decode_ctx r4q_decode_ctx;

/* Allocate the scratch of a decode step for this model on the current device
 * (the layer table is copied; the weights/caches it points to stay owned by the
 * caller).  Replaces the lazily grown global scratch `g_ds`
 * (int4_decode_step.hip:2325-2412). */
int r4q_decode_ctx_create(const r4q_model_desc* model, const r4q_layer_desc* layers,
                          r4q_decode_ctx** out);
void r4q_decode_ctx_destroy(r4q_decode_ctx* ctx);

/* Enqueue one decode step for all `batch` rows at position `pos` on `stream`:
 * hidden_in fp16 [batch, hidden] (device) -> hidden_out (NULL to skip) and
 * logits_out fp16 [batch, lm_n] (NULL to skip the final norm + lm_head).  K/V of
 * `pos` are written to every layer's cache.  use_graph = 1 captures the step
 * once into a CUDA graph (the position is a device scalar) and replays it on
 * later calls.  Replaces int4_decode_step / int4_decode_step_logits
 * (int4_decode_step.hip:2343-2595) and the graph replay of :2801-3041.  A
 * context is not thread-safe and must not run on two streams at once. */
int r4q_decode_step(r4q_decode_ctx* ctx, const void* hidden_in, int pos, void* hidden_out,
                    void* logits_out, int use_graph, void* stream);

/* r4q_decode_step with a position per row (host int array [batch]): row b's
 * token is decoded at pos[b], its K/V written there and its attention runs
 * over [0, pos[b]], so each row can be a different request of a continuously
 * batched server (r4q/serve.py).  Same graph as r4q_decode_step (positions
 * are device values).  The reference serialises requests behind one lock and
 * decodes one sequence at a time (api_server.py:40, 58-150); this entry
 * point has no direct counterpart there. */
int r4q_decode_step_rows(r4q_decode_ctx* ctx, const void* hidden_in, const int* pos, void* hidden_out,
                         void* logits_out, int use_graph, void* stream);

/* Greedy decode of num_tokens tokens entirely on the device: token t runs the
 * step at position start_pos + t with logits, takes the argmax (first maximum,
 * NaN skipped) and feeds the embedding row of that token (embed fp16
 * [vocab, hidden]) into step t + 1.  hidden_first fp16 [batch, hidden] is the
 * first step's input.  tokens_out: device int64 [num_tokens, batch].  With
 * use_graph each token is one CUDA-graph launch (step + argmax + embedding,
 * captured once per context and table); no host synchronisation.  Replaces
 * decode_loop / decode_bench / decode_bench_graph
 * (int4_decode_step.hip:2601-2795, 2801-3041, 3284-3466). */
int r4q_decode_loop(r4q_decode_ctx* ctx, const void* embed, const void* hidden_first, int start_pos,
                    int num_tokens, long long* tokens_out, int use_graph, void* stream);

/* One eager step with logits at `pos`, timed with events per kernel group:
 * out5 (host) = [total, gemv, attention, norm, rest] in ms, as decode_profile
 * (int4_decode_step.hip:3047-3281).  Synchronous.  Single-GPU contexts time
 * every group; tensor-parallel contexts report the total (rest = total). */
int r4q_decode_profile(r4q_decode_ctx* ctx, const void* hidden_in, int pos, float* out5, void* stream);

/* Exchange timeline of a tensor-parallel context created with the environment
 * variable R4Q_TP_TRACE set (synchronous; host array of 8 x 256 u64 global-timer
 * stamps in ns, per exchange index: producer compute start, producer signal,
 * consumer wait start, consumer wait end, consumer input staged, producer
 * entry, producer CTA 0 done, producer's last CTA arrived; an exchange of
 * tagged words has no signal, so its events 1, 6 and 7 stay 0).  A profiling aid; R4Q_ERR_ARG when the context has no trace. */
int r4q_decode_tp_trace(r4q_decode_ctx* ctx, unsigned long long* host);

/* Timeout status of the context's GEMV and attention kernels (synchronises the
 * device's legacy stream; see r4q_ws_status): R4Q_ERR_TIMEOUT if a bounded
 * wait gave up since the last clear, else R4Q_OK. */
int r4q_decode_status(r4q_decode_ctx* ctx, int clear);

/* ------------------------------------------- tensor-parallel exchange --- */
/* One comm per rank, one process per GPU.  The reference runs on one GPU and
 * has no collectives; this is the all-reduce of a Megatron-style tensor-
 * parallel split between the per-layer GEMVs (an NCCL all_reduce arm of the
 * same step lives in r4q/tp_nccl.py for comparison): each rank
 * owns a peer-visible buffer, producers push fp32 partials straight into the
 * peers' buffers over NVLink and a sync kernel (signal, bounded wait, reduce in
 * rank order) finishes the exchange.  Set-up: r4q_comm_create on every rank,
 * exchange the R4Q_COMM_HANDLE_BYTES handles out of band (all ranks' handles,
 * rank order), then r4q_comm_open.  Every rank must issue the same sequence of
 * exchanges.  A wait that times out (~2 s) records R4Q_ERR_TIMEOUT, readable
 * with r4q_comm_status, and the kernel returns instead of hanging. */
#define R4Q_COMM_HANDLE_BYTES 64
/* max_batch x hidden: the decode all-reduce size; vocab: the full gathered
 * vocabulary (0 if no lm_head gather); sa_cap: elements of the standalone
 * all-reduce.  Writes this rank's handle to handle_out (host, 64 bytes). */
int r4q_comm_create(int rank, int world, int max_batch, int hidden, int vocab, long sa_cap,
                    r4q_comm** out, void* handle_out);
/* handles: host array [world][R4Q_COMM_HANDLE_BYTES] in rank order. */
int r4q_comm_open(r4q_comm* comm, const void* handles);
/* Synchronous: R4Q_OK, or R4Q_ERR_TIMEOUT naming the ranks a wait gave up on. */
int r4q_comm_status(r4q_comm* comm);
int r4q_comm_clear_status(r4q_comm* comm);
/* y[n] = sum over ranks of x[n] (fp32, summed in rank order: identical on
 * every rank); x and y are device arrays of this rank, n <= sa_cap. */
int r4q_comm_allreduce_f32(r4q_comm* comm, const float* x, float* y, long n, void* stream);
void r4q_comm_destroy(r4q_comm* comm);

/* --------------------------------------------------------- conversions --- */
/* out[N, K] fp16 = fp16((q - z) * s); bit-exact to `dequant_int4_kernel`
 * (int4_decode_step.hip:3568-3603) and dequantize_int4_asym
 * (int4_quant_v2.py:105-127). */
int r4q_dequant_int4(const void* packed, const void* sz, void* out, int N, int K, void* stream);

/* n fp16 -> n FP8 bytes with the reference encoder; `fp16_to_fp8`
 * (int4_decode_step.hip:3606-3618). */
int r4q_fp16_to_fp8(const void* src, void* dst, long n, void* stream);

/* n FP8 bytes -> n fp32 with the reference decoder (int4_decode_step.hip:71-81). */
int r4q_fp8_to_fp32(const void* src, void* dst, long n, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* R4Q_H */
