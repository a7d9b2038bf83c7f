// Dequant-GEMV for the decode path: y[b, n] = sum_k W[n, k] * x'[b, k].
//
// Design (B200, HBM-bound matvec):
//  * every weight byte is read exactly once with 128-bit streaming loads
//    (ld.global.nc.L1::no_allocate); each thread owns a 16-byte chunk of two
//    rows (g and g+8 of a 16-row tile), so the dequantised values land directly
//    in the A-fragment registers of an m16n8k16 tensor-core MMA — no shared
//    memory round trip for weights;
//  * nibbles / int8 bytes become fp16 with integer bit tricks (lop3/prmt into
//    the 0x6400 exponent), then (q - z) and * s in fp16 give exactly the
//    reference dequant value fp16((q - z) * s); the MMA multiplies those by the
//    fp16 activations and accumulates in fp32;
//  * activations are staged once per CTA in shared memory, already permuted
//    into the order the B fragments need, and the prologue (H32 FWHT, SiLU*up)
//    is applied while staging — no separate activation kernel;
//  * the grid is planned to fill all SMs in one wave: 16-row tiles x K splits;
//    split partials go to an fp32 workspace and the last CTA of a tile sums
//    them in split order (deterministic), then resets the tile counter.
//
// Replaces gemv_warp<4>/launch_gemv (int4_decode_step.hip:116-170,230-235);
// the reference maps one warp to 4 rows with scalar FMAs.
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <mutex>
#include <unordered_map>

#include "gemv_dev.cuh"

namespace r4q {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxSplit = 16;
constexpr int kMaxXSmem = 96 * 1024;

template <int FMT>
__device__ __forceinline__ void load_chunk(const GemvParams& p, int row, int chunk, bool valid,
                                           RowChunk& r) {
  using F = Fmt<FMT>;
  if (!valid) {
    r.w = make_uint4(0, 0, 0, 0);
    r.s = 0;
    return;
  }
  const long rowbytes = (FMT == W_INT4) ? (p.K >> 1) : (FMT == W_INT8 ? p.K : 2L * p.K);
  r.w = ldg_stream128(p.w + (long)row * rowbytes + (long)chunk * 16);
  if constexpr (FMT == W_INT4) {
    r.s = ldg_stream32(p.s + ((long)row * (p.K >> 5) + chunk) * 2);
  } else if constexpr (FMT == W_INT8) {
    const uint16_t sv = __ldg(reinterpret_cast<const unsigned short*>(p.s) +
                              (long)row * (p.K >> 5) + (chunk >> 1));
    r.s = sv;
  } else {
    r.s = 0;
  }
  (void)F::CK;
}

// --------------------------------------------------------------- kernel ---
// CTA exit of a tensor-parallel producer: the last CTA signals every rank
// (called by all threads of the CTA; tp_signal_cta fences at system scope).
__device__ __forceinline__ void tp_exit(const GemvParams& p) {
  if (!p.tpx.nsig) return;
  __syncthreads();
  if (threadIdx.x == 0) tp_signal_cta(p.tpx);
}

template <int FMT, int NG>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const GemvParams p) {
  using F = Fmt<FMT>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;

  const int nsteps = steps_total(p.K, F::CK, F::U);
  const int ks = blockIdx.y;
  const int s0 = (int)((long)ks * nsteps / p.ksplit);
  const int s1 = (int)((long)(ks + 1) * nsteps / p.ksplit);
  const int nst = s1 - s0;
  const int nch_pad = nst * 4 * F::U;           // chunks covered by this CTA (padded)
  const int chunk0 = s0 * 4 * F::U;             // first global chunk
  const int nchunks = p.K / F::CK;
  const int colstride = x_colstride(nst, F::NSUB, F::U);
  const int ncolx = p.B;

  // ---- main loop: warp -> (m-tile, interleaved steps) ----
  const int wpm = kWarps / p.mt;
  const int mt = warp % p.mt, wi = warp / p.mt;
  const int row0 = blockIdx.x * p.mt * 16 + mt * 16;
  const bool tile_ok = row0 < p.N;
  const int row_a = row0 + g, row_b = row0 + g + 8;
  int colx[NG];
#pragma unroll
  for (int cg = 0; cg < NG; ++cg) colx[cg] = min(cg * 8 + g, p.B - 1);

  float acc[NG][4];
#pragma unroll
  for (int cg = 0; cg < NG; ++cg)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[cg][i] = 0.0f;

  // first weight chunks are requested before the activations are staged, so
  // the HBM latency overlaps the prologue
  RowChunk cur_a[F::U], cur_b[F::U], nxt_a[F::U], nxt_b[F::U];
  const bool active = tile_ok && wi < nst;
  if (active) {
#pragma unroll
    for (int u = 0; u < F::U; ++u) {
      const int lc = wi * 4 * F::U + u * 4 + t;
      const bool v = chunk0 + lc < nchunks;
      load_chunk<FMT>(p, row_a, chunk0 + lc, v, cur_a[u]);
      load_chunk<FMT>(p, row_b, chunk0 + lc, v, cur_b[u]);
    }
  }

  // ---- RMSNorm prologue: one rrms per activation column ----
  __shared__ float s_rrms[16];
  if (p.prologue == R4Q_PRO_RMSNORM_FWHT) {
    if (p.ss_in) {
      // sum of the producer's per-tile partials in tile order (deterministic)
      if (warp < ncolx) {
        float ss = 0.0f;
        for (int i = lane; i < p.ss_in_parts; i += 32) ss += p.ss_in[(long)i * ncolx + warp];
        ss = warp_sum(ss);
        if (lane == 0) s_rrms[warp] = rsqrtf(ss / (float)p.K + p.eps);
      }
      if (ncolx > kWarps && warp + kWarps < ncolx) {
        const int c = warp + kWarps;
        float ss = 0.0f;
        for (int i = lane; i < p.ss_in_parts; i += 32) ss += p.ss_in[(long)i * ncolx + c];
        ss = warp_sum(ss);
        if (lane == 0) s_rrms[c] = rsqrtf(ss / (float)p.K + p.eps);
      }
    } else {
      // sum of squares of the fp16 input itself (fused_rmsnorm_fwht, hip:1195-1215)
      for (int c = warp; c < ncolx; c += kWarps) {
        const __half2* xr = reinterpret_cast<const __half2*>(p.x + (long)c * p.ldx);
        float ss = 0.0f;
        for (int i = lane; i < (p.K >> 1); i += 32) {
          const float2 f = __half22float2(xr[i]);
          ss += f.x * f.x + f.y * f.y;
        }
        ss = warp_sum(ss);
        if (lane == 0) s_rrms[c] = rsqrtf(ss / (float)p.K + p.eps);
      }
    }
    __syncthreads();
  }

  // ---- stage activations (with prologue) into shared memory ----
  {
    const int nblk = nch_pad * F::CK / 32;
    const int k_base = chunk0 * F::CK;
    for (int item = tid; item < ncolx * nblk; item += kThreads) {
      const int col = item / nblk, blk = item - col * nblk;
      __half v[32];
      load_block32(p, col, k_base + blk * 32,
                   p.prologue == R4Q_PRO_RMSNORM_FWHT ? s_rrms[col] : 1.0f, v);
      store_block32<FMT>(smem + (long)col * colstride, nch_pad, blk, v);
    }
  }
  __syncthreads();

  if (active) {
    for (int s = wi; s < nst; s += wpm) {
      const int sn = s + wpm;
      if (sn < nst) {
#pragma unroll
        for (int u = 0; u < F::U; ++u) {
          const int lc = sn * 4 * F::U + u * 4 + t;
          const bool v = chunk0 + lc < nchunks;
          load_chunk<FMT>(p, row_a, chunk0 + lc, v, nxt_a[u]);
          load_chunk<FMT>(p, row_b, chunk0 + lc, v, nxt_b[u]);
        }
      }
#pragma unroll
      for (int u = 0; u < F::U; ++u) {
        const int lc = s * 4 * F::U + u * 4 + t;
        chunk_mma<FMT, NG>(cur_a[u], cur_b[u], smem, colstride, nch_pad, lc, colx, acc);
      }
#pragma unroll
      for (int u = 0; u < F::U; ++u) {
        cur_a[u] = nxt_a[u];
        cur_b[u] = nxt_b[u];
      }
    }
  }

  // ---- reduce the warps that share an m-tile ----
  __syncthreads();  // activation smem no longer needed: reuse it
  float* red = reinterpret_cast<float*>(smem);  // [warp][NG*4][32]
#pragma unroll
  for (int cg = 0; cg < NG; ++cg)
#pragma unroll
    for (int i = 0; i < 4; ++i) red[(warp * NG * 4 + cg * 4 + i) * 32 + lane] = acc[cg][i];
  __syncthreads();

  __shared__ unsigned s_last;
  if (wi == 0 && tile_ok) {
#pragma unroll
    for (int cg = 0; cg < NG; ++cg)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float v = 0.0f;
        for (int j = 0; j < wpm; ++j) v += red[((mt + j * p.mt) * NG * 4 + cg * 4 + i) * 32 + lane];
        acc[cg][i] = v;
      }
    if (p.ksplit == 1) {
      // fp16 output, optionally + residual (fp16(fp16(acc) + res)) and the
      // per-16-row sum of squares of the unrounded sum
#pragma unroll
      for (int cg = 0; cg < NG; ++cg) {
        float sq[2] = {0.0f, 0.0f};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int c = cg * 8 + 2 * t + h;
          if (c < p.B && p.npush) {
            const unsigned ll_tag = p.tpx.ll_sig ? (unsigned)tp_epoch(p.tpx, p.tpx.sig_idx) : 0u;
            for (int q = 0; q < p.npush; ++q) {
              if (p.tpx.ll_sig) {
                tp_push_word(p.y32p[q], (long)c * p.ldy + row_a, ll_tag, acc[cg][h]);
                tp_push_word(p.y32p[q], (long)c * p.ldy + row_b, ll_tag, acc[cg][2 + h]);
              } else {
                p.y32p[q][(long)c * p.ldy + row_a] = acc[cg][h];
                p.y32p[q][(long)c * p.ldy + row_b] = acc[cg][2 + h];
              }
            }
          } else if (c < p.B) {
            float va = __half2float(__float2half(acc[cg][h]));
            float vb = __half2float(__float2half(acc[cg][2 + h]));
            if (p.res) {
              va += __half2float(p.res[(long)c * p.ldres + row_a]);
              vb += __half2float(p.res[(long)c * p.ldres + row_b]);
            }
            sq[h] = va * va + vb * vb;
            p.y[(long)c * p.ldy + row_a] = __float2half(va);
            p.y[(long)c * p.ldy + row_b] = __float2half(vb);
          }
        }
        if (p.ss_out) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float v = sq[h];
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            v += __shfl_xor_sync(0xffffffffu, v, 8);
            v += __shfl_xor_sync(0xffffffffu, v, 16);
            const int c = cg * 8 + 2 * t + h;
            if (g == 0 && c < p.B) p.ss_out[(long)(row0 >> 4) * p.B + c] = v;
          }
        }
      }
    } else {
      float* part = p.part + (long)ks * p.B * p.N;
#pragma unroll
      for (int cg = 0; cg < NG; ++cg) {
        const int c0 = cg * 8 + 2 * t, c1 = c0 + 1;
        if (c0 < p.B) {
          part[(long)c0 * p.N + row_a] = acc[cg][0];
          part[(long)c0 * p.N + row_b] = acc[cg][2];
        }
        if (c1 < p.B) {
          part[(long)c1 * p.N + row_a] = acc[cg][1];
          part[(long)c1 * p.N + row_b] = acc[cg][3];
        }
      }
    }
  }
  if (p.npush > 1 && !p.tpx.nsig && !p.tpx.ll_sig) __threadfence_system();  // peer outputs complete before exit
  if (p.ksplit == 1) {
    tp_exit(p);
    return;
  }

  // ---- split-K fixup: the last CTA of this row tile sums partials in order ----
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned old = atomicAdd(&p.cnt[blockIdx.x], 1u);
    s_last = (old == (unsigned)p.ksplit - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (!s_last) {
    tp_exit(p);
    return;
  }
  __threadfence();
  const int trow0 = blockIdx.x * p.mt * 16;
  const int tiles16 = min(p.mt, (p.N - trow0) >> 4);
  // one warp per (16-row tile, column): lanes 0..15 own one row each
  for (int task = warp; task < tiles16 * p.B; task += kWarps) {
    const int ti = task / p.B, col = task - ti * p.B;
    const int r = trow0 + ti * 16 + (lane & 15);
    float v = 0.0f;
    for (int k2 = 0; k2 < p.ksplit; ++k2) v += __ldcg(p.part + ((long)k2 * p.B + col) * p.N + r);
    if (p.npush) {
      if (lane < 16)
        for (int q = 0; q < p.npush; ++q) {
          if (p.tpx.ll_sig) tp_push_word(p.y32p[q], (long)col * p.ldy + r, (unsigned)tp_epoch(p.tpx, p.tpx.sig_idx), v);
          else p.y32p[q][(long)col * p.ldy + r] = v;
        }
      continue;
    }
    v = __half2float(__float2half(v));
    if (p.res) v += __half2float(p.res[(long)col * p.ldres + r]);
    if (lane < 16) p.y[(long)col * p.ldy + r] = __float2half(v);
    float sq = (lane < 16) ? v * v : 0.0f;
    sq = warp_sum(sq);
    if (p.ss_out && lane == 0) p.ss_out[(long)((trow0 >> 4) + ti) * p.B + col] = sq;
  }
  if (tid == 0) p.cnt[blockIdx.x] = 0u;  // leave the workspace zeroed for the next launch
  if (p.npush > 1 && !p.tpx.nsig && !p.tpx.ll_sig) __threadfence_system();
  tp_exit(p);
}

// ------------------------------------------------------------- planning ---
struct Plan {
  int mt, ksplit;
  size_t smem;
};

template <int FMT, int NG>
static int occupancy_for(size_t smem) {
  static std::mutex mu;
  static std::unordered_map<size_t, int> cache;
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(smem);
  if (it != cache.end()) return it->second;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(gemv_kernel<FMT, NG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kMaxXSmem + 16384);
    attr_set = true;
  }
  int nb = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, gemv_kernel<FMT, NG>, kThreads, smem) !=
      cudaSuccess)
    nb = 1;
  cache[smem] = nb < 1 ? 1 : nb;
  return cache[smem];
}

template <int FMT, int NG>
static Plan make_plan(int B, int N, int K, size_t ws_bytes) {
  using F = Fmt<FMT>;
  const int nsm = num_sms();
  const int nsteps = steps_total(K, F::CK, F::U);
  Plan best{1, 1, 0};
  double best_score = -1.0;
  for (int mt : {4, 2, 1}) {
    const int tiles = (N + 16 * mt - 1) / (16 * mt);
    const int wpm = kWarps / mt;
    for (int ks = 1; ks <= kMaxSplit && ks <= nsteps; ++ks) {
      if (ks > 1) {
        const size_t need = gemv_ws_bytes_for(B, N, ks);
        if (need > ws_bytes) break;
      }
      const int nst = (nsteps + ks - 1) / ks;
      const size_t xs = (size_t)x_colstride(nst, F::NSUB, F::U) * B;
      const size_t red = (size_t)kWarps * NG * 4 * 32 * sizeof(float);
      const size_t smem = xs > red ? xs : red;
      if (xs > (size_t)kMaxXSmem) continue;
      const int occ = occupancy_for<FMT, NG>(smem);
      const long slots = (long)occ * nsm;
      const long ctas = (long)tiles * ks;
      const long waves = (ctas + slots - 1) / slots;
      double eff = (double)ctas / (double)(waves * slots);
      const double busy = (double)(nsteps / ks) / wpm;  // warps with work
      if (busy < 1.0) eff *= busy;
      // prefer fewer splits / bigger tiles on (near) ties
      const double score = eff - 0.002 * ks - 0.001 * (4 - mt);
      if (score > best_score) {
        best_score = score;
        best = Plan{mt, ks, smem};
      }
    }
  }
  return best;
}

template <int FMT, int NG>
static int launch_gemv_t(const GemvArgs& a) {
  const Plan pl = make_plan<FMT, NG>(a.B, a.N, a.K, a.ws_bytes);
  GemvParams p;
  p.x = reinterpret_cast<const __half*>(a.x);
  p.ldx = a.ldx;
  p.w = reinterpret_cast<const uint8_t*>(a.w);
  p.s = reinterpret_cast<const __half*>(a.s);
  p.y = reinterpret_cast<__half*>(a.y);
  p.ldy = a.ldy;
  p.B = a.B;
  p.N = a.N;
  p.K = a.K;
  p.mt = pl.mt;
  p.ksplit = pl.ksplit;
  p.prologue = a.prologue;
  p.norm_w = reinterpret_cast<const __half*>(a.norm_w);
  p.eps = a.eps;
  p.ss_in = a.ss_in;
  p.ss_in_parts = a.ss_in_parts;
  p.res = reinterpret_cast<const __half*>(a.res);
  p.ldres = a.ldres;
  p.ss_out = a.ss_out;
  p.npush = a.npush;
  for (int q = 0; q < 8; ++q) p.y32p[q] = q < a.npush ? a.y32p[q] : nullptr;
  p.tpx = a.tpx;
  p.cnt = gemv_counters(a.ws);
  p.part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(a.ws) + gemv_cnt_bytes(a.N));
  if (pl.ksplit > 1 && a.ws == nullptr)
    return set_error(R4Q_ERR_CAPACITY, "gemv: workspace required for N=%d K=%d", a.N, a.K);
  dim3 grid((a.N + 16 * pl.mt - 1) / (16 * pl.mt), pl.ksplit);
  gemv_kernel<FMT, NG><<<grid, kThreads, pl.smem, a.stream>>>(p);
  return check_launch("gemv_kernel");
}

// Workspace layout: a 256-byte header whose first int is the status word (set
// to 1 by a kernel whose bounded wait gave up; read by r4q_ws_status), then
// the tile counters, then the fp32 split-K partials.  The counter region has
// a fixed size so that it never overlaps the partials of a call with a
// different N (partials are left behind, counters are not).
constexpr int kMaxTiles16 = 16384;
size_t gemv_cnt_bytes(int N) { (void)N; return kGemvHdrBytes + (size_t)kMaxTiles16 * 4; }
unsigned* gemv_counters(void* ws) {
  return ws ? reinterpret_cast<unsigned*>(reinterpret_cast<uint8_t*>(ws) + kGemvHdrBytes) : nullptr;
}
size_t gemv_ws_bytes_for(int B, int N, int ksplit) {
  return gemv_cnt_bytes(N) + (size_t)ksplit * B * N * sizeof(float);
}

int gemv_validate(const GemvArgs& a, int fmt) {
  if (!a.x || !a.w || (!a.y && !a.npush) || (fmt != W_FP16 && !a.s))
    return set_error(R4Q_ERR_ARG, "gemv: null pointer");
  if (a.npush < 0 || a.npush > 8) return set_error(R4Q_ERR_ARG, "gemv: %d fp32 outputs (max 8)", a.npush);
  for (int q = 0; q < a.npush; ++q)
    if (!a.y32p[q] || !aligned(a.y32p[q], 4)) return set_error(R4Q_ERR_ALIGN, "gemv: fp32 output %d null or misaligned", q);
  if (a.B < 1 || a.B > 16) return set_error(R4Q_ERR_ARG, "gemv: B=%d outside 1..16", a.B);
  if (a.N <= 0 || a.N % 16) return set_error(R4Q_ERR_ARG, "gemv: N=%d must be a positive multiple of 16", a.N);
  if (a.N / 16 > kMaxTiles16) return set_error(R4Q_ERR_ARG, "gemv: N=%d above %d", a.N, kMaxTiles16 * 16);
  if (a.K <= 0 || a.K % 32) return set_error(R4Q_ERR_ARG, "gemv: K=%d must be a positive multiple of 32", a.K);
  if (a.prologue < R4Q_PRO_NONE || a.prologue > R4Q_PRO_RMSNORM_FWHT)
    return set_error(R4Q_ERR_ARG, "gemv: unknown prologue %d", a.prologue);
  if (a.prologue == R4Q_PRO_RMSNORM_FWHT) {
    if (!a.norm_w || !aligned(a.norm_w, 16))
      return set_error(R4Q_ERR_ARG, "gemv: RMSNorm prologue needs a 16-byte aligned norm weight");
    if (a.ss_in && a.ss_in_parts <= 0) return set_error(R4Q_ERR_ARG, "gemv: ss_in_parts must be > 0");
  }
  if (a.res && (a.B > 1 && a.ldres < a.N)) return set_error(R4Q_ERR_ARG, "gemv: ldres < N");
  const long kin = (a.prologue == R4Q_PRO_SILU_FWHT) ? 2L * a.K : a.K;
  if (a.B > 1 && a.ldx < kin) return set_error(R4Q_ERR_ARG, "gemv: ldx=%ld < %ld", a.ldx, kin);
  if (a.B > 1 && a.ldy < a.N) return set_error(R4Q_ERR_ARG, "gemv: ldy=%ld < N", a.ldy);
  if (!aligned(a.x, 16) || (a.ldx % 8)) return set_error(R4Q_ERR_ALIGN, "gemv: x must be 16-byte aligned with ldx % 8 == 0");
  if (!aligned(a.w, 16)) return set_error(R4Q_ERR_ALIGN, "gemv: weights must be 16-byte aligned");
  if (fmt == W_INT4 && !aligned(a.s, 4)) return set_error(R4Q_ERR_ALIGN, "gemv: scales must be 4-byte aligned");
  if (fmt == W_INT8 && !aligned(a.s, 2)) return set_error(R4Q_ERR_ALIGN, "gemv: scales must be 2-byte aligned");
  if (!aligned(a.y, 2)) return set_error(R4Q_ERR_ALIGN, "gemv: y misaligned");
  return R4Q_OK;
}

int launch_gemv(const GemvArgs& a, int fmt) {
  int st = gemv_validate(a, fmt);
  if (st) return st;
  // The TMA kernel takes every shape it supports (measured on B200 at B =
  // 1..16 against this file's register-staged kernel, which stays for the
  // shapes TMA cannot take); the choice depends on the shape only, never on
  // the output type, so fp16(y32) == y16 holds bit for bit.
  // R4Q_GEMV_PATH=ldg forces the register-staged kernel (testing only).
  static const bool force_ldg = [] {
    const char* e = getenv("R4Q_GEMV_PATH");
    return e && e[0] == 'l';
  }();
  // R4Q_GEMV_TC=1: INT4 at B = 3..16 through the tcgen05 kernel (weights
  // dequantised into tensor memory; measured slower than the TMA kernel, so
  // opt-in); it declines (capacity) when the workspace cannot hold its
  // prepared activations, and takes no tensor-parallel exchange.
  if (!force_ldg && gemv_tc_eligible(a, fmt)) {
    st = launch_gemv_tc(a);
    if (st != R4Q_ERR_CAPACITY) return st;
  }
  if (!force_ldg && gemv_tma_supported(a, fmt)) {
    st = launch_gemv_tma(a, fmt);
    if (st != R4Q_ERR_CAPACITY) return st;  // no TMA plan fits: take the LDG kernel
  }
  if (a.tpx.nwait)
    return set_error(R4Q_ERR_ARG, "gemv: the tensor-parallel reduce prologue needs the TMA path");
  const bool two = a.B > 8;
  switch (fmt) {
    case W_INT4: return two ? launch_gemv_t<W_INT4, 2>(a) : launch_gemv_t<W_INT4, 1>(a);
    case W_INT8: return two ? launch_gemv_t<W_INT8, 2>(a) : launch_gemv_t<W_INT8, 1>(a);
    case W_FP16: return two ? launch_gemv_t<W_FP16, 2>(a) : launch_gemv_t<W_FP16, 1>(a);
  }
  return set_error(R4Q_ERR_ARG, "gemv: unknown weight format %d", fmt);
}

}  // namespace r4q

// ------------------------------------------------------------------ C ABI --
using namespace r4q;

extern "C" size_t r4q_gemv_workspace_bytes(int B, int N, int K) {
  if (B < 1) B = 1;
  if (N < 16) N = 16;
  // enough partial slots for the K splits the planners pick (they cap the
  // split count by the workspace they are given)
  long cap = ((long)num_sms() * 64 * 8 + N - 1) / N;
  if (cap < kMaxSplit) cap = kMaxSplit;
  if (cap > 32) cap = 32;
  return gemv_ws_bytes_for(B, N, (int)cap) + (B >= 3 ? gemv_tc_extra_bytes(B, K < 128 ? 128 : K) : 0);
}

static GemvArgs mk(const void* x, long ldx, const void* w, const void* s, void* y, long ldy, int B,
                   int N, int K, int prologue, void* ws, size_t wsb, void* stream) {
  GemvArgs a{};
  a.x = x; a.ldx = ldx; a.w = w; a.s = s; a.y = y; a.ldy = ldy;
  a.B = B; a.N = N; a.K = K; a.prologue = prologue;
  a.ws = ws; a.ws_bytes = ws ? wsb : 0;
  a.stream = reinterpret_cast<cudaStream_t>(stream);
  return a;
}

extern "C" int r4q_gemv_int4(const void* x, long ldx, const void* w, const void* sz, void* y,
                             long ldy, int B, int N, int K, int prologue, void* ws, size_t wsb,
                             void* stream) {
  return launch_gemv(mk(x, ldx, w, sz, y, ldy, B, N, K, prologue, ws, wsb, stream), W_INT4);
}
extern "C" int r4q_gemv_int8(const void* x, long ldx, const void* w, const void* s, void* y,
                             long ldy, int B, int N, int K, int prologue, void* ws, size_t wsb,
                             void* stream) {
  return launch_gemv(mk(x, ldx, w, s, y, ldy, B, N, K, prologue, ws, wsb, stream), W_INT8);
}
extern "C" int r4q_gemv_fp16(const void* x, long ldx, const void* w, void* y, long ldy, int B,
                             int N, int K, int prologue, void* ws, size_t wsb, void* stream) {
  return launch_gemv(mk(x, ldx, w, nullptr, y, ldy, B, N, K, prologue, ws, wsb, stream), W_FP16);
}

extern "C" int r4q_gemv(int wfmt, const void* x, long ldx, const void* w, const void* s, void* y,
                        long ldy, int B, int N, int K, int prologue, const r4q_gemv_fused* f,
                        void* ws, size_t wsb, void* stream) {
  GemvArgs a = mk(x, ldx, w, s, y, ldy, B, N, K, prologue, ws, wsb, stream);
  if (f) {
    a.norm_w = f->norm_w;
    a.eps = f->eps;
    a.ss_in = f->ss_in;
    a.ss_in_parts = f->ss_in_parts;
    a.res = f->residual;
    a.ldres = (B > 1) ? f->ldres : N;
    a.ss_out = f->ss_out;
    if (f->y32) {
      a.y32p[0] = f->y32;
      a.npush = 1;
    }
  }
  if (a.prologue == R4Q_PRO_RMSNORM_FWHT && !f)
    return set_error(R4Q_ERR_ARG, "gemv: RMSNorm prologue needs fused parameters");
  return launch_gemv(a, wfmt);
}
