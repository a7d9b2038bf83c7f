// Mixture-of-experts decode FFN (benchmark config 4, Qwen3-30B-A3B shape: 128
// experts, top-8 softmax routing, INT4 experts).  No counterpart in the
// reference, whose engine is dense; the expert projections reuse the dense
// path's conventions: INT4 runtime layout (nibbles [N, K/2], (scale, zero)
// fp16 pairs [N, K/16]), H32-rotated weights fed FWHT'd activations, exact
// fp16((q - z) s) dequantisation, fp32 accumulation.
//
// Kernels (one decode layer's FFN):
//  * moe_route_kernel: per token softmax over the router logits (fp32), top-k
//    (ties to the lower expert), weights renormalised over the k; then the
//    (token, slot) pairs grouped by expert in token order — a deterministic
//    counting sort in one CTA (warp scan of the counts, match_any ranks) —
//    and the ascending list of active experts;
//  * moe_gemv_kernel: grouped dequant-GEMV.  CTAs walk the work items
//    (active expert, 64-row tile), an expert's tiles adjacent, the item count
//    read on the device; the grid is fixed (one CTA per possible item), so
//    the launch can live in a CUDA graph.  8 warps = 4 m-tiles x 2 K halves.  Lane t of a warp
//    owns whole 32-k blocks (block 4q + t of batch q): one 128-bit load per
//    row brings its 32 nibbles, so a warp load covers 64 contiguous bytes of
//    8 rows; the k order inside the m16n8k16 fragments is permuted to match
//    (the activations are read with the same permutation, so the dot products
//    are unchanged).  Tokens are the N dimension, 8 per pass.  Mode 2 is
//    gate_up with the SiLU(gate)·up + H32 FWHT epilogue (the tile holds 32
//    gate rows and the matching 32 up rows), writing down_proj's input;
//  * moe_combine_kernel: h = fp16(fp16(Σ_k w_k fp16(y_k)) + residual) in slot
//    order, with the per-16-row sums of squares the next RMSNorm prologue takes.
#include <cuda.h>

#include <atomic>
#include <cstdlib>
#include <mutex>

#include "r4q_common.cuh"

namespace r4q {
namespace {

constexpr int kMoeTok = 8;              // tokens per pass (one m16n8k16 n-group)
constexpr int kMoeThreads = 256;        // 8 warps: 4 m-tiles x 2 K halves
constexpr int kMoeKp = 2;
constexpr int kMoeUnroll = 4;           // 128-k batches whose weight loads are in flight together

struct MoeRoute {
  const int* counts;      // [E]
  const int* offsets;     // [E + 1]
  const int* list;        // [B * topk] entries t * topk + k grouped by expert
  const int* active;      // [E] active experts, ascending
  const int* n_active;    // [1]
};

// ---------------------------------------------------------------- routing
// Top-k of B tokens, G lanes per token (32 / G tokens per warp at once):
// logits in registers (expert sub + G i, PL = 256 / G per lane), softmax,
// top-k by repeated arg-max over the experts not yet taken; reductions stay
// inside the G-lane group.  Writes ids / wts, s_ids and the counts s_cnt.
template <int G>
__device__ __forceinline__ void route_topk(const __half* logits, int B, int E, int topk, int* ids, float* wts,
                                           int* s_cnt, int* s_ids, int warp, int lane, int nw) {
  constexpr int PL = 256 / G;
  const int sub = lane & (G - 1);
  for (int b0 = warp * (32 / G); b0 < B; b0 += nw * (32 / G)) {
    const int b = b0 + lane / G;
    const bool valid = b < B;
    const __half* lr = logits + (long)b * E;
    float lv[PL];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      const int e = sub + G * i;
      lv[i] = (valid && e < E) ? __half2float(__ldcg(lr + e)) : -INFINITY;
      mx = fmaxf(mx, lv[i]);
    }
    for (int o = G / 2; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < PL; ++i)
      if (valid && sub + G * i < E) sum += expf(lv[i] - mx);
    for (int o = G / 2; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    uint32_t taken = 0;
    float psel = 0.0f, pm[2] = {0.f, 0.f};
    int im[2] = {0, 0};
    for (int k = 0; k < topk; ++k) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < PL; ++i) {
        const int e = sub + G * i;
        if (e < E && !((taken >> i) & 1u) && (lv[i] > bv || (lv[i] == bv && e < bi))) {
          bv = lv[i];
          bi = e;
        }
      }
      for (int o = G / 2; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (valid && bi < E && (bi & (G - 1)) == sub) taken |= 1u << (bi / G);
      const float p = expf(bv - mx) / sum;
      psel += p;
      if (k % G == sub) {
        if (k < G) {
          pm[0] = p;
          im[0] = bi;
        } else {
          pm[1] = p;
          im[1] = bi;
        }
      }
    }
    if (valid)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int kk = sub + G * h;
        if (kk < topk) {
          ids[b * topk + kk] = im[h];
          wts[b * topk + kk] = pm[h] / psel;
          s_ids[b * topk + kk] = im[h];
          atomicAdd(&s_cnt[im[h]], 1);
        }
      }
  }
}

// The whole routing of B tokens by one CTA (any multiple of 32 threads);
// sm: (3 E + B * topk) ints.  Logits are read through L2 (.cg): in the fused
// router they were written by other CTAs of the same grid.
__device__ void route_tokens(const __half* logits, int B, int E, int topk, int e_lo, int e_hi, int* ids, float* wts,
                             int* counts, int* offsets, int* list, int* active, int* n_active, int* sm) {
  int* s_cnt = sm;                  // [E]
  int* s_off = sm + E;              // [E]
  int* s_run = sm + 2 * E;          // [E]
  int* s_ids = sm + 3 * E;          // [B * topk]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
  for (int e = tid; e < E; e += blockDim.x) s_cnt[e] = s_run[e] = 0;
  __syncthreads();
  // small batches: a warp per token (short per-lane loops); large: 8 lanes
  if (B <= nw) route_topk<32>(logits, B, E, topk, ids, wts, s_cnt, s_ids, warp, lane, nw);
  else route_topk<8>(logits, B, E, topk, ids, wts, s_cnt, s_ids, warp, lane, nw);
  __syncthreads();
  const int n = B * topk;
  if (warp == 0) {
    // offsets (exclusive scan of the counts) and the active experts in
    // [e_lo, e_hi), ascending: lane owns experts [lane * per, lane * per + per)
    const int per = (E + 31) / 32;
    int c = 0, a = 0;
    for (int i = 0; i < per; ++i) {
      const int e = lane * per + i;
      if (e < E) {
        c += s_cnt[e];
        a += (s_cnt[e] > 0 && e >= e_lo && e < e_hi);
      }
    }
    int cs = c, as = a;
    for (int o = 1; o < 32; o <<= 1) {
      const int oc = __shfl_up_sync(0xffffffffu, cs, o), oa = __shfl_up_sync(0xffffffffu, as, o);
      if (lane >= o) {
        cs += oc;
        as += oa;
      }
    }
    int off = cs - c, na = as - a;
    for (int i = 0; i < per; ++i) {
      const int e = lane * per + i;
      if (e < E) {
        s_off[e] = off;
        offsets[e] = off;
        counts[e] = s_cnt[e];
        if (s_cnt[e] > 0 && e >= e_lo && e < e_hi) active[na++] = e;
        off += s_cnt[e];
      }
    }
    if (lane == 31) {
      offsets[E] = off;
      *n_active = na;
    }
    __syncwarp();
    // stable placement, 32 entries at a time: rank among the same expert's
    // entries of this group, after those of the earlier groups
    for (int c0 = 0; c0 < n; c0 += 32) {
      const int j = c0 + lane;
      const int e = j < n ? s_ids[j] : -1;
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      const int r = __popc(peers & ((1u << lane) - 1u));
      if (j < n) list[s_off[e] + s_run[e] + r] = j;
      __syncwarp();
      if (j < n && r == 0) s_run[e] += __popc(peers);
      __syncwarp();
    }
  }
}

__global__ void __launch_bounds__(512) moe_route_kernel(const __half* __restrict__ logits, int B, int E, int topk,
                                                        int e_lo, int e_hi, int* ids, float* wts, int* counts,
                                                        int* offsets, int* list, int* active, int* n_active) {
  pdl_wait_trigger();
  extern __shared__ int sm_route[];
  route_tokens(logits, B, E, topk, e_lo, e_hi, ids, wts, counts, offsets, list, active, n_active, sm_route);
}

// rrms of row b from the per-16-row sums of squares [parts][rows] (fixed
// order: lane-strided partial sums, then lanes 0..31) — the arithmetic of
// the GEMV prologue.  Called by warp 0; result in lane 0..31 alike.
__device__ __forceinline__ float rrms_from_parts(const float* ss_in, int parts, int rows, int b, int D, float eps,
                                                 int lane) {
  float ss = 0.0f;
  for (int i = lane; i < parts; i += 32) ss += ss_in[(long)i * rows + b];
  float t = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) t += __shfl_sync(0xffffffffu, ss, i);
  return rsqrtf(t / (float)D + eps);
}

// ------------------------------------------------------------ fused router
// One pass for the router of a decode layer: xn = fp16(H32(r * rrms * w))
// (when w is given; else xn is read as given), logits[b][e] = fp16(W_r[e] ·
// xn[b]) with W_r fp16 [E, D] (H32-rotated), then the last CTA to finish
// routes (route_tokens).  CTA (c, t): experts [8c, 8c + 8), one warp each
// (the router row in registers, D <= 2048), tokens [16t, 16t + 16) staged in
// shared memory.  `done` [1] int counts finished CTAs
// and is reset by the last one.
constexpr int kRouterTok = 16;
__global__ void __launch_bounds__(256) moe_router_kernel(const __half* __restrict__ x, const float* __restrict__ ss_in,
                                                         int parts, const __half* __restrict__ nw, float eps,
                                                         __half* __restrict__ xn, const __half* __restrict__ wr,
                                                         __half* logits, int B, int D, int E, int topk, int e_lo,
                                                         int e_hi, int* ids, float* wts, int* counts, int* offsets,
                                                         int* list, int* active, int* n_active, int* done) {
  extern __shared__ __align__(16) uint8_t sm_r[];
  __half* xs = reinterpret_cast<__half*>(sm_r);                  // [16][D]
  __shared__ float s_rr[kRouterTok];
  __shared__ int s_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int e = blockIdx.x * 8 + warp;
  const int nv = D / 256;                                         // uint4 per lane
  uint4 wv[8];
  if (e < E) {                                                    // weights: no dependence on the previous kernel
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < nv) wv[i] = __ldg(reinterpret_cast<const uint4*>(wr + (long)e * D) + i * 32 + lane);
  }
  pdl_wait_trigger();
  {
    const int b0 = blockIdx.y * kRouterTok;          // this CTA's 16 tokens
    const int nb = min(kRouterTok, B - b0);
    if (nw) {
      // one warp per (row, 32-block), 8 blocks per warp per round with their
      // loads first; the first round's loads go out before the rrms is known.
      // CTA c also stores the blocks c, c + G, ... of xn.
      const int items = nb * (D / 32);                 // >= 8: every warp takes part in round 0
      for (int i0 = warp; i0 < items; i0 += 64) {
        float xv[8], wv8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int i = i0 + 8 * u;
          if (i < items) {
            const int r = i / (D / 32), k = (i - r * (D / 32)) * 32 + lane;
            xv[u] = __half2float(x[(long)(b0 + r) * D + k]);
            wv8[u] = __half2float(nw[k]);
          }
        }
        if (i0 == warp) {
          if (warp == 0)
            for (int r = 0; r < nb; ++r) {
              const float rr = rrms_from_parts(ss_in, parts, B, b0 + r, D, eps, lane);
              if (lane == 0) s_rr[r] = rr;
            }
          __syncthreads();
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int i = i0 + 8 * u;
          if (i < items) {
            const int r = i / (D / 32), blk = i - r * (D / 32), k = blk * 32 + lane;
            const __half h = __float2half(fwht32_lane(xv[u] * s_rr[r] * wv8[u], lane));
            xs[r * D + k] = h;
            if (blk % gridDim.x == blockIdx.x) xn[(long)(b0 + r) * D + k] = h;
          }
        }
      }
    } else {
      for (int i = tid; i < nb * (D / 8); i += 256) {
        const int r = i / (D / 8), c = i - r * (D / 8);
        reinterpret_cast<uint4*>(xs + r * D)[c] = reinterpret_cast<const uint4*>(xn + (long)(b0 + r) * D)[c];
      }
    }
    __syncthreads();
    if (e < E)
      for (int r0 = 0; r0 < nb; r0 += 4) {             // 4 tokens at once: independent FMA chains
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (i < nv) {
            const uint32_t wq[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int r = min(r0 + u, nb - 1);
              const uint4 xv = reinterpret_cast<const uint4*>(xs + r * D)[i * 32 + lane];
              const uint32_t xq[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float2 wf = __half22float2(u32_as_h2(wq[j])), xf = __half22float2(u32_as_h2(xq[j]));
                acc[u] = fmaf(wf.x, xf.x, acc[u]);
                acc[u] = fmaf(wf.y, xf.y, acc[u]);
              }
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float v = warp_sum(acc[u]);
          if (lane == 0 && r0 + u < nb) logits[(long)(b0 + r0 + u) * E + e] = __float2half(v);
        }
      }
  }
  // ---- the last CTA routes
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = (atomicAdd(done, 1) == (int)(gridDim.x * gridDim.y) - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  route_tokens(logits, B, E, topk, e_lo, e_hi, ids, wts, counts, offsets, list, active, n_active,
               reinterpret_cast<int*>(sm_r));
  if (tid == 0) *done = 0;
}

// ------------------------------------------------- row RMSNorm + H32 FWHT
// y = fp16(H32(fp16... x * rrms * w)) per 32-block: the RMSNorm+FWHT prologue
// of the dense GEMVs as a standalone pass (rrms from ss_in partials or x).
__global__ void norm_fwht_kernel(const __half* __restrict__ x, const float* __restrict__ ss_in, int parts,
                                 const __half* __restrict__ w, float eps, __half* __restrict__ y, int D) {
  pdl_wait_trigger();
  const int b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  __shared__ float s_r;
  __shared__ float s_part[32];
  const __half* xr = x + (long)b * D;
  if (warp == 0) {
    float ss = 0.0f;
    if (ss_in) {
      for (int i = lane; i < parts; i += 32) ss += ss_in[(long)i * gridDim.x + b];
    }
    s_part[lane] = ss;
  }
  float ssx = 0.0f;
  if (!ss_in)
    for (int i = tid; i < D; i += blockDim.x) {
      const float v = __half2float(xr[i]);
      ssx += v * v;
    }
  ssx = warp_sum(ssx);
  __syncthreads();
  if (!ss_in && lane == 0) s_part[warp] = ssx;
  __syncthreads();
  if (tid == 0) {
    float t = 0.0f;
    for (int i = 0; i < (ss_in ? 32 : nw); ++i) t += s_part[i];
    s_r = rsqrtf(t / (float)D + eps);
  }
  __syncthreads();
  const float rr = s_r;
  for (int b0 = warp; b0 < D / 32; b0 += 8 * nw) {     // 8 blocks per warp per round, loads first
    float xv[8], wv8[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int blk = b0 + u * nw;
      if (blk < D / 32) {
        xv[u] = __half2float(xr[blk * 32 + lane]);
        wv8[u] = __half2float(w[blk * 32 + lane]);
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int blk = b0 + u * nw;
      if (blk < D / 32) y[(long)b * D + blk * 32 + lane] = __float2half(fwht32_lane(xv[u] * rr * wv8[u], lane));
    }
  }
}

// ------------------------------------------------------ grouped expert GEMV
// MODE 0: plain, activation of entry j = xin[j / topk] (rows of K), y[j] [N].
// MODE 1: plain, activation of entry j = xin[j].
// MODE 2 (gate_up, N = 2 Ie): activation xin[j / topk]; y[j] [Ie] =
// fp16(H32(silu(g) * u)), g, u = fp16 gate / up outputs, one rounding
// (silu_hadamard_ds, :1031-1051).  Tile x of mode 2 covers gate rows
// [32x, 32x + 32) (m-tiles 0, 1) and up rows Ie + [32x, 32x + 32) (2, 3).
template <int MODE>
__global__ void __launch_bounds__(kMoeThreads, 2)
    moe_gemv_kernel(const uint8_t* __restrict__ w, const __half* __restrict__ sz, const __half* __restrict__ xin,
                    long ldx, __half* __restrict__ y, long ldy, int N, int K, int topk, int e_lo,
                    const MoeRoute rt) {
  pdl_wait_trigger();
  __shared__ float red[4][4][32];                 // K half 1 -> K half 0
  __shared__ float cs[kMoeTok][64];               // mode 2: fp16-rounded gate | up per token
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int mt = warp & 3, kp = warp >> 2;
  const int nbat = K / 128;                        // 4 blocks of 32 k per batch
  const int q0 = (nbat * kp) / kMoeKp, q1 = (nbat * (kp + 1)) / kMoeKp;
  const long wrow = (long)K / 2, srow = (long)K / 16;
  const int tiles = N / 64;
  const int items = *rt.n_active * tiles;          // (active expert, 64-row tile), tiles of an expert adjacent
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    const int a = it / tiles, tile = it - a * tiles;
    const int e = rt.active[a];
    const int cnt = rt.counts[e];
    const int* ent = rt.list + rt.offsets[e];
    int ra;
    if (MODE == 2) ra = (mt < 2 ? 0 : N / 2) + tile * 32 + (mt & 1) * 16 + g;
    else ra = tile * 64 + mt * 16 + g;
    const long el = e - e_lo;                        // this GPU's expert slice starts at e_lo
    const uint8_t* wa = w + (el * N + ra) * wrow + t * 16;
    const uint8_t* wb = wa + 8 * wrow;
    const __half* sa = sz + (el * N + ra) * srow + t * 2;
    const __half* sb = sa + 8 * srow;

    for (int c0 = 0; c0 < cnt; c0 += kMoeTok) {
      const int nc = min(kMoeTok, cnt - c0);
      const bool tok_ok = g < nc;
      const __half* xr = xin + t * 32;
      if (tok_ok) {
        const int j = ent[c0 + g];
        xr += (long)(MODE == 1 ? j : j / topk) * ldx;
      }
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int q = q0; q < q1; q += kMoeUnroll) {
        uint4 qa[kMoeUnroll], qb[kMoeUnroll];
        uint32_t pa[kMoeUnroll], pb[kMoeUnroll];
#pragma unroll
        for (int u = 0; u < kMoeUnroll; ++u) {          // every weight load of the batches first
          if (q + u < q1) {
            qa[u] = __ldg(reinterpret_cast<const uint4*>(wa + (long)(q + u) * 64));
            qb[u] = __ldg(reinterpret_cast<const uint4*>(wb + (long)(q + u) * 64));
            pa[u] = __ldg(reinterpret_cast<const unsigned*>(sa + (q + u) * 8));
            pb[u] = __ldg(reinterpret_cast<const unsigned*>(sb + (q + u) * 8));
          }
        }
#pragma unroll
        for (int u = 0; u < kMoeUnroll; ++u) {
          if (q + u >= q1) break;
          uint4 xv[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            xv[i] = tok_ok ? __ldg(reinterpret_cast<const uint4*>(xr + (long)(q + u) * 128 + 8 * i))
                           : make_uint4(0, 0, 0, 0);
          const __half2 pha = u32_as_h2(pa[u]), phb = u32_as_h2(pb[u]);
          // biased nibbles: low half 1024 + q (nibble in mantissa bits 0-3),
          // high half 64 + q (bits 4-7 of a 64-based fp16), both exact, so
          // subtracting (1024 + z, 64 + z) and one multiply by s give the
          // reference's fp16((q - z) s)
          const __half2 bias = __halves2half2(__float2half(1024.0f), __float2half(64.0f));
          const __half2 s2a = __half2half2(__low2half(pha)), z2a = __hadd2(__half2half2(__high2half(pha)), bias);
          const __half2 s2b = __half2half2(__low2half(phb)), z2b = __hadd2(__half2half2(__high2half(phb)), bias);
          const uint32_t wa4[4] = {qa[u].x, qa[u].y, qa[u].z, qa[u].w};
          const uint32_t wb4[4] = {qb[u].x, qb[u].y, qb[u].z, qb[u].w};
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            // k-step jj: this lane's block bytes 2jj (k 4jj, 4jj+1) and 2jj+1
            // (k 4jj+2, 4jj+3) stand for fragment k (2t, 2t+1) and (2t+8, 2t+9);
            // the byte is copied to both halves and one LOP3 keeps lo / hi nibble
            const uint32_t sl = (uint32_t)(2 * (jj & 1)) * 0x1111u, sh = sl + 0x1111u;
            const uint32_t wA = wa4[jj >> 1], wB = wb4[jj >> 1];
            const uint32_t lA = lop3_and_or(__byte_perm(wA, 0, sl), 0x00F0000Fu, 0x54006400u);
            const uint32_t hA = lop3_and_or(__byte_perm(wA, 0, sh), 0x00F0000Fu, 0x54006400u);
            const uint32_t lB = lop3_and_or(__byte_perm(wB, 0, sl), 0x00F0000Fu, 0x54006400u);
            const uint32_t hB = lop3_and_or(__byte_perm(wB, 0, sh), 0x00F0000Fu, 0x54006400u);
            const uint32_t a0 = h2_as_u32(__hmul2(__hsub2(u32_as_h2(lA), z2a), s2a));
            const uint32_t a2 = h2_as_u32(__hmul2(__hsub2(u32_as_h2(hA), z2a), s2a));
            const uint32_t a1 = h2_as_u32(__hmul2(__hsub2(u32_as_h2(lB), z2b), s2b));
            const uint32_t a3 = h2_as_u32(__hmul2(__hsub2(u32_as_h2(hB), z2b), s2b));
            const uint4 xq = xv[jj >> 1];
            const uint32_t b0 = (jj & 1) ? xq.z : xq.x, b1 = (jj & 1) ? xq.w : xq.y;
            mma16816(acc, a0, a1, a2, a3, b0, b1);
          }
        }
      }
      // ---- K half 1 hands its partial to K half 0 (fixed order)
      if (kp == 1) {
#pragma unroll
        for (int i = 0; i < 4; ++i) red[mt][i][lane] = acc[i];
      }
      __syncthreads();
      if (kp == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i] += red[mt][i][lane];
        // C: (row g, tokens 2t, 2t+1), (row g + 8, tokens 2t, 2t+1)
        if (MODE == 2) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            cs[2 * t + (i & 1)][mt * 16 + g + 8 * (i >> 1)] = __half2float(__float2half(acc[i]));
        } else {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int tok = 2 * t + h;
            if (tok < nc) {
              __half* yr = y + (long)ent[c0 + tok] * ldy;
              yr[ra] = __float2half(acc[h]);
              yr[ra + 8] = __float2half(acc[2 + h]);
            }
          }
        }
      }
      if (MODE == 2) {
        __syncthreads();
        if (warp < nc) {      // warp = token of the pass
          const float gg = cs[warp][lane], uu = cs[warp][32 + lane];
          const float v = fwht32_lane(gg / (1.0f + expf(-gg)) * uu, lane);
          y[(long)ent[c0 + warp] * ldy + tile * 32 + lane] = __float2half(v);
        }
      }
      __syncthreads();        // red / cs are rewritten by the next pass
    }
  }
}

// ------------------------------------------- grouped expert GEMV, TMA tiles
// Same work and modes as moe_gemv_kernel, for K % 256 == 0 and a 64-row tile
// that fits shared memory (64 x K/2 bytes): one TMA burst brings the tile's
// nibbles (128-byte columns x 32-row boxes, 128-byte swizzle) while the
// (scale, zero) pairs and the routing metadata load; up to three CTAs per SM
// keep ~200 KB per SM in flight, where the register-staged kernel holds
// 64 KB.  Lane (g, t) then reads its 16-byte block chunks from shared memory
// (conflict-free under the swizzle) and computes exactly as the LDG kernel.
__device__ __forceinline__ uint32_t moe_su32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ bool moe_mbar_wait(uint64_t* b, unsigned parity) {
  const uint32_t a = moe_su32(b);
  for (long i = 0; i < (1L << 26); ++i) {
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                 " selp.u32 %0, 1, 0, p;\n}\n" : "=r"(ok) : "r"(a), "r"(parity) : "memory");
    if (ok) return true;
  }
  return false;
}

constexpr int kMoeTmaMaxPairs = 8;      // 128-k batches per K half held in registers (K <= 8192)

template <int MODE>
__global__ void __launch_bounds__(kMoeThreads, 3)
    moe_gemv_tma_kernel(const __grid_constant__ CUtensorMap tmw, const __half* __restrict__ sz,
                        const __half* __restrict__ xin, long ldx, __half* __restrict__ y, long ldy, int N, int K,
                        int topk, int e_lo, const MoeRoute rt, int* status) {
  extern __shared__ __align__(1024) uint8_t moe_smem[];
  uint8_t* wsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(moe_smem) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bars[kMoeKp];             // one per K half: its warps start when it lands
  __shared__ float red[4][4][32];
  __shared__ float cs[kMoeTok][64];
  pdl_wait_trigger();
  const int a = blockIdx.y;
  if (a >= *rt.n_active) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int mt = warp & 3, kp = warp >> 2;
  const int e = rt.active[a];
  const int tile = blockIdx.x;
  const long el = e - e_lo;
  // tile rows: smem rows 0-31 from global row r0, 32-63 from r1
  const int r0 = MODE == 2 ? tile * 32 : tile * 64;
  const int r1 = MODE == 2 ? N / 2 + tile * 32 : tile * 64 + 32;
  const int ncol = K / 256;                                   // 128-byte columns of nibbles
  // K half p covers 128-k batches [nbat p / 2, nbat (p + 1) / 2); its 128-byte
  // columns (two batches each, a batch is 64 bytes of a row) load on bars[p]
  const int nbat = K / 128;
  const int q0 = (nbat * kp) / kMoeKp, q1 = (nbat * (kp + 1)) / kMoeKp;
  if (tid == 0) {
#pragma unroll
    for (int p = 0; p < kMoeKp; ++p) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(moe_su32(&bars[p])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0) {
    // column b (batches 2b, 2b + 1) belongs to the half of batch 2b; a
    // column split between halves (odd batch count per half) goes to the
    // first half, whose warps then also hold the second half's first batch
    int cb[kMoeKp + 1];
    cb[0] = 0;
    for (int p = 1; p <= kMoeKp; ++p) cb[p] = ((nbat * p) / kMoeKp + 1) / 2;
    for (int p = 0; p < kMoeKp; ++p) {
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(moe_su32(&bars[p])),
                   "r"((cb[p + 1] - cb[p]) * 8192) : "memory");
      for (int b = cb[p]; b < cb[p + 1]; ++b)
#pragma unroll
        for (int h = 0; h < 2; ++h)
          asm volatile(
              "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
              " [%0], [%1, {%2, %3}], [%4];" ::"r"(moe_su32(wsm + (2 * b + h) * 4096)),
              "l"(reinterpret_cast<uint64_t>(&tmw)), "r"(b * 128), "r"((int)(el * N) + (h ? r1 : r0)),
              "r"(moe_su32(&bars[p]))
              : "memory");
    }
  }
  // while the tile lands: this lane's (scale, zero) pairs and the routing
  const int lr = mt * 16 + g;                                  // tile row of fragment rows g (and g + 8)
  const int gra = (lr < 32 ? r0 + lr : r1 + lr - 32), grb = gra + 8;
  const long srow = (long)K / 16;
  const __half* sa = sz + (el * N + gra) * srow + t * 2;
  const __half* sb = sz + (el * N + grb) * srow + t * 2;
  uint32_t pa[kMoeTmaMaxPairs], pb[kMoeTmaMaxPairs];
#pragma unroll
  for (int i = 0; i < kMoeTmaMaxPairs; ++i) {
    if (q0 + i < q1) {
      pa[i] = __ldg(reinterpret_cast<const unsigned*>(sa + (q0 + i) * 8));
      pb[i] = __ldg(reinterpret_cast<const unsigned*>(sb + (q0 + i) * 8));
    }
  }
  const int cnt = rt.counts[e];
  const int* ent = rt.list + rt.offsets[e];
  // the columns this warp reads: batches [q0, q1) lie in columns
  // [q0 / 2, (q1 + 1) / 2), which bars[kp] covers — and, when q0 is odd,
  // column q0 / 2 sits with the previous half
  bool landed = moe_mbar_wait(&bars[kp], 0);
  if (landed && kp > 0 && (q0 & 1)) landed = moe_mbar_wait(&bars[kp - 1], 0);
  if (__syncthreads_or(!landed)) {                            // a wait gave up: the whole CTA leaves
    if (tid == 0 && status) atomicExch(status, 1);
    return;
  }
  const int ra_out = MODE == 2 ? 0 : tile * 64 + lr;           // plain modes: output rows ra_out, ra_out + 8
  const uint32_t rowa = moe_su32(wsm) + (lr >> 5) * 4096 + (lr & 31) * 128;
  const uint32_t rowb = moe_su32(wsm) + ((lr + 8) >> 5) * 4096 + ((lr + 8) & 31) * 128;
  const int swa = (lr & 31) & 7, swb = ((lr + 8) & 31) & 7;
  const __half2 bias = __halves2half2(__float2half(1024.0f), __float2half(64.0f));

  for (int c0 = 0; c0 < cnt; c0 += kMoeTok) {
    const int nc = min(kMoeTok, cnt - c0);
    const bool tok_ok = g < nc;
    const __half* xr = xin + t * 32;
    if (tok_ok) {
      const int j = ent[c0 + g];
      xr += (long)(MODE == 1 ? j : j / topk) * ldx;
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < kMoeTmaMaxPairs; ++i) {
      const int q = q0 + i;
      if (q >= q1) break;
      const int blk = 4 * q + t, col = blk >> 3, cc = blk & 7;
      uint4 qa, qb;
      asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                   : "=r"(qa.x), "=r"(qa.y), "=r"(qa.z), "=r"(qa.w)
                   : "r"(rowa + col * 8192 + ((cc ^ swa) << 4)));
      asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                   : "=r"(qb.x), "=r"(qb.y), "=r"(qb.z), "=r"(qb.w)
                   : "r"(rowb + col * 8192 + ((cc ^ swb) << 4)));
      uint4 xv[4];
#pragma unroll
      for (int k4 = 0; k4 < 4; ++k4)
        xv[k4] = tok_ok ? __ldg(reinterpret_cast<const uint4*>(xr + (long)q * 128 + 8 * k4)) : make_uint4(0, 0, 0, 0);
      const __half2 pha = u32_as_h2(pa[i]), phb = u32_as_h2(pb[i]);
      const __half2 s2a = __half2half2(__low2half(pha)), z2a = __hadd2(__half2half2(__high2half(pha)), bias);
      const __half2 s2b = __half2half2(__low2half(phb)), z2b = __hadd2(__half2half2(__high2half(phb)), bias);
      const uint32_t wa4[4] = {qa.x, qa.y, qa.z, qa.w}, wb4[4] = {qb.x, qb.y, qb.z, qb.w};
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const uint32_t sl = (uint32_t)(2 * (jj & 1)) * 0x1111u, sh = sl + 0x1111u;
        const uint32_t wA = wa4[jj >> 1], wB = wb4[jj >> 1];
        const uint32_t lA = lop3_and_or(__byte_perm(wA, 0, sl), 0x00F0000Fu, 0x54006400u);
        const uint32_t hA = lop3_and_or(__byte_perm(wA, 0, sh), 0x00F0000Fu, 0x54006400u);
        const uint32_t lB = lop3_and_or(__byte_perm(wB, 0, sl), 0x00F0000Fu, 0x54006400u);
        const uint32_t hB = lop3_and_or(__byte_perm(wB, 0, sh), 0x00F0000Fu, 0x54006400u);
        const uint32_t a0 = h2_as_u32(__hmul2(__hsub2(u32_as_h2(lA), z2a), s2a));
        const uint32_t a2 = h2_as_u32(__hmul2(__hsub2(u32_as_h2(hA), z2a), s2a));
        const uint32_t a1 = h2_as_u32(__hmul2(__hsub2(u32_as_h2(lB), z2b), s2b));
        const uint32_t a3 = h2_as_u32(__hmul2(__hsub2(u32_as_h2(hB), z2b), s2b));
        const uint4 xq = xv[jj >> 1];
        const uint32_t b0 = (jj & 1) ? xq.z : xq.x, b1 = (jj & 1) ? xq.w : xq.y;
        mma16816(acc, a0, a1, a2, a3, b0, b1);
      }
    }
    if (kp == 1) {
#pragma unroll
      for (int i = 0; i < 4; ++i) red[mt][i][lane] = acc[i];
    }
    __syncthreads();
    if (kp == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] += red[mt][i][lane];
      if (MODE == 2) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          cs[2 * t + (i & 1)][mt * 16 + g + 8 * (i >> 1)] = __half2float(__float2half(acc[i]));
      } else {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int tok = 2 * t + h;
          if (tok < nc) {
            __half* yr = y + (long)ent[c0 + tok] * ldy;
            yr[ra_out] = __float2half(acc[h]);
            yr[ra_out + 8] = __float2half(acc[2 + h]);
          }
        }
      }
    }
    if (MODE == 2) {
      __syncthreads();
      if (warp < nc) {
        const float gg = cs[warp][lane], uu = cs[warp][32 + lane];
        const float v = fwht32_lane(gg / (1.0f + expf(-gg)) * uu, lane);
        y[(long)ent[c0 + warp] * ldy + tile * 32 + lane] = __float2half(v);
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------- combine
// Entries of experts in [e_lo, e_hi) only.  out32: the fp32 partial
// Σ_k w[b,k] y[b*topk+k] (expert-parallel: summed over GPUs afterwards).
// Otherwise h[b] = fp16(fp16(Σ) + res[b]) in slot order with ss_out [D/16][B]
// the per-16-row sums of squares of the unrounded h.
__global__ void moe_combine_kernel(const __half* __restrict__ yk, const float* __restrict__ wts,
                                   const int* __restrict__ ids, int e_lo, int e_hi, const __half* res, __half* out,
                                   float* __restrict__ out32, float* __restrict__ ss_out, int B, int D, int topk) {
  pdl_wait_trigger();
  const long i = ((long)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  const bool ok = i < (long)B * D;
  float sq = 0.0f;
  if (ok) {
    const int b = (int)(i / D), d = (int)(i - (long)b * D);
    float s4[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < topk; ++k) {
      const int e = ids[b * topk + k];
      if (e < e_lo || e >= e_hi) continue;
      const float wk = wts[b * topk + k];
      const __half* yr = yk + ((long)b * topk + k) * D + d;
#pragma unroll
      for (int j = 0; j < 4; ++j) s4[j] += wk * __half2float(yr[j]);
    }
    if (out32) {
#pragma unroll
      for (int j = 0; j < 4; ++j) out32[i + j] = s4[j];
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float v = __half2float(__float2half(s4[j]));
        if (res) v += __half2float(res[i + j]);
        sq += v * v;
        out[i + j] = __float2half(v);
      }
    }
  }
  sq += __shfl_xor_sync(0xffffffffu, sq, 1);
  sq += __shfl_xor_sync(0xffffffffu, sq, 2);
  if (ok && ss_out && !out32 && (threadIdx.x & 3) == 0) {
    const int b = (int)(i / D), d = (int)(i - (long)b * D);
    ss_out[(long)(d >> 4) * B + b] = sq;
  }
}

// h[b] = fp16(fp16(sum[b]) + res[b]) and the sums of squares, for the fp32
// sum of the expert-parallel partials (F16: sum already fp16, a GEMM output).
template <bool F16>
__global__ void residual_f32_kernel(const void* __restrict__ sumv, const __half* res, __half* out,
                                    float* __restrict__ ss_out, int B, int D) {
  pdl_wait_trigger();
  const long i = ((long)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  const bool ok = i < (long)B * D;
  float sq = 0.0f;
  if (ok) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float v = F16 ? __half2float(reinterpret_cast<const __half*>(sumv)[i + j])
                    : __half2float(__float2half(reinterpret_cast<const float*>(sumv)[i + j]));
      if (res) v += __half2float(res[i + j]);
      sq += v * v;
      out[i + j] = __float2half(v);
    }
  }
  sq += __shfl_xor_sync(0xffffffffu, sq, 1);
  sq += __shfl_xor_sync(0xffffffffu, sq, 2);
  if (ok && ss_out && (threadIdx.x & 3) == 0) {
    const int b = (int)(i / D), d = (int)(i - (long)b * D);
    ss_out[(long)(d >> 4) * B + b] = sq;
  }
}

}  // namespace
}  // namespace r4q

using namespace r4q;

typedef CUresult (*MoeEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Stacked expert nibbles [rows, row_bytes] as a 2-D byte tensor, box 128 bytes
// x 32 rows, 128-byte swizzle.
static int moe_weight_map(CUtensorMap* m, const void* base, long rows, long row_bytes) {
  static MoeEncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<MoeEncodeFn>(f);
  });
  if (!fn) return set_error(R4Q_ERR_CUDA, "moe_gemv: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {128, 32};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(R4Q_ERR_CUDA, "moe_gemv: tensor map encode failed (%d)", (int)r);
  return R4Q_OK;
}

static int pdl_status(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(R4Q_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  }
  return R4Q_OK;
}

extern "C" int r4q_moe_route(const void* logits, int B, int E, int topk, int e_lo, int e_hi, int* ids, float* wts,
                             int* counts, int* offsets, int* list, int* active, int* n_active, void* stream) {
  if (!logits || !ids || !wts || !counts || !offsets || !list || !active || !n_active || B < 1 || E < 1 ||
      E > 256 || topk < 1 || topk > 16 || topk > E || B * topk > 4096 || e_lo < 0 || e_hi > E || e_lo >= e_hi)
    return set_error(R4Q_ERR_ARG, "moe_route: bad arguments (B %d E %d topk %d)", B, E, topk);
  const size_t smem = (size_t)(3 * E + B * topk) * sizeof(int);
  return pdl_status(launch_pdl(moe_route_kernel, dim3(1), dim3(512), smem, (cudaStream_t)stream,
                               (const __half*)logits, B, E, topk, e_lo, e_hi, ids, wts, counts, offsets, list, active,
                               n_active), "moe_route_kernel");
}

extern "C" int r4q_moe_router(const void* x, const float* ss_in, int ss_parts, const void* norm_w, float eps,
                              void* xn, const void* router_w, void* logits, int B, int D, int E, int topk, int e_lo,
                              int e_hi, int* ids, float* wts, int* counts, int* offsets, int* list, int* active,
                              int* n_active, int* done, void* stream) {
  if (!xn || !router_w || !logits || !ids || !wts || !counts || !offsets || !list || !active || !n_active || !done ||
      B < 1 || D < 256 || D % 256 || D > 2048 || E < 1 || E > 256 || topk < 1 || topk > 16 || topk > E ||
      B * topk > 4096 || e_lo < 0 || e_hi > E || e_lo >= e_hi || (norm_w && (!x || !ss_in || ss_parts < 1)))
    return set_error(R4Q_ERR_ARG, "moe_router: bad arguments (B %d D %d E %d topk %d)", B, D, E, topk);
  if (!aligned(router_w, 16) || !aligned(xn, 16))
    return set_error(R4Q_ERR_ALIGN, "moe_router: router weights / xn not 16-byte aligned");
  const size_t smem_x = (size_t)kRouterTok * D * 2, smem_r = (size_t)(3 * E + B * topk) * sizeof(int);
  const size_t smem = smem_x > smem_r ? smem_x : smem_r;
  if (smem > 48 * 1024) {
    static std::atomic<size_t> set_to{0};
    if (set_to.load() < smem) {
      cudaFuncSetAttribute(moe_router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      set_to.store(smem);
    }
  }
  return pdl_status(launch_pdl(moe_router_kernel, dim3((E + 7) / 8, (B + kRouterTok - 1) / kRouterTok), dim3(256), smem, (cudaStream_t)stream,
                               (const __half*)x, ss_in, ss_parts, (const __half*)norm_w, eps, (__half*)xn,
                               (const __half*)router_w, (__half*)logits, B, D, E, topk, e_lo, e_hi, ids, wts, counts,
                               offsets, list, active, n_active, done),
                    "moe_router_kernel");
}

extern "C" int r4q_norm_fwht_rows(const void* x, const float* ss_in, int ss_parts, const void* w, float eps, void* y,
                                  int rows, int D, void* stream) {
  if (!x || !w || !y || rows < 1 || D < 32 || D % 32 || (ss_in && ss_parts < 1))
    return set_error(R4Q_ERR_ARG, "norm_fwht_rows: bad arguments");
  return pdl_status(launch_pdl(norm_fwht_kernel, dim3(rows), dim3(256), 0, (cudaStream_t)stream, (const __half*)x,
                               ss_in, ss_parts, (const __half*)w, eps, (__half*)y, D), "norm_fwht_kernel");
}

extern "C" int r4q_moe_gemv(int mode, const void* w, const void* sz, const void* x, long ldx, void* y, long ldy,
                            int N, int K, int E, int e_lo, int e_hi, int B, int topk, const int* counts,
                            const int* offsets, const int* list, const int* active, const int* n_active,
                            int* status, void* stream) {
  if (!w || !sz || !x || !y || !counts || !offsets || !list || !active || !n_active || N < 64 || N % 64 ||
      K < 128 || K % 128 || E < 1 || B < 1 || topk < 1 || mode < 0 || mode > 2 || e_lo < 0 || e_hi > E ||
      e_lo >= e_hi)
    return set_error(R4Q_ERR_ARG, "moe_gemv: bad arguments (mode %d N %d K %d; N %% 64, K %% 128)", mode, N, K);
  if (!aligned(w, 16) || !aligned(sz, 4) || !aligned(x, 16) || ldx % 8)
    return set_error(R4Q_ERR_ALIGN, "moe_gemv: weights / activations misaligned");
  MoeRoute rt{counts, offsets, list, active, n_active};
  const int el = e_hi - e_lo;
  const int slots = (el < B * topk) ? el : B * topk;
  cudaStream_t st = (cudaStream_t)stream;
  const uint8_t* wp = (const uint8_t*)w;
  const __half *sp = (const __half*)sz, *xp = (const __half*)x;
  // TMA tiles when the 64-row tile fits two or more CTAs per SM
  // (R4Q_MOE_LDG = 1 forces the register-staged kernel, measurement only)
  static const int force_ldg = [] {
    const char* v = getenv("R4Q_MOE_LDG");
    return v ? atoi(v) : 0;
  }();
  const size_t tma_smem = (size_t)32 * K + 1024;
  if (!force_ldg && K % 256 == 0 && tma_smem <= 100 * 1024) {
    CUtensorMap tm;
    int rc = moe_weight_map(&tm, w, (long)el * N, K / 2);
    if (rc) return rc;
    auto k = mode == 0 ? moe_gemv_tma_kernel<0> : mode == 1 ? moe_gemv_tma_kernel<1> : moe_gemv_tma_kernel<2>;
    static std::atomic<size_t> set_to[3];
    if (set_to[mode].load() < tma_smem) {
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tma_smem);
      set_to[mode].store(tma_smem);
    }
    return pdl_status(launch_pdl(k, dim3(N / 64, slots), dim3(kMoeThreads), tma_smem, st, tm, sp, xp, ldx, (__half*)y,
                                 ldy, N, K, topk, e_lo, rt, status),
                      "moe_gemv_tma_kernel");
  }
  // one CTA per (active-expert slot, tile); the kernel also runs as a
  // persistent grid (R4Q_MOE_GRID = CTA count, measurement only) — measured
  // on B200 the full grid is faster (B = 64: 101 us against 115 us for 296
  // persistent CTAs, gate_up of 127 experts)
  static const int forced = [] {
    const char* v = getenv("R4Q_MOE_GRID");
    return v ? atoi(v) : -1;
  }();
  const long items_max = (long)slots * (N / 64);
  long ctas = forced > 0 ? forced : items_max;
  if (ctas > items_max) ctas = items_max;
  dim3 grid((unsigned)ctas);
  auto k = mode == 0 ? moe_gemv_kernel<0> : mode == 1 ? moe_gemv_kernel<1> : moe_gemv_kernel<2>;
  return pdl_status(launch_pdl(k, grid, dim3(kMoeThreads), 0, st, wp, sp, xp, ldx, (__half*)y, ldy, N, K, topk, e_lo,
                               rt), "moe_gemv_kernel");
}

extern "C" int r4q_moe_combine(const void* yk, const float* wts, const int* ids, int e_lo, int e_hi, const void* res,
                               void* out, float* out32, float* ss_out, int B, int D, int topk, void* stream) {
  if (!yk || !wts || !ids || (!out && !out32) || B < 1 || D < 16 || D % 16 || topk < 1 || e_lo >= e_hi)
    return set_error(R4Q_ERR_ARG, "moe_combine: bad arguments");
  const long n4 = (long)B * D / 4;
  return pdl_status(launch_pdl(moe_combine_kernel, dim3((unsigned)((n4 + 255) / 256)), dim3(256), 0,
                               (cudaStream_t)stream, (const __half*)yk, wts, ids, e_lo, e_hi, (const __half*)res,
                               (__half*)out, out32, ss_out, B, D, topk), "moe_combine_kernel");
}

extern "C" int r4q_residual_f32(const float* sum, const void* res, void* out, float* ss_out, int B, int D,
                                void* stream) {
  if (!sum || !out || B < 1 || D < 16 || D % 16) return set_error(R4Q_ERR_ARG, "residual_f32: bad arguments");
  const long n4 = (long)B * D / 4;
  return pdl_status(launch_pdl(residual_f32_kernel<false>, dim3((unsigned)((n4 + 255) / 256)), dim3(256), 0,
                               (cudaStream_t)stream, (const void*)sum, (const __half*)res, (__half*)out, ss_out, B, D),
                    "residual_f32_kernel");
}

extern "C" int r4q_residual_f16(const void* a, const void* res, void* out, float* ss_out, int B, int D,
                                void* stream) {
  if (!a || !out || B < 1 || D < 16 || D % 16) return set_error(R4Q_ERR_ARG, "residual_f16: bad arguments");
  const long n4 = (long)B * D / 4;
  return pdl_status(launch_pdl(residual_f32_kernel<true>, dim3((unsigned)((n4 + 255) / 256)), dim3(256), 0,
                               (cudaStream_t)stream, a, (const __half*)res, (__half*)out, ss_out, B, D),
                    "residual_f16_kernel");
}
