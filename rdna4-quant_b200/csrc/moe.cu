// Mixture-of-experts decode FFN (Qwen3-30B-A3B shape: 128
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
//    counting sort in one CTA — and the ascending list of active experts;
//  * moe_gemv_kernel: grouped dequant-GEMV.  CTA = (64-row tile, active-expert
//    slot); a fixed grid (so it can live in a CUDA graph) whose CTAs past the
//    active count exit.  The CTA stages the activations of its expert's
//    tokens (16 at a time) in shared memory — for down_proj with the
//    SiLU(gate)·up + FWHT prologue applied — and 8 warps (4 m-tiles x 2 K
//    halves) stream the expert's weights with 128-bit loads, dequantise in
//    registers and accumulate on the tensor cores (m16n8k16, tokens as N);
//  * moe_combine_kernel: h = fp16(fp16(Σ_k w_k fp16(y_k)) + residual) in slot
//    order, with the per-16-row sums of squares the next RMSNorm prologue takes.
#include "r4q_common.cuh"

namespace r4q {
namespace {

constexpr int kMoeTile = 64;
constexpr int kMoeTokChunk = 16;        // tokens staged per pass (2 n-groups of 8)
constexpr int kMoeThreads = 512;       // 16 warps: 4 m-tiles x 4 K quarters
constexpr int kMoeKq = 4;
constexpr int kMoeBatch = 4;            // 32-k blocks whose loads are in flight together

struct MoeRoute {
  const int* counts;      // [E]
  const int* offsets;     // [E + 1]
  const int* list;        // [B * topk] entries t * topk + k grouped by expert
  const int* active;      // [E] active experts, ascending
  const int* n_active;    // [1]
};

// ---------------------------------------------------------------- routing
__global__ void moe_route_kernel(const __half* __restrict__ logits, int B, int E, int topk, int e_lo, int e_hi,
                                 int* ids, float* wts, int* counts, int* offsets, int* list, int* active,
                                 int* n_active) {
  extern __shared__ int sm[];
  int* s_cnt = sm;                  // [E]
  int* s_ids = sm + E;              // [B * topk]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
  for (int e = tid; e < E; e += blockDim.x) s_cnt[e] = 0;
  // one warp per token: softmax, then top-k by repeated arg-max
  for (int b = warp; b < B; b += nw) {
    const __half* lr = logits + (long)b * E;
    float mx = -INFINITY;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, __half2float(lr[e]));
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
    for (int e = lane; e < E; e += 32) sum += expf(__half2float(lr[e]) - mx);
    sum = warp_sum(sum);
    unsigned long long taken[4] = {0, 0, 0, 0};      // E <= 256
    float psel = 0.0f;
    float pk[16];
    int ik[16];
    for (int k = 0; k < topk; ++k) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int e = lane; e < E; e += 32) {
        if ((taken[e >> 6] >> (e & 63)) & 1ull) continue;
        const float v = __half2float(lr[e]);
        if (v > bv || (v == bv && e < bi)) {
          bv = v;
          bi = e;
        }
      }
      for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      taken[bi >> 6] |= 1ull << (bi & 63);
      const float p = expf(bv - mx) / sum;
      pk[k] = p;
      ik[k] = bi;
      psel += p;
    }
    if (lane == 0)
      for (int k = 0; k < topk; ++k) {
        ids[b * topk + k] = ik[k];
        wts[b * topk + k] = pk[k] / psel;
        s_ids[b * topk + k] = ik[k];
        atomicAdd(&s_cnt[ik[k]], 1);
      }
  }
  __syncthreads();
  if (tid == 0) {
    int off = 0, na = 0;
    for (int e = 0; e < E; ++e) {
      offsets[e] = off;
      counts[e] = s_cnt[e];
      if (s_cnt[e] && e >= e_lo && e < e_hi) active[na++] = e;
      off += s_cnt[e];
    }
    offsets[E] = off;
    *n_active = na;
  }
  __syncthreads();
  // stable placement: entry j goes after the earlier entries of its expert
  for (int j = tid; j < B * topk; j += blockDim.x) {
    const int e = s_ids[j];
    int before = 0;
    for (int i = 0; i < j; ++i) before += (s_ids[i] == e);
    list[offsets[e] + before] = j;
  }
}

// ------------------------------------------------- row RMSNorm + H32 FWHT
// y = fp16(H32(fp16... x * rrms * w)) per 32-block: the RMSNorm+FWHT prologue
// of the dense GEMVs as a standalone pass (rrms from ss_in partials or x).
__global__ void norm_fwht_kernel(const __half* __restrict__ x, const float* __restrict__ ss_in, int parts,
                                 const __half* __restrict__ w, float eps, __half* __restrict__ y, int D) {
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
  for (int blk = warp; blk < D / 32; blk += nw) {
    const int i = blk * 32 + lane;
    const float v = __half2float(xr[i]) * rr * __half2float(w[i]);
    y[(long)b * D + i] = __float2half(fwht32_lane(v, lane));
  }
}

// ------------------------------------------------------ grouped expert GEMV
// MODE 0 (gate_up): activation of entry j is xin[j / topk] (rows of K).
// MODE 1 (down): activation of entry j is fp16(FWHT(silu(g) * u)), g, u =
// halves of xin[j] (rows of 2K), one rounding (silu_hadamard_ds, :1031-1051).
template <int MODE>
__global__ void __launch_bounds__(kMoeThreads)
    moe_gemv_kernel(const uint8_t* __restrict__ w, const __half* __restrict__ sz, const __half* __restrict__ xin,
                    long ldx, __half* __restrict__ y, long ldy, int N, int K, int topk, int e_lo,
                    const MoeRoute rt) {
  const int a = blockIdx.y;
  if (a >= *rt.n_active) return;
  const int e = rt.active[a];
  const int cnt = rt.counts[e];
  const int* ent = rt.list + rt.offsets[e];
  const int row0 = blockIdx.x * kMoeTile;
  extern __shared__ __align__(16) uint8_t smem[];
  __half* xs = reinterpret_cast<__half*>(smem);                           // [16][K + 8]
  float* red = reinterpret_cast<float*>(xs + kMoeTokChunk * (K + 8));     // [3 quarters][4][2 ng][4][32]
  const int ldxs = K + 8;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int mt = warp & 3, kh = warp >> 2;                // m-tile, K quarter
  const int nblk = K / 32;
  const int b0 = (nblk * kh) / kMoeKq, b1 = (nblk * (kh + 1)) / kMoeKq;
  const long wrow = (long)K / 2, srow = (long)K / 16;
  const int ra = row0 + mt * 16 + g, rb = ra + 8;
  const long el = e - e_lo;                              // this GPU's expert slice starts at e_lo
  const uint8_t* wa = w + (el * N + ra) * wrow;
  const uint8_t* wb = w + (el * N + rb) * wrow;
  const __half* sa = sz + (el * N + ra) * srow;
  const __half* sb = sz + (el * N + rb) * srow;

  for (int c0 = 0; c0 < cnt; c0 += kMoeTokChunk) {
    const int nc = min(kMoeTokChunk, cnt - c0);
    __syncthreads();
    // ---- stage the activations of tokens c0 .. c0 + nc (zeros past nc)
    if (MODE == 0) {
      for (int i = tid; i < kMoeTokChunk * (K / 8); i += kMoeThreads) {
        const int r = i / (K / 8), c8 = i - r * (K / 8);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < nc) v = *reinterpret_cast<const uint4*>(xin + (long)(ent[c0 + r] / topk) * ldx + c8 * 8);
        *reinterpret_cast<uint4*>(xs + r * ldxs + c8 * 8) = v;
      }
    } else {
      // one warp per (token, 32-block): silu(g) * u -> fp16 -> H32 -> fp16
      for (int i = warp; i < kMoeTokChunk * nblk; i += kMoeThreads / 32) {
        const int r = i / nblk, blk = i - r * nblk;
        float v = 0.0f;
        if (r < nc) {
          const __half* xr = xin + (long)ent[c0 + r] * ldx;
          const float gg = __half2float(xr[blk * 32 + lane]);
          const float uu = __half2float(xr[K + blk * 32 + lane]);
          v = fwht32_lane(gg / (1.0f + expf(-gg)) * uu, lane);
        }
        xs[r * ldxs + blk * 32 + lane] = __float2half(v);
      }
    }
    __syncthreads();
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    const bool live = ra < N;
    if (live) {
      for (int bb = b0; bb < b1; bb += kMoeBatch) {
        uint4 qa[kMoeBatch], qb[kMoeBatch];
        __half2 pa[kMoeBatch], pb[kMoeBatch];
#pragma unroll
        for (int u = 0; u < kMoeBatch; ++u) {       // every load of the batch first
          const int blk = min(bb + u, b1 - 1);
          qa[u] = __ldg(reinterpret_cast<const uint4*>(wa + blk * 16));
          qb[u] = __ldg(reinterpret_cast<const uint4*>(wb + blk * 16));
          pa[u] = __ldg(reinterpret_cast<const __half2*>(sa + blk * 2));
          pb[u] = __ldg(reinterpret_cast<const __half2*>(sb + blk * 2));
        }
#pragma unroll
        for (int u = 0; u < kMoeBatch; ++u) {
          const int blk = bb + u;
          if (blk >= b1) break;
          const uint32_t wa4[4] = {qa[u].x, qa[u].y, qa[u].z, qa[u].w}, wb4[4] = {qb[u].x, qb[u].y, qb[u].z, qb[u].w};
          // this lane's bytes t, t + 4, t + 8, t + 12 of each row: k pairs
          // (2t, 2t+1), (2t+8, 2t+9), (16+2t, ..), (24+2t, ..)
          uint32_t fa[4], fb[4];
          const __half2 s2a = __half2half2(__low2half(pa[u])),
                        z2a = __hadd2(__half2half2(__high2half(pa[u])), __float2half2_rn(1024.0f));
          const __half2 s2b = __half2half2(__low2half(pb[u])),
                        z2b = __hadd2(__half2half2(__high2half(pb[u])), __float2half2_rn(1024.0f));
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t byte_a = (wa4[q] >> (8 * t)) & 0xFFu;   // byte 4q + t
            const uint32_t byte_b = (wb4[q] >> (8 * t)) & 0xFFu;
            const uint32_t ha = (byte_a & 0xFu) | ((byte_a >> 4) << 16);
            const uint32_t hb = (byte_b & 0xFu) | ((byte_b >> 4) << 16);
            fa[q] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(ha | 0x64006400u), z2a), s2a));
            fb[q] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(hb | 0x64006400u), z2b), s2b));
          }
          const int kb = blk * 32;
#pragma unroll
          for (int ks = 0; ks < 2; ++ks) {
            const uint32_t a0 = fa[2 * ks], a1 = fb[2 * ks], a2 = fa[2 * ks + 1], a3 = fb[2 * ks + 1];
#pragma unroll
            for (int ng = 0; ng < 2; ++ng) {
              const __half* xr = xs + (ng * 8 + g) * ldxs + kb + ks * 16 + 2 * t;
              const uint32_t bb0 = *reinterpret_cast<const uint32_t*>(xr);
              const uint32_t bb1 = *reinterpret_cast<const uint32_t*>(xr + 8);
              mma16816(acc[ng], a0, a1, a2, a3, bb0, bb1);
            }
          }
        }
      }
    }
    // ---- the K quarters meet in shared memory (fixed order); quarter 0 writes
    if (kh != 0) {
#pragma unroll
      for (int ng = 0; ng < 2; ++ng)
#pragma unroll
        for (int i = 0; i < 4; ++i) red[((((kh - 1) * 4 + mt) * 2 + ng) * 4 + i) * 32 + lane] = acc[ng][i];
    }
    __syncthreads();
    if (kh == 0 && live) {
#pragma unroll
      for (int ng = 0; ng < 2; ++ng) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int q = 0; q < kMoeKq - 1; ++q) acc[ng][i] += red[(((q * 4 + mt) * 2 + ng) * 4 + i) * 32 + lane];
        // C: (row g, tokens 2t, 2t+1), (row g + 8, tokens 2t, 2t+1)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int tok = ng * 8 + 2 * t + h;
          if (tok < nc) {
            __half* yr = y + (long)ent[c0 + tok] * ldy;
            yr[ra] = __float2half(acc[ng][h]);
            if (rb < N) yr[rb] = __float2half(acc[ng][2 + h]);
          }
        }
      }
    }
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

extern "C" int r4q_moe_route(const void* logits, int B, int E, int topk, int e_lo, int e_hi, int* ids, float* wts,
                             int* counts, int* offsets, int* list, int* active, int* n_active, void* stream) {
  if (!logits || !ids || !wts || !counts || !offsets || !list || !active || !n_active || B < 1 || E < 1 ||
      E > 256 || topk < 1 || topk > 16 || topk > E || B * topk > 4096 || e_lo < 0 || e_hi > E || e_lo >= e_hi)
    return set_error(R4Q_ERR_ARG, "moe_route: bad arguments (B %d E %d topk %d)", B, E, topk);
  const size_t smem = (size_t)(E + B * topk) * sizeof(int);
  moe_route_kernel<<<1, 512, smem, (cudaStream_t)stream>>>((const __half*)logits, B, E, topk, e_lo, e_hi, ids, wts,
                                                          counts, offsets, list, active, n_active);
  return check_launch("moe_route_kernel");
}

extern "C" int r4q_norm_fwht_rows(const void* x, const float* ss_in, int ss_parts, const void* w, float eps, void* y,
                                  int rows, int D, void* stream) {
  if (!x || !w || !y || rows < 1 || D < 32 || D % 32 || (ss_in && ss_parts < 1))
    return set_error(R4Q_ERR_ARG, "norm_fwht_rows: bad arguments");
  norm_fwht_kernel<<<rows, 256, 0, (cudaStream_t)stream>>>((const __half*)x, ss_in, ss_parts, (const __half*)w, eps,
                                                           (__half*)y, D);
  return check_launch("norm_fwht_kernel");
}

extern "C" int r4q_moe_gemv(int mode, const void* w, const void* sz, const void* x, long ldx, void* y, long ldy,
                            int N, int K, int E, int e_lo, int e_hi, int B, int topk, const int* counts,
                            const int* offsets, const int* list, const int* active, const int* n_active,
                            void* stream) {
  if (!w || !sz || !x || !y || !counts || !offsets || !list || !active || !n_active || N < 16 || N % 16 ||
      K < 32 || K % 32 || E < 1 || B < 1 || topk < 1 || (mode != 0 && mode != 1) || e_lo < 0 || e_hi > E ||
      e_lo >= e_hi)
    return set_error(R4Q_ERR_ARG, "moe_gemv: bad arguments (N %d K %d)", N, K);
  if (!aligned(w, 16) || !aligned(sz, 4) || !aligned(x, 16) || ldx % 8)
    return set_error(R4Q_ERR_ALIGN, "moe_gemv: weights / activations misaligned");
  MoeRoute rt{counts, offsets, list, active, n_active};
  const size_t smem = (size_t)kMoeTokChunk * (K + 8) * 2 + (kMoeKq - 1) * 4 * 2 * 4 * 32 * 4;
  const int el = e_hi - e_lo;
  const int slots = (el < B * topk) ? el : B * topk;
  dim3 grid((N + kMoeTile - 1) / kMoeTile, slots);
  cudaStream_t st = (cudaStream_t)stream;
  if (mode == 0) {
    if (smem > 48 * 1024) cudaFuncSetAttribute(moe_gemv_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    moe_gemv_kernel<0><<<grid, kMoeThreads, smem, st>>>((const uint8_t*)w, (const __half*)sz, (const __half*)x, ldx,
                                                        (__half*)y, ldy, N, K, topk, e_lo, rt);
  } else {
    if (smem > 48 * 1024) cudaFuncSetAttribute(moe_gemv_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    moe_gemv_kernel<1><<<grid, kMoeThreads, smem, st>>>((const uint8_t*)w, (const __half*)sz, (const __half*)x, ldx,
                                                        (__half*)y, ldy, N, K, topk, e_lo, rt);
  }
  return check_launch("moe_gemv_kernel");
}

extern "C" int r4q_moe_combine(const void* yk, const float* wts, const int* ids, int e_lo, int e_hi, const void* res,
                               void* out, float* out32, float* ss_out, int B, int D, int topk, void* stream) {
  if (!yk || !wts || !ids || (!out && !out32) || B < 1 || D < 16 || D % 16 || topk < 1 || e_lo >= e_hi)
    return set_error(R4Q_ERR_ARG, "moe_combine: bad arguments");
  const long n4 = (long)B * D / 4;
  moe_combine_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      (const __half*)yk, wts, ids, e_lo, e_hi, (const __half*)res, (__half*)out, out32, ss_out, B, D, topk);
  return check_launch("moe_combine_kernel");
}

extern "C" int r4q_residual_f32(const float* sum, const void* res, void* out, float* ss_out, int B, int D,
                                void* stream) {
  if (!sum || !out || B < 1 || D < 16 || D % 16) return set_error(R4Q_ERR_ARG, "residual_f32: bad arguments");
  const long n4 = (long)B * D / 4;
  residual_f32_kernel<false><<<(unsigned)((n4 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      sum, (const __half*)res, (__half*)out, ss_out, B, D);
  return check_launch("residual_f32_kernel");
}

extern "C" int r4q_residual_f16(const void* a, const void* res, void* out, float* ss_out, int B, int D,
                                void* stream) {
  if (!a || !out || B < 1 || D < 16 || D % 16) return set_error(R4Q_ERR_ARG, "residual_f16: bad arguments");
  const long n4 = (long)B * D / 4;
  residual_f32_kernel<true><<<(unsigned)((n4 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      a, (const __half*)res, (__half*)out, ss_out, B, D);
  return check_launch("residual_f16_kernel");
}
