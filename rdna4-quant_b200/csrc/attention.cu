// Split-K flash-decode GQA attention over the FP8 E4M3 KV cache.
//
// Replaces flash_decode_partial / flash_decode_reduce / flash_decode_fused
// (int4_decode_step.hip:1326-1593).  One query token per batch row; for every
// (batch row, kv head) the query heads of its GQA group attend over positions
// [0, seq_len) of the cache.
//
// B200 design:
//  * CTA = (K split, kv head, batch row), 4 warps; each warp streams its own
//    64-position K and V tiles (8 KB each) with TMA (128-byte swizzle) into a
//    2-slot ring and keeps an online softmax in registers;
//  * scores on the tensor cores: m16n8k16 with A = Q (GQA heads as rows, fp16,
//    held in registers for the whole CTA) and B = K (FP8 -> f16 with the
//    hardware pair conversion, which equals the reference decoder on every byte
//    the reference encoder emits); the head dimension is visited in a permuted
//    order (lane t owns d = 32t..32t+31) so each lane reads 32 contiguous bytes;
//  * the score accumulator layout is the A-fragment layout of P·V, so P stays
//    in registers; V's B fragment is assembled from four 16-byte rows with PRMT
//    and the pair conversion; O accumulates in fp32;
//  * Q stays in full precision (the reference packs Q to FP8 before Q·K,
//    :1349-1358; the parity target is fp32 softmax over the dequantised cache);
//  * warps merge through shared memory, K splits through an fp32 workspace:
//    the last CTA of a (row, kv head) merges the splits in split order
//    (log-sum-exp, :1416-1463), normalises, optionally applies the H32 FWHT per
//    32-element block of every head (:1448-1461) and writes fp16.
//  * optional per-(row, kv head) fp32 scales: scores use q·k·s_k, outputs o·s_v.
#include <cuda.h>

#include <mutex>

#include "r4q_common.cuh"

namespace r4q {

constexpr int kAttnWarps = 4;
constexpr int kAttnTile = 64;     // positions per tile
constexpr int kAttnD = 128;
constexpr int kAttnSlots = 2;
constexpr int kTileBytes = kAttnTile * kAttnD;          // 8 KB per K or V tile
constexpr long kAttnSpin = 1L << 26;

struct AttnParams {
  const __half* q;
  long ldq;
  const float* k_scale;
  const float* v_scale;
  __half* o;
  long ldo;
  int B, H, Hk, Hg, max_seq, seq_len;
  const long long* seq_dev;
  int nsplit, tps;                 // K splits per (row, kv head), tiles per split
  int fwht;
  float* part;                     // [B][Hk][nsplit][Hg][2 + 128]
  unsigned* cnt;                   // [B][Hk]
  int* status;
};

__device__ __forceinline__ uint32_t a_smem(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint4 a_lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ bool a_wait(uint64_t* bar, unsigned parity, int* status) {
  const uint32_t b = a_smem(bar);
  for (long i = 0; i < kAttnSpin; ++i) {
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                 " selp.u32 %0, 1, 0, p;\n}\n" : "=r"(ok) : "r"(b), "r"(parity) : "memory");
    if (ok) return true;
  }
  if (status) atomicExch(status, 1);
  return false;
}
__device__ __forceinline__ void a_issue(const CUtensorMap* tk, const CUtensorMap* tv, uint8_t* ks,
                                        uint8_t* vs, uint64_t* bar, int row) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a_smem(bar)),
               "r"(2 * kTileBytes) : "memory");
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(a_smem(ks)), "l"(reinterpret_cast<uint64_t>(tk)), "r"(0),
      "r"(row), "r"(a_smem(bar)) : "memory");
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(a_smem(vs)), "l"(reinterpret_cast<uint64_t>(tv)), "r"(0),
      "r"(row), "r"(a_smem(bar)) : "memory");
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  return h2_as_u32(__floats2half2_rn(lo, hi));
}

__global__ void __launch_bounds__(kAttnWarps * 32, 1)
    attn_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                const AttnParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  uint8_t* ring = smem + warp * (kAttnSlots * 2 * kTileBytes);     // [slot][K|V][8 KB]
  float* mbuf = reinterpret_cast<float*>(smem + kAttnWarps * kAttnSlots * 2 * kTileBytes);  // [warp][8][130]
  uint64_t* bars = reinterpret_cast<uint64_t*>(mbuf + kAttnWarps * 8 * 130);               // [warp][slot]
  __shared__ unsigned s_last;

  int seq = p.seq_dev ? (int)p.seq_dev[b] : p.seq_len;
  seq = max(0, min(seq, p.max_seq));
  const int T = (seq + kAttnTile - 1) / kAttnTile;
  const int t0 = split * p.tps, t1 = min(T, t0 + p.tps);
  const long row_base = ((long)b * p.Hk + kh) * p.max_seq;

  if (lane == 0) {
    for (int s = 0; s < kAttnSlots; ++s)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(a_smem(&bars[warp * kAttnSlots + s])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  if (lane == 0) {
    for (int i = 0; i < kAttnSlots; ++i) {
      const int tile = t0 + warp + kAttnWarps * i;
      if (tile < t1)
        a_issue(&tmk, &tmv, ring + i * 2 * kTileBytes, ring + i * 2 * kTileBytes + kTileBytes,
                &bars[warp * kAttnSlots + i], (int)(row_base + (long)tile * kAttnTile));
    }
  }

  // Q fragments: head g of the group, d = 32t + 4j + {0..3} for k-step j
  uint32_t qa[8], qb[8];
  const int head = kh * p.Hg + g;
  if (g < p.Hg) {
    const uint4* qp = reinterpret_cast<const uint4*>(p.q + (long)b * p.ldq + (long)head * kAttnD + 32 * t);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 v = qp[i];
      qa[2 * i] = v.x; qb[2 * i] = v.y; qa[2 * i + 1] = v.z; qb[2 * i + 1] = v.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) qa[j] = qb[j] = 0u;
  }
  const float ks = p.k_scale ? p.k_scale[b * p.Hk + kh] : 1.0f;
  const float qk_scale = ks * rsqrtf((float)kAttnD) * 1.4426950408889634f;  // log2 domain

  float m = -1e30f, l = 0.0f;
  float oacc[16][4];
#pragma unroll
  for (int jd = 0; jd < 16; ++jd)
#pragma unroll
    for (int i = 0; i < 4; ++i) oacc[jd][i] = 0.0f;

  bool ok = true;
  for (int i = 0;; ++i) {
    const int tile = t0 + warp + kAttnWarps * i;
    if (tile >= t1) break;
    const int slot = i & 1;
    if (ok) ok = a_wait(&bars[warp * kAttnSlots + slot], (unsigned)(i >> 1) & 1u, p.status);
    const uint32_t kb = a_smem(ring + slot * 2 * kTileBytes);
    const uint32_t vb = kb + kTileBytes;
    const int nvalid = min(kAttnTile, seq - tile * kAttnTile);

    // ---- S = Q K^T for 64 positions (8 n-tiles of 8) ----
    float sc[8][2];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int pr = nt * 8 + g;                       // position row of this lane's B column
      const uint4 k0 = a_lds128(kb + pr * 128 + (((2 * t) ^ (pr & 7)) << 4));
      const uint4 k1 = a_lds128(kb + pr * 128 + (((2 * t + 1) ^ (pr & 7)) << 4));
      const uint32_t kw[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
      float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t b01 = fp8x2_to_h2((uint16_t)(kw[j] & 0xFFFFu));
        const uint32_t b23 = fp8x2_to_h2((uint16_t)(kw[j] >> 16));
        mma16816(c, qa[j], 0u, qb[j], 0u, b01, b23);
      }
      const int p0 = nt * 8 + 2 * t;
      sc[nt][0] = p0 < nvalid ? c[0] * qk_scale : -INFINITY;
      sc[nt][1] = p0 + 1 < nvalid ? c[1] * qk_scale : -INFINITY;
    }
    // ---- online softmax for head g (rows are shared by the 4 lanes of a quad) ----
    float mx = -1e30f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) mx = fmaxf(mx, fmaxf(sc[nt][0], sc[nt][1]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mnew = fmaxf(m, mx);
    const float corr = exp2f(m - mnew);
    m = mnew;
    float psum = 0.0f;
    uint32_t pa[4], pb[4];                                 // P as A fragments for 4 k-steps
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const float e0 = exp2f(sc[2 * kk][0] - m), e1 = exp2f(sc[2 * kk][1] - m);
      const float e2 = exp2f(sc[2 * kk + 1][0] - m), e3 = exp2f(sc[2 * kk + 1][1] - m);
      psum += (e0 + e1) + (e2 + e3);
      pa[kk] = pack_h2(e0, e1);
      pb[kk] = pack_h2(e2, e3);
    }
    l = l * corr + psum;
#pragma unroll
    for (int jd = 0; jd < 16; ++jd) {
      oacc[jd][0] *= corr;
      oacc[jd][1] *= corr;
    }
    // ---- O += P V: k-step kk covers positions 16kk..16kk+15 ----
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int r0 = kk * 16 + 2 * t, r1 = r0 + 1, r2 = r0 + 8, r3 = r0 + 9;
      const uint4 v0 = a_lds128(vb + r0 * 128 + ((g ^ (r0 & 7)) << 4));
      const uint4 v1 = a_lds128(vb + r1 * 128 + ((g ^ (r1 & 7)) << 4));
      const uint4 v2 = a_lds128(vb + r2 * 128 + ((g ^ (r2 & 7)) << 4));
      const uint4 v3 = a_lds128(vb + r3 * 128 + ((g ^ (r3 & 7)) << 4));
      const uint32_t w0[4] = {v0.x, v0.y, v0.z, v0.w}, w1[4] = {v1.x, v1.y, v1.z, v1.w};
      const uint32_t w2[4] = {v2.x, v2.y, v2.z, v2.w}, w3[4] = {v3.x, v3.y, v3.z, v3.w};
#pragma unroll
      for (int wi = 0; wi < 4; ++wi) {
        // bytes k of rows (r0, r1) and (r2, r3) side by side: pairs for d-columns 4wi + k
        const uint32_t lo01 = prmt(w0[wi], w1[wi], 0x5140u), hi01 = prmt(w0[wi], w1[wi], 0x7362u);
        const uint32_t lo23 = prmt(w2[wi], w3[wi], 0x5140u), hi23 = prmt(w2[wi], w3[wi], 0x7362u);
        const uint32_t pr01[4] = {lo01 & 0xFFFFu, lo01 >> 16, hi01 & 0xFFFFu, hi01 >> 16};
        const uint32_t pr23[4] = {lo23 & 0xFFFFu, lo23 >> 16, hi23 & 0xFFFFu, hi23 >> 16};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int jd = 4 * wi + k;                   // d = 16 g + jd for this lane's column
          mma16816(oacc[jd], pa[kk], 0u, pb[kk], 0u, fp8x2_to_h2((uint16_t)pr01[k]),
                   fp8x2_to_h2((uint16_t)pr23[k]));
        }
      }
    }
    // slot reuse: this warp's generic reads precede the next async-proxy write
    __syncwarp();
    if (lane == 0) {
      const int nt2 = t0 + warp + kAttnWarps * (i + kAttnSlots);
      if (nt2 < t1) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        a_issue(&tmk, &tmv, ring + slot * 2 * kTileBytes, ring + slot * 2 * kTileBytes + kTileBytes,
                &bars[warp * kAttnSlots + slot], (int)(row_base + (long)nt2 * kAttnTile));
      }
    }
  }
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);

  // ---- merge the 4 warps: mbuf[warp][head][m, l, o[128]] ----
  if (g < p.Hg) {
    float* mb = mbuf + (warp * 8 + g) * 130;
    if (t == 0) {
      mb[0] = m;
      mb[1] = l;
    }
#pragma unroll
    for (int jd = 0; jd < 16; ++jd) {
      mb[2 + 16 * (2 * t) + jd] = oacc[jd][0];
      mb[2 + 16 * (2 * t + 1) + jd] = oacc[jd][1];
    }
  }
  __syncthreads();
  // thread -> (head, 4 d values): 8 heads x 32 lanes of 4 d = 128 threads x ... loop
  float* outp = p.part + ((((long)b * p.Hk + kh) * p.nsplit + split) * p.Hg) * 130;
  for (int idx = tid; idx < p.Hg * 32; idx += kAttnWarps * 32) {
    const int hg = idx >> 5, dl = idx & 31;
    float M = -1e30f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, mbuf[(w * 8 + hg) * 130]);
    float L = 0.0f, O[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float* mb = mbuf + (w * 8 + hg) * 130;
      const float f = exp2f(mb[0] - M);
      L += mb[1] * f;
#pragma unroll
      for (int i = 0; i < 4; ++i) O[i] += mb[2 + dl + 32 * i] * f;
    }
    float* op = outp + hg * 130;
    if (dl == 0) {
      op[0] = M;
      op[1] = L;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) op[2 + dl + 32 * i] = O[i];
  }
  // ---- the last CTA of (row, kv head) merges the splits in split order ----
  __syncthreads();
  if (tid == 0) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old)
                 : "l"(p.cnt + b * p.Hk + kh) : "memory");
    s_last = (old == (unsigned)p.nsplit - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (!s_last) return;
  const float vs = p.v_scale ? p.v_scale[b * p.Hk + kh] : 1.0f;
  const float* base = p.part + (((long)b * p.Hk + kh) * p.nsplit) * p.Hg * 130;
  for (int hg = warp; hg < p.Hg; hg += kAttnWarps) {
    float M = -1e30f;
    for (int s = 0; s < p.nsplit; ++s) M = fmaxf(M, __ldcg(base + ((long)s * p.Hg + hg) * 130));
    float L = 0.0f, O[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < p.nsplit; ++s) {
      const float* op = base + ((long)s * p.Hg + hg) * 130;
      const float f = exp2f(__ldcg(op) - M);
      L += __ldcg(op + 1) * f;
#pragma unroll
      for (int i = 0; i < 4; ++i) O[i] += __ldcg(op + 2 + lane + 32 * i) * f;
    }
    const float inv = L > 0.0f ? vs / L : 0.0f;
    __half* orow = p.o + (long)b * p.ldo + (long)(kh * p.Hg + hg) * kAttnD;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float v = O[i] * inv;
      if (p.fwht) v = fwht32_lane(v, lane);
      orow[lane + 32 * i] = __float2half(v);
    }
  }
  if (tid == 0) p.cnt[b * p.Hk + kh] = 0u;
}

typedef CUresult (*EncodeTiledFnA)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static int cache_map(CUtensorMap* m, const void* base, long rows) {
  static EncodeTiledFnA fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFnA>(f);
  });
  if (!fn) return set_error(R4Q_ERR_CUDA, "flash_decode: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)kAttnD, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)kAttnD};
  cuuint32_t box[2] = {(cuuint32_t)kAttnD, (cuuint32_t)kAttnTile};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(R4Q_ERR_CUDA, "flash_decode: tensor map encode failed (%d)", (int)r);
  return R4Q_OK;
}

static int attn_splits(int B, int Hk, int max_tiles) {
  const int nsm = num_sms();
  int ns = (nsm + B * Hk - 1) / (B * Hk);
  const int cap = (max_tiles + kAttnWarps - 1) / kAttnWarps;   // >= one tile per warp
  if (ns > cap) ns = cap;
  return ns < 1 ? 1 : ns;
}

// Fixed-size counter region (+ status word at its end): partials of an earlier
// call with other shapes never overlap the counters of a later one.
constexpr int kAttnMaxPairs = 16383;
static size_t attn_cnt_bytes(int B, int Hk) { (void)B; (void)Hk; return (size_t)(kAttnMaxPairs + 1) * 4; }

static size_t attn_ws_bytes(int B, int H, int Hk, int max_seq) {
  const int T = (max_seq + kAttnTile - 1) / kAttnTile;
  const int ns = attn_splits(B, Hk, T);
  return attn_cnt_bytes(B, Hk) + (size_t)B * H * ns * 130 * sizeof(float);
}

}  // namespace r4q

using namespace r4q;

extern "C" size_t r4q_flash_decode_workspace_bytes(int B, int H, int Hk, int max_seq) {
  if (B < 1 || H < 1 || Hk < 1 || max_seq < 1) return 0;
  return attn_ws_bytes(B, H, Hk, max_seq);
}

extern "C" int r4q_flash_decode(const void* q, long ldq, const void* k_cache, const void* v_cache,
                                const float* k_scale, const float* v_scale, void* o, long ldo,
                                int B, int H, int Hk, int D, int max_seq, int seq_len,
                                const long long* seq_dev, int flags, void* ws, size_t ws_bytes,
                                void* stream) {
  if (!q || !k_cache || !v_cache || !o) return set_error(R4Q_ERR_ARG, "flash_decode: null pointer");
  if (D != kAttnD) return set_error(R4Q_ERR_ARG, "flash_decode: head_dim %d (only 128)", D);
  if (B < 1 || Hk < 1 || H < Hk || H % Hk) return set_error(R4Q_ERR_ARG, "flash_decode: bad heads H=%d Hk=%d", H, Hk);
  if (H / Hk > 8) return set_error(R4Q_ERR_ARG, "flash_decode: GQA group %d > 8", H / Hk);
  if ((long)B * Hk > kAttnMaxPairs) return set_error(R4Q_ERR_ARG, "flash_decode: B*Hk above %d", kAttnMaxPairs);
  if (max_seq < 1 || (!seq_dev && (seq_len < 0 || seq_len > max_seq)))
    return set_error(R4Q_ERR_ARG, "flash_decode: seq_len %d outside [0, %d]", seq_len, max_seq);
  if (!aligned(q, 16) || (ldq % 8) || !aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(o, 2))
    return set_error(R4Q_ERR_ALIGN, "flash_decode: q/caches must be 16-byte aligned");
  const size_t need = attn_ws_bytes(B, H, Hk, max_seq);
  if (!ws || ws_bytes < need)
    return set_error(R4Q_ERR_CAPACITY, "flash_decode: workspace %zu < %zu bytes", ws_bytes, need);
  const long rows = (long)B * Hk * max_seq;
  CUtensorMap tmk, tmv;
  int st = cache_map(&tmk, k_cache, rows);
  if (!st) st = cache_map(&tmv, v_cache, rows);
  if (st) return st;
  const int Tmax = ((seq_dev ? max_seq : seq_len) + kAttnTile - 1) / kAttnTile;
  AttnParams p;
  p.q = (const __half*)q; p.ldq = ldq;
  p.k_scale = k_scale; p.v_scale = v_scale;
  p.o = (__half*)o; p.ldo = ldo;
  p.B = B; p.H = H; p.Hk = Hk; p.Hg = H / Hk; p.max_seq = max_seq; p.seq_len = seq_len;
  p.seq_dev = seq_dev;
  p.nsplit = attn_splits(B, Hk, (max_seq + kAttnTile - 1) / kAttnTile);
  const int Tsplit = Tmax > 0 ? Tmax : 1;
  p.tps = (Tsplit + p.nsplit - 1) / p.nsplit;
  if (!seq_dev) {
    // fewer splits for a short context (same workspace layout, smaller count)
    p.nsplit = attn_splits(B, Hk, Tsplit);
    p.tps = (Tsplit + p.nsplit - 1) / p.nsplit;
  }
  p.fwht = (flags & R4Q_ATTN_FWHT) ? 1 : 0;
  p.cnt = (unsigned*)ws;
  p.status = (int*)((uint8_t*)ws + attn_cnt_bytes(B, Hk) - 4);
  p.part = (float*)((uint8_t*)ws + attn_cnt_bytes(B, Hk));
  const size_t smem = 1024 + (size_t)kAttnWarps * kAttnSlots * 2 * kTileBytes +
                      (size_t)kAttnWarps * 8 * 130 * 4 + kAttnWarps * kAttnSlots * 8;
  static std::once_flag attr_once;
  std::call_once(attr_once, [smem] {
    cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaGetLastError();
  });
  dim3 grid(p.nsplit, Hk, B);
  attn_kernel<<<grid, kAttnWarps * 32, smem, (cudaStream_t)stream>>>(tmk, tmv, p);
  return check_launch("attn_kernel");
}
