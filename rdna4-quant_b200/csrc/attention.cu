// Split-K flash-decode GQA attention over the FP8 E4M3 KV cache, optionally
// fused with the per-head QK-RMSNorm + RoPE + FP8 KV write of the new token.
//
// Replaces flash_decode_partial / flash_decode_reduce / flash_decode_fused
// (int4_decode_step.hip:1326-1593) and, fused, head_rmsnorm_rope_kv
// (:1620-1683).  One query token per batch row; for every (batch row, kv
// head) the query heads of its GQA group attend over positions [0, seq_len).
//
// B200 design:
//  * one thread-block cluster of C CTAs (1, 2, 4 or 8: see attn_cluster) per (kv head, batch row),
//    4 warps per CTA; the cluster's 4C warps take consecutive 64-position tiles
//    round-robin, each streaming its K and V tiles (8 KB each) with TMA
//    (128-byte swizzle) into a 2-slot ring and keeping an online softmax in
//    registers;
//  * programmatic dependent launch: inside the decode step the K/V tiles are
//    requested before griddepcontrol.wait — the cache rows before the new
//    position are final long before this kernel; the new token's row is
//    patched into shared memory (fused) or its tile requested after the wait;
//  * fused head ops: each CTA normalises + rotates the query heads of its group
//    (fp32, one fp16 rounding: the head_rmsnorm_rope_kv arithmetic); the warp
//    that owns the newest tile also normalises + rotates K, encodes K and V
//    with the reference FP8 encoder (optionally divided by the per-head scale),
//    writes them to the cache and into its shared-memory tile;
//  * scores on the tensor cores: m16n8k16 with A = Q (GQA heads as rows, fp16)
//    and B = K (FP8 -> f16 with the hardware pair conversion, which equals the
//    reference decoder on every byte the reference encoder emits); the head
//    dimension is visited in a permuted order (lane t owns d = 32t..32t+31) so
//    each lane reads 32 contiguous bytes;
//  * the score accumulator layout is the A-fragment layout of P·V, so P stays
//    in registers; V's B fragment is assembled from four 16-byte rows with PRMT
//    and the pair conversion; O accumulates in fp32;
//  * Q stays in full precision (the reference packs Q to FP8 before Q·K,
//    :1349-1358; the parity target is fp32 softmax over the dequantised cache);
//  * warps merge through shared memory, the cluster's CTAs through distributed
//    shared memory: CTA 0 reads every CTA's (max, sum, O) in rank order
//    (log-sum-exp, :1416-1463), normalises, optionally applies the H32 FWHT per
//    32-element block of every head (:1448-1461) and writes fp16.  No global
//    workspace beyond a status word, no atomics.
//  * optional per-(row, kv head) fp32 scales: scores use q·k·s_k, outputs o·s_v.
#include <cuda.h>

#include <cstdlib>
#include <mutex>

#include "attention.cuh"
#include "r4q_common.cuh"

namespace r4q {

constexpr int kAttnWarps = 4;
constexpr int kAttnTile = 64;     // positions per tile
constexpr int kAttnD = 128;
constexpr int kAttnSlots = 2;
constexpr int kTileBytes = kAttnTile * kAttnD;          // 8 KB per K or V tile
constexpr long kAttnSpin = 1L << 26;

struct AttnParams {
  const __half* q;                 // [B][ldq]: raw q (fused) or normalised q
  long ldq;
  // fused head ops (k_new null: q is already normalised, the cache complete)
  const __half *k_new, *v_new;     // raw k / v of the new token, row stride ldq
  const __half *qw, *kw;           // per-head norm weights [128]
  const __half *cos_tab, *sin_tab; // RoPE tables [rows][64]
  long tab_stride;
  float eps;
  uint8_t *kc, *vc;                // caches (for the new token's write)
  const float* k_scale;
  const float* v_scale;
  __half* o;
  long ldo;
  int B, H, Hk, Hg, max_seq, seq_len;
  const long long* seq_dev;
  int fwht;
  int early;                       // seq_dev and the cache rows before the newest are final before
                                   // the previous kernel ends: request tiles before griddepcontrol.wait
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

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_cluster_f32(const float* p, uint32_t rank) {
  uint32_t a = a_smem(p), ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
  return v;
}

// Per-head RMSNorm + RoPE of one 128-element head held 4 per lane (element
// l + 32 j), the head_kernel arithmetic: fp32 throughout, fp16 tables.
__device__ __forceinline__ void head_norm_rope4(float (&v)[4], const __half* w, const __half* cr,
                                                const __half* sr, float eps, int lane) {
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) ss += v[j] * v[j];
  ss = warp_sum(ss);
  const float rrms = rsqrtf(ss / (float)kAttnD + eps);
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = v[j] * rrms * __half2float(w[lane + 32 * j]);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int i = lane + 32 * j;
    const float c = __half2float(cr[i]), s = __half2float(sr[i]);
    const float e = v[j], o = v[j + 2];
    v[j] = e * c - o * s;
    v[j + 2] = o * c + e * s;
  }
}

__device__ __forceinline__ void issue_first(const CUtensorMap* tmk, const CUtensorMap* tmv, uint8_t* ring,
                                            uint64_t* bars, int wg, int W, int T, long row_base, bool skip_last,
                                            bool (&issued)[kAttnSlots]) {
  for (int i = 0; i < kAttnSlots; ++i) {
    const int tile = wg + W * i;
    if (tile < T && !issued[i] && !(skip_last && tile == T - 1)) {
      a_issue(tmk, tmv, ring + i * 2 * kTileBytes, ring + i * 2 * kTileBytes + kTileBytes, &bars[i],
              (int)(row_base + (long)tile * kAttnTile));
      issued[i] = true;
    }
  }
}

__global__ void __launch_bounds__(kAttnWarps * 32, 1)
    attn_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                const AttnParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int kh = blockIdx.y, b = blockIdx.z;
  const int C = gridDim.x;                                  // CTAs per cluster = per (row, kv head)
  const int rank = (int)cluster_rank();
  uint8_t* ring = smem + warp * (kAttnSlots * 2 * kTileBytes);     // [slot][K|V][8 KB]
  float* mbuf = reinterpret_cast<float*>(smem + kAttnWarps * kAttnSlots * 2 * kTileBytes);  // [warp][8][130]
  float* cpart = mbuf + kAttnWarps * 8 * 130;                                              // [8][130]
  __half* qs = reinterpret_cast<__half*>(cpart + 8 * 130);                                 // [8][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(qs + 8 * kAttnD);                           // [warp][slot]
  uint64_t* wbars = bars + warp * kAttnSlots;
  const bool fused = p.k_new != nullptr;

  if (lane == 0) {
    for (int s = 0; s < kAttnSlots; ++s)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(a_smem(&wbars[s])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  if (!p.early) asm volatile("griddepcontrol.wait;" ::: "memory");
  int seq = p.seq_dev ? (int)p.seq_dev[b] : p.seq_len;
  seq = max(0, min(seq, p.max_seq));
  const int T = (seq + kAttnTile - 1) / kAttnTile;
  const int pos = seq - 1;                                  // the newest position
  const long row_base = ((long)b * p.Hk + kh) * p.max_seq;
  const int W = C * kAttnWarps;
  const int wg = rank * kAttnWarps + warp;                  // this warp's place in the cluster
  const bool owner = fused && T > 0 && wg == (T - 1) % W;   // holds the newest tile

  // tiles of earlier positions go out before the previous kernel ends (early);
  // the newest tile too when its row is patched in shared memory (fused)
  bool issued[kAttnSlots] = {false, false};
  if (lane == 0) issue_first(&tmk, &tmv, ring, wbars, wg, W, T, row_base, p.early && !fused, issued);
  if (p.early) asm volatile("griddepcontrol.wait;" ::: "memory");
  if (lane == 0) issue_first(&tmk, &tmv, ring, wbars, wg, W, T, row_base, false, issued);
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // ---- queries of the group: normalised + rotated here (fused) or as given
  for (int hg = warp; hg < p.Hg; hg += kAttnWarps) {
    const __half* src = p.q + (long)b * p.ldq + (long)(kh * p.Hg + hg) * kAttnD;
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = __half2float(src[lane + 32 * j]);
    if (fused && pos >= 0)
      head_norm_rope4(v, p.qw, p.cos_tab + (long)pos * p.tab_stride, p.sin_tab + (long)pos * p.tab_stride,
                      p.eps, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) qs[hg * kAttnD + lane + 32 * j] = __float2half(v[j]);
  }
  // ---- the newest K / V: normalise + rotate K, encode, write the cache row
  uint32_t knew = 0, vnew = 0;                             // 4 FP8 bytes (d = lane + 32 j)
  if (owner) {
    const __half* ksrc = p.k_new + (long)b * p.ldq + (long)kh * kAttnD;
    const __half* vsrc = p.v_new + (long)b * p.ldq + (long)kh * kAttnD;
    float kv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) kv[j] = __half2float(ksrc[lane + 32 * j]);
    head_norm_rope4(kv, p.kw, p.cos_tab + (long)pos * p.tab_stride, p.sin_tab + (long)pos * p.tab_stride,
                    p.eps, lane);
    const float ksc = p.k_scale ? p.k_scale[b * p.Hk + kh] : 1.0f;
    const float vsc = p.v_scale ? p.v_scale[b * p.Hk + kh] : 1.0f;
    uint8_t* kd = p.kc + (row_base + pos) * kAttnD;
    uint8_t* vd = p.vc + (row_base + pos) * kAttnD;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float kf = kv[j];
      const uint32_t kb = fp8_encode(p.k_scale ? kf / ksc : kf);
      const float vv = __half2float(vsrc[lane + 32 * j]);
      const uint32_t vb = fp8_encode(p.v_scale ? vv / vsc : vv);
      kd[lane + 32 * j] = (uint8_t)kb;
      vd[lane + 32 * j] = (uint8_t)vb;
      knew |= kb << (8 * j);
      vnew |= vb << (8 * j);
    }
  }
  __syncthreads();

  // Q fragments: head g of the group, d = 32t + 4j + {0..3} for k-step j
  uint32_t qa[8], qb[8];
  if (g < p.Hg) {
    const uint4* qp = reinterpret_cast<const uint4*>(qs + g * kAttnD + 32 * t);
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
    const int tile = wg + W * i;
    if (tile >= T) break;
    const int slot = i & 1;
    if (ok) ok = a_wait(&wbars[slot], (unsigned)(i >> 1) & 1u, p.status);
    const uint32_t kb = a_smem(ring + slot * 2 * kTileBytes);
    const uint32_t vb = kb + kTileBytes;
    const int nvalid = min(kAttnTile, seq - tile * kAttnTile);
    if (owner && tile == T - 1) {
      // the newest row into the swizzled tiles: byte d of row r sits at
      // r * 128 + ((d >> 4) ^ (r & 7)) * 16 + (d & 15)
      const int r = pos - tile * kAttnTile;
      uint8_t* kt = ring + slot * 2 * kTileBytes;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int d = lane + 32 * j;
        const int off = r * 128 + (((d >> 4) ^ (r & 7)) << 4) + (d & 15);
        kt[off] = (uint8_t)(knew >> (8 * j));
        kt[kTileBytes + off] = (uint8_t)(vnew >> (8 * j));
      }
      __syncwarp();
    }

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
    // slot reuse: this warp's generic reads (and the patched row) precede the
    // next async-proxy write
    __syncwarp();
    if (lane == 0) {
      const int nt2 = wg + W * (i + kAttnSlots);
      if (nt2 < T) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        a_issue(&tmk, &tmv, ring + slot * 2 * kTileBytes, ring + slot * 2 * kTileBytes + kTileBytes,
                &wbars[slot], (int)(row_base + (long)nt2 * kAttnTile));
      }
    }
  }
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);

  // ---- merge the 4 warps: mbuf[warp][head][m, l, o[128]] -> cpart[head] ----
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
    float* op = cpart + hg * 130;
    if (dl == 0) {
      op[0] = M;
      op[1] = L;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) op[2 + dl + 32 * i] = O[i];
  }
  // ---- CTA 0 of the cluster merges every CTA's partial in rank order ----
  cluster_sync_all();
  if (rank == 0) {
    const float vs = p.v_scale ? p.v_scale[b * p.Hk + kh] : 1.0f;
    for (int hg = warp; hg < p.Hg; hg += kAttnWarps) {
      const float* op = cpart + hg * 130;
      float M = -1e30f;
      for (int s = 0; s < C; ++s) M = fmaxf(M, ld_cluster_f32(op, s));
      float L = 0.0f, O[4] = {0.f, 0.f, 0.f, 0.f};
      for (int s = 0; s < C; ++s) {
        const float f = exp2f(ld_cluster_f32(op, s) - M);
        L += ld_cluster_f32(op + 1, s) * f;
#pragma unroll
        for (int i = 0; i < 4; ++i) O[i] += ld_cluster_f32(op + 2 + lane + 32 * i, s) * f;
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
  }
  cluster_sync_all();  // every CTA's shared memory stays alive until CTA 0 has read it
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

static size_t attn_smem() {
  return 1024 + (size_t)kAttnWarps * kAttnSlots * 2 * kTileBytes + (size_t)(kAttnWarps + 1) * 8 * 130 * 4 +
         (size_t)8 * kAttnD * 2 + kAttnWarps * kAttnSlots * 8;
}

// CTAs per cluster: no more than gives every warp one 64-position tile (1, 2,
// 4 or 8: at most 8, portable), then halved while the grid would exceed one
// wave of resident CTAs (one per SM: the K/V rings take ~155 KB of shared
// memory).  A second wave of clusters costs a whole CTA lifetime, more than the
// longer split of a smaller cluster.  Measured on B200 (40 q / 8 kv heads, CUDA
// graph over cache copies > L2), old rule (4 or 8, halved above two CTAs per SM)
// -> this one: B = 4 ctx 2048 19.2 -> 9.6 us, B = 8 ctx 128 11.3 -> 5.5 us,
// B = 16 ctx 128 10.9 -> 5.4 us, B = 16 ctx 2048 22.6 -> 16.7 us, B = 1
// unchanged at ctx >= 2048; clusters of 16 (non-portable) schedule badly (15 us
// at B = 1, ctx 2048, against 6.7 us for 8).  R4Q_ATTN_CLUSTER forces 1, 2, 4,
// 8 or 16 (measurement only).
static int attn_cluster(int B, int Hk, int max_tiles) {
  static const int forced = [] {
    const char* e = getenv("R4Q_ATTN_CLUSTER");
    return e ? atoi(e) : 0;
  }();
  if (forced == 1 || forced == 2 || forced == 4 || forced == 8 || forced == 16) return forced;
  int dev = 0, sms = 148, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_kernel, kAttnWarps * 32, attn_smem()) !=
          cudaSuccess || per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  int c = 8;
  while (c > 1 && (long)c * kAttnWarps / 2 >= max_tiles) c >>= 1;   // keep >= 1 tile per warp
  while (c > 1 && (long)B * Hk * c > (long)per_sm * sms) c >>= 1;
  return c;
}


constexpr size_t kAttnWsBytes = 256;   // status word only

static int launch_attn(const AttnParams& p, const void* k_cache, const void* v_cache, int Tmax, void* stream) {
  const long rows = (long)p.B * p.Hk * p.max_seq;
  CUtensorMap tmk, tmv;
  int st = cache_map(&tmk, k_cache, rows);
  if (!st) st = cache_map(&tmv, v_cache, rows);
  if (st) return st;
  const size_t smem = attn_smem();
  static std::mutex mu;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 64 && !attr_done[dev]) {
      cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      cudaGetLastError();
      attr_done[dev] = true;
    }
  }
  const int C = attn_cluster(p.B, p.Hk, Tmax);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(C, p.Hk, p.B);
  cfg.blockDim = dim3(kAttnWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = C;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, attn_kernel, tmk, tmv, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(R4Q_ERR_CUDA, "attn_kernel (cluster %d): %s", C, cudaGetErrorString(e));
  }
  return R4Q_OK;
}

static int attn_check(const void* q, long ldq, const void* k_cache, const void* v_cache, void* o, int B, int H,
                      int Hk, int D, int max_seq, int seq_len, const long long* seq_dev, void* ws,
                      size_t ws_bytes) {
  if (!q || !k_cache || !v_cache || !o) return set_error(R4Q_ERR_ARG, "flash_decode: null pointer");
  if (D != kAttnD) return set_error(R4Q_ERR_ARG, "flash_decode: head_dim %d (only 128)", D);
  if (B < 1 || B > 65535 || Hk < 1 || Hk > 65535 || H < Hk || H % Hk)
    return set_error(R4Q_ERR_ARG, "flash_decode: bad heads H=%d Hk=%d", H, Hk);
  if (H / Hk > 8) return set_error(R4Q_ERR_ARG, "flash_decode: GQA group %d > 8", H / Hk);
  if (max_seq < 1 || (!seq_dev && (seq_len < 0 || seq_len > max_seq)))
    return set_error(R4Q_ERR_ARG, "flash_decode: seq_len %d outside [0, %d]", seq_len, max_seq);
  if (!aligned(q, 16) || (ldq % 8) || !aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(o, 2))
    return set_error(R4Q_ERR_ALIGN, "flash_decode: q/caches must be 16-byte aligned");
  if ((long)B * Hk * max_seq > 0x7fffffffL)
    return set_error(R4Q_ERR_ARG, "flash_decode: B*Hk*max_seq above 2^31 cache rows");
  if (!ws || ws_bytes < kAttnWsBytes)
    return set_error(R4Q_ERR_CAPACITY, "flash_decode: workspace %zu < %zu bytes", ws_bytes, kAttnWsBytes);
  return R4Q_OK;
}

}  // namespace r4q

using namespace r4q;

extern "C" size_t r4q_flash_decode_workspace_bytes(int B, int H, int Hk, int max_seq) {
  if (B < 1 || H < 1 || Hk < 1 || max_seq < 1) return 0;
  return kAttnWsBytes;
}

extern "C" int r4q_flash_decode(const void* q, long ldq, const void* k_cache, const void* v_cache,
                                const float* k_scale, const float* v_scale, void* o, long ldo,
                                int B, int H, int Hk, int D, int max_seq, int seq_len,
                                const long long* seq_dev, int flags, void* ws, size_t ws_bytes,
                                void* stream) {
  int st = attn_check(q, ldq, k_cache, v_cache, o, B, H, Hk, D, max_seq, seq_len, seq_dev, ws, ws_bytes);
  if (st) return st;
  AttnParams p{};
  p.q = (const __half*)q; p.ldq = ldq;
  p.k_scale = k_scale; p.v_scale = v_scale;
  p.o = (__half*)o; p.ldo = ldo;
  p.B = B; p.H = H; p.Hk = Hk; p.Hg = H / Hk; p.max_seq = max_seq; p.seq_len = seq_len;
  p.seq_dev = seq_dev;
  p.fwht = (flags & R4Q_ATTN_FWHT) ? 1 : 0;
  p.early = 0;
  p.status = (int*)ws;
  const int Tmax = ((seq_dev ? max_seq : seq_len) + kAttnTile - 1) / kAttnTile;
  return launch_attn(p, k_cache, v_cache, Tmax, stream);
}

int r4q_attn_decode_fused_ex(const void* qkv, long ld, const void* q_norm_w, const void* k_norm_w,
                             const void* cos_tab, const void* sin_tab, long tab_stride, float eps,
                             void* k_cache, void* v_cache, const float* k_scale, const float* v_scale, void* o,
                             long ldo, int B, int H, int Hk, int D, int max_seq, int seq_len,
                             const long long* seq_dev, int flags, int early, void* ws, size_t ws_bytes,
                             void* stream) {
  int st = attn_check(qkv, ld, k_cache, v_cache, o, B, H, Hk, D, max_seq, seq_len, seq_dev, ws, ws_bytes);
  if (st) return st;
  if (!q_norm_w || !k_norm_w || !cos_tab || !sin_tab)
    return set_error(R4Q_ERR_ARG, "attn_decode_fused: norm weights and RoPE tables required");
  if (!seq_dev && seq_len < 1) return set_error(R4Q_ERR_ARG, "attn_decode_fused: seq_len must be >= 1");
  if (ld < (long)(H + 2 * Hk) * D)
    return set_error(R4Q_ERR_ARG, "attn_decode_fused: row stride %ld below (H + 2 Hk) * D", ld);
  AttnParams p{};
  const __half* base = (const __half*)qkv;
  p.q = base; p.ldq = ld;
  p.k_new = base + (long)H * D;
  p.v_new = base + (long)(H + Hk) * D;
  p.qw = (const __half*)q_norm_w; p.kw = (const __half*)k_norm_w;
  p.cos_tab = (const __half*)cos_tab; p.sin_tab = (const __half*)sin_tab;
  p.tab_stride = tab_stride > 0 ? tab_stride : D / 2;
  p.eps = eps;
  p.kc = (uint8_t*)k_cache; p.vc = (uint8_t*)v_cache;
  p.k_scale = k_scale; p.v_scale = v_scale;
  p.o = (__half*)o; p.ldo = ldo;
  p.B = B; p.H = H; p.Hk = Hk; p.Hg = H / Hk; p.max_seq = max_seq; p.seq_len = seq_len;
  p.seq_dev = seq_dev;
  p.fwht = (flags & R4Q_ATTN_FWHT) ? 1 : 0;
  p.early = early;
  p.status = (int*)ws;
  const int Tmax = ((seq_dev ? max_seq : seq_len) + kAttnTile - 1) / kAttnTile;
  return launch_attn(p, k_cache, v_cache, Tmax, stream);
}

extern "C" int r4q_attn_decode_fused(const void* qkv, long ld, const void* q_norm_w, const void* k_norm_w,
                                     const void* cos_tab, const void* sin_tab, long tab_stride, float eps,
                                     void* k_cache, void* v_cache, const float* k_scale, const float* v_scale,
                                     void* o, long ldo, int B, int H, int Hk, int D, int max_seq, int seq_len,
                                     const long long* seq_dev, int flags, void* ws, size_t ws_bytes,
                                     void* stream) {
  return r4q_attn_decode_fused_ex(qkv, ld, q_norm_w, k_norm_w, cos_tab, sin_tab, tab_stride, eps, k_cache,
                                  v_cache, k_scale, v_scale, o, ldo, B, H, Hk, D, max_seq, seq_len, seq_dev,
                                  flags, 0, ws, ws_bytes, stream);
}
