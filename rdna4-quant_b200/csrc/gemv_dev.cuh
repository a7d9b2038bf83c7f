// Device-side pieces shared by the GEMV kernels (LDG path and TMA path).
#pragma once
#include "r4q_common.cuh"
#include "gemv.cuh"

namespace r4q {

template <int FMT> struct Fmt;
// INT4: a chunk is 16 bytes of one row = 32 k = one quantisation block.
template <> struct Fmt<W_INT4> { static constexpr int CK = 32, NSUB = 4, U = 1; };
// INT8: a chunk is 16 bytes = 16 k (half a block); two chunks per thread-step.
template <> struct Fmt<W_INT8> { static constexpr int CK = 16, NSUB = 2, U = 2; };
// FP16: a chunk is 16 bytes = 8 k.
template <> struct Fmt<W_FP16> { static constexpr int CK = 8, NSUB = 1, U = 2; };

struct GemvParams {
  const __half* x;
  long ldx;
  const uint8_t* w;
  const __half* s;
  __half* y;
  long ldy;
  int B, N, K;
  int mt;        // 16-row m-tiles per CTA (1, 2 or 4)
  int ksplit;    // K splits (gridDim.y)
  int prologue;
  unsigned* cnt; // per-row-tile arrival counters (zero between launches)
  float* part;   // [ksplit][B][N] fp32 partial sums
  // fused RMSNorm prologue
  const __half* norm_w;  // [K]
  float eps;
  const float* ss_in;    // [ss_in_parts][B] or null (then computed from x)
  int ss_in_parts;
  // fused residual epilogue
  const __half* res;     // [B][ldres] or null
  long ldres;
  float* ss_out;         // [N/16][B] or null
  // fp32 outputs instead of y (no rounding, no residual): each value goes to
  // all npush arrays, y32p[q][c * ldy + n] (tensor-parallel partials pushed
  // straight into the peers' reduce buffers)
  float* y32p[8];
  int npush;
  TpExchange tpx;  // tensor-parallel exchange (zero outside TP)
};

// Tensor-parallel consumer input: 8 fp16 values r = fp16(fp16(sum over src of
// the fp32 partials) + residual) of row `col`, elements k..k+7 (K = hidden).
__device__ __forceinline__ void tp_sum8(const GemvParams& p, int col, int k, float (&a)[8]) {
  const float* rb = p.tpx.red + (long)col * p.K + k;      // element index (float or word)
  if (p.tpx.ll_wait) {
    // 16-byte L2 loads of the tagged words (a stale word just fails its tag
    // check); any word not yet arrived is then polled on its own
    const unsigned tag = (unsigned)tp_epoch(p.tpx, p.tpx.wait_idx);
    for (int s = 0; s < p.tpx.nwait; ++s) {
      const long i0 = (long)s * p.tpx.red_slot + (long)col * p.K + k;
      const ulonglong2* w2 = reinterpret_cast<const ulonglong2*>(reinterpret_cast<const unsigned long long*>(p.tpx.red) + i0);
      unsigned long long w[8];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const ulonglong2 v = __ldcg(w2 + h);
        w[2 * h] = v.x;
        w[2 * h + 1] = v.y;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float f = (unsigned)(w[j] >> 32) == tag ? __uint_as_float((unsigned)w[j])
                                                       : tp_read_word(p.tpx, p.tpx.red, i0 + j, tag, s);
        a[j] = s == 0 ? f : a[j] + f;
      }
    }
    return;
  }
  float4 a0 = __ldcg(reinterpret_cast<const float4*>(rb));
  float4 a1 = __ldcg(reinterpret_cast<const float4*>(rb + 4));
  for (int s = 1; s < p.tpx.nwait; ++s) {
    const float4 b0 = __ldcg(reinterpret_cast<const float4*>(rb + s * p.tpx.red_slot));
    const float4 b1 = __ldcg(reinterpret_cast<const float4*>(rb + s * p.tpx.red_slot + 4));
    a0.x += b0.x; a0.y += b0.y; a0.z += b0.z; a0.w += b0.w;
    a1.x += b1.x; a1.y += b1.y; a1.z += b1.z; a1.w += b1.w;
  }
  a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
  a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
}

__device__ __forceinline__ uint4 tp_row8(const GemvParams& p, int col, int k) {
  float a[8];
  tp_sum8(p, col, k, a);
  const uint4 rr = *reinterpret_cast<const uint4*>(p.tpx.red_res + (long)col * p.K + k);
  const __half* hr = reinterpret_cast<const __half*>(&rr);
  uint4 out;
  __half* ho = reinterpret_cast<__half*>(&out);
#pragma unroll
  for (int j = 0; j < 8; ++j) ho[j] = __float2half(__half2float(__float2half(a[j])) + __half2float(hr[j]));
  return out;
}

// tp_row8 plus the sum of squares of the unrounded fp16(sum) + residual
// values (what the residual epilogue of the 1-GPU path accumulates).
__device__ __forceinline__ uint4 tp_row8_ss(const GemvParams& p, int col, int k, float& ss) {
  float a[8];
  tp_sum8(p, col, k, a);
  const uint4 rr = *reinterpret_cast<const uint4*>(p.tpx.red_res + (long)col * p.K + k);
  const __half* hr = reinterpret_cast<const __half*>(&rr);
  uint4 out;
  __half* ho = reinterpret_cast<__half*>(&out);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float v = __half2float(__float2half(a[j])) + __half2float(hr[j]);
    ss += v * v;
    ho[j] = __float2half(v);
  }
  return out;
}

__host__ __device__ inline int steps_total(int K, int ck, int u) {
  const int nch = K / ck;
  return (nch + 4 * u - 1) / (4 * u);
}

// shared-memory bytes per activation column for a CTA covering `nsteps` steps
__host__ __device__ inline int x_colstride(int nsteps, int nsub, int u) {
  int b = nsub * nsteps * 4 * u * 16;
  b = (b + 127) / 128 * 128 + 64;  // odd multiple of 64: columns g, g+1 hit disjoint banks
  return b;
}

// ------------------------------------------------------------ prologue ----
// Loads 32 activations of column `col` starting at k0, applies the prologue
// PRO (compile-time, so a kernel carries only its own prologue's code) and
// returns them as fp16 in v[0..31].
template <int PRO>
__device__ __forceinline__ void load_block32_t(const GemvParams& p, int col, int k0, float rrms,
                                               __half (&v)[32]) {
  const __half* xr = p.x + (long)col * p.ldx;
  if (k0 >= p.K) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __float2half(0.0f);
    return;
  }
  if constexpr (PRO == R4Q_PRO_NONE) {
    const uint4* src = reinterpret_cast<const uint4*>(xr + k0);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 q = src[i];
      *reinterpret_cast<uint4*>(&v[8 * i]) = q;
    }
    return;
  } else {
    float f[32];
    if constexpr (PRO == R4Q_PRO_RMSNORM_FWHT) {
      // fp16(x) * rrms * w, then H32 (fused_res_norm_fwht phase 2, hip:1178-1190)
      const uint4* src = reinterpret_cast<const uint4*>(xr + k0);
      const uint4* ws = reinterpret_cast<const uint4*>(p.norm_w + k0);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 q = src[i], wq = __ldg(ws + i);
        const __half* h = reinterpret_cast<const __half*>(&q);
        const __half* wh = reinterpret_cast<const __half*>(&wq);
#pragma unroll
        for (int j = 0; j < 8; ++j) f[8 * i + j] = __half2float(h[j]) * rrms * __half2float(wh[j]);
      }
    } else if constexpr (PRO == R4Q_PRO_FWHT) {
      const uint4* src = reinterpret_cast<const uint4*>(xr + k0);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 q = src[i];
        const __half* h = reinterpret_cast<const __half*>(&q);
#pragma unroll
        for (int j = 0; j < 8; ++j) f[8 * i + j] = __half2float(h[j]);
      }
    } else {  // R4Q_PRO_SILU_FWHT: g = x[:, k], u = x[:, K + k]   (hip:1031-1051)
      const uint4* sg = reinterpret_cast<const uint4*>(xr + k0);
      const uint4* su = reinterpret_cast<const uint4*>(xr + p.K + k0);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 qg = sg[i], qu = su[i];
        const __half* hg = reinterpret_cast<const __half*>(&qg);
        const __half* hu = reinterpret_cast<const __half*>(&qu);
#pragma unroll
        for (int j = 0; j < 8; ++j) f[8 * i + j] = silu_f(__half2float(hg[j])) * __half2float(hu[j]);
      }
    }
    fwht32_regs(f);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __float2half(f[i]);
  }
}

// Runtime-prologue form (the register-staged kernel).
__device__ __forceinline__ void load_block32(const GemvParams& p, int col, int k0, float rrms,
                                             __half (&v)[32]) {
  switch (p.prologue) {
    case R4Q_PRO_FWHT: load_block32_t<R4Q_PRO_FWHT>(p, col, k0, rrms, v); return;
    case R4Q_PRO_SILU_FWHT: load_block32_t<R4Q_PRO_SILU_FWHT>(p, col, k0, rrms, v); return;
    case R4Q_PRO_RMSNORM_FWHT: load_block32_t<R4Q_PRO_RMSNORM_FWHT>(p, col, k0, rrms, v); return;
    default: load_block32_t<R4Q_PRO_NONE>(p, col, k0, rrms, v); return;
  }
}

// Writes one 32-block of activations into the permuted shared layout.
// Layout per column: [sub][chunk][16 bytes]; chunk = local chunk index.
template <int FMT>
__device__ __forceinline__ void store_block32(uint8_t* xs_col, int nch_pad, int blk_local,
                                              const __half (&v)[32]) {
  using F = Fmt<FMT>;
  auto put = [&](int sub, int chunk, __half a0, __half a1, __half a2, __half a3, __half a4,
                 __half a5, __half a6, __half a7) {
    __half t[8] = {a0, a1, a2, a3, a4, a5, a6, a7};
    *reinterpret_cast<uint4*>(xs_col + ((long)sub * nch_pad + chunk) * 16) =
        *reinterpret_cast<uint4*>(t);
  };
  if constexpr (FMT == W_INT4) {
    // word m (k = 8m..8m+7) pairs (0,4),(1,5),(2,6),(3,7)
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int b = 8 * m;
      put(m, blk_local, v[b], v[b + 4], v[b + 1], v[b + 5], v[b + 2], v[b + 6], v[b + 3], v[b + 7]);
    }
  } else if constexpr (FMT == W_INT8) {
    // chunk of 16 k: word m (k = 4m..4m+3) pairs (0,2),(1,3); sub = m / 2
#pragma unroll
    for (int c = 0; c < 2; ++c) {
#pragma unroll
      for (int sub = 0; sub < 2; ++sub) {
        const int b = 16 * c + 8 * sub;
        put(sub, 2 * blk_local + c, v[b], v[b + 2], v[b + 1], v[b + 3], v[b + 4], v[b + 6],
            v[b + 5], v[b + 7]);
      }
    }
  } else {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int b = 8 * c;
      put(0, 4 * blk_local + c, v[b], v[b + 1], v[b + 2], v[b + 3], v[b + 4], v[b + 5], v[b + 6],
          v[b + 7]);
    }
  }
  (void)F::CK;
}

// --------------------------------------------------------- dequant math ---
struct RowChunk {
  uint4 w;      // 16 weight bytes
  uint32_t s;   // INT4: (scale, zero) half2;  INT8: scale in the low half
};

// INT4 word -> 4 half2 of fp16((q - z) * s), pairs (k0,k4),(k1,k5),(k2,k6),(k3,k7)
__device__ __forceinline__ void deq_int4_word(uint32_t w, __half2 z1024, __half2 nz64, __half2 s2,
                                              uint32_t (&o)[4]) {
  const __half2 sixteenth = __float2half2_rn(0.0625f);
  const uint32_t w8 = w >> 8;
  __half2 p0 = u32_as_h2(lop3_and_or(w, 0x000F000Fu, 0x64006400u));
  __half2 p1 = u32_as_h2(lop3_and_or(w, 0x00F000F0u, 0x64006400u));
  __half2 p2 = u32_as_h2(lop3_and_or(w8, 0x000F000Fu, 0x64006400u));
  __half2 p3 = u32_as_h2(lop3_and_or(w8, 0x00F000F0u, 0x64006400u));
  o[0] = h2_as_u32(__hmul2(__hsub2(p0, z1024), s2));
  o[1] = h2_as_u32(__hmul2(__hfma2(p1, sixteenth, nz64), s2));
  o[2] = h2_as_u32(__hmul2(__hsub2(p2, z1024), s2));
  o[3] = h2_as_u32(__hmul2(__hfma2(p3, sixteenth, nz64), s2));
}

// INT8 word (4 signed bytes k0..k3) -> (k0,k2),(k1,k3) as fp16(q * s)
__device__ __forceinline__ void deq_int8_word(uint32_t w, __half2 s2, uint32_t& o0, uint32_t& o1) {
  const __half2 off = __float2half2_rn(1152.0f);
  const uint32_t wx = w ^ 0x80808080u;
  __half2 p0 = u32_as_h2(prmt(wx, 0x64646464u, 0x4240u));
  __half2 p1 = u32_as_h2(prmt(wx, 0x64646464u, 0x4341u));
  o0 = h2_as_u32(__hmul2(__hsub2(p0, off), s2));
  o1 = h2_as_u32(__hmul2(__hsub2(p1, off), s2));
}

template <int FMT, int NG>
__device__ __forceinline__ void chunk_mma(const RowChunk& ra, const RowChunk& rb,
                                          const uint8_t* xs, int colstride, int nch_pad,
                                          int lchunk, const int (&colx)[NG], float (&acc)[NG][4]) {
  using F = Fmt<FMT>;
  // activation fragments for this chunk, per column group
  uint4 xf[NG][F::NSUB];
#pragma unroll
  for (int cg = 0; cg < NG; ++cg)
#pragma unroll
    for (int sub = 0; sub < F::NSUB; ++sub)
      xf[cg][sub] = *reinterpret_cast<const uint4*>(xs + (long)colx[cg] * colstride +
                                                    ((long)sub * nch_pad + lchunk) * 16);
  if constexpr (FMT == W_INT4) {
    const __half2 sza = u32_as_h2(ra.s), szb = u32_as_h2(rb.s);
    const __half2 c1024 = __float2half2_rn(1024.0f), c64 = __float2half2_rn(64.0f);
    const __half2 za = __high2half2(sza), zb = __high2half2(szb);
    const __half2 za1024 = __hadd2(za, c1024), zb1024 = __hadd2(zb, c1024);
    const __half2 nza64 = __hneg2(__hadd2(za, c64)), nzb64 = __hneg2(__hadd2(zb, c64));
    const __half2 sa = __low2half2(sza), sb = __low2half2(szb);
    const uint32_t wa[4] = {ra.w.x, ra.w.y, ra.w.z, ra.w.w};
    const uint32_t wb[4] = {rb.w.x, rb.w.y, rb.w.z, rb.w.w};
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      uint32_t A[4], Bq[4];
      deq_int4_word(wa[m], za1024, nza64, sa, A);
      deq_int4_word(wb[m], zb1024, nzb64, sb, Bq);
#pragma unroll
      for (int cg = 0; cg < NG; ++cg) {
        mma16816(acc[cg], A[0], Bq[0], A[1], Bq[1], xf[cg][m].x, xf[cg][m].y);
        mma16816(acc[cg], A[2], Bq[2], A[3], Bq[3], xf[cg][m].z, xf[cg][m].w);
      }
    }
  } else if constexpr (FMT == W_INT8) {
    const __half2 sa = __low2half2(u32_as_h2(ra.s)), sb = __low2half2(u32_as_h2(rb.s));
    const uint32_t wa[4] = {ra.w.x, ra.w.y, ra.w.z, ra.w.w};
    const uint32_t wb[4] = {rb.w.x, rb.w.y, rb.w.z, rb.w.w};
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      uint32_t a0, a1, b0, b1;
      deq_int8_word(wa[m], sa, a0, a1);
      deq_int8_word(wb[m], sb, b0, b1);
#pragma unroll
      for (int cg = 0; cg < NG; ++cg) {
        const uint4& q = xf[cg][m >> 1];
        const uint32_t x0 = (m & 1) ? q.z : q.x;
        const uint32_t x1 = (m & 1) ? q.w : q.y;
        mma16816(acc[cg], a0, b0, a1, b1, x0, x1);
      }
    }
  } else {
#pragma unroll
    for (int cg = 0; cg < NG; ++cg) {
      mma16816(acc[cg], ra.w.x, rb.w.x, ra.w.y, rb.w.y, xf[cg][0].x, xf[cg][0].y);
      mma16816(acc[cg], ra.w.z, rb.w.z, ra.w.w, rb.w.w, xf[cg][0].z, xf[cg][0].w);
    }
  }
}


// Activation staging with 4 lanes per 32-block: lane q of a quad owns k =
// 8q..8q+7, applies the prologue, runs the FWHT (strides 1,2,4 in registers,
// 8 and 16 across the quad, same stage order as the 32-register form) and
// stores its 8 values as one 16-byte sub-row of the permuted layout.
// Split in two so that a thread can issue the loads of several items before
// it waits for any of them (one memory round trip for the whole staging):
// stage_load reads the raw inputs, stage_finish computes and stores.  All 32
// lanes of the warp must call stage_finish (shuffles); `valid` masks stores.
struct QuadIn {
  uint4 a;   // 8 fp16 of x (SiLU prologue: the gate half)
  uint4 b;   // SiLU prologue: the 8 matching values of the up half
  uint4 w;   // RMSNorm prologue: the 8 norm weights
};

__device__ __forceinline__ QuadIn stage_load(const GemvParams& p, int col, int k0, int q, bool valid,
                                             bool have_raw = false, uint4 raw_in = uint4{0, 0, 0, 0}) {
  QuadIn in{};
  if (!(valid && k0 < p.K)) return in;
  const __half* xr = p.x + (long)col * p.ldx + k0 + 8 * q;
  if (have_raw) in.a = raw_in;
  else if (p.tpx.nwait && p.prologue != R4Q_PRO_NONE) in.a = tp_row8(p, col, k0 + 8 * q);
  else in.a = *reinterpret_cast<const uint4*>(xr);
  if (p.prologue == R4Q_PRO_SILU_FWHT) in.b = *reinterpret_cast<const uint4*>(xr + p.K);
  if (p.prologue == R4Q_PRO_RMSNORM_FWHT) in.w = __ldg(reinterpret_cast<const uint4*>(p.norm_w + k0 + 8 * q));
  return in;
}

template <int FMT, bool DIAG>
__device__ __forceinline__ void stage_finish(const GemvParams& p, const QuadIn& in, int k0, int q, float rrms,
                                             uint8_t* xs_col, int nch_pad, int blk, bool valid,
                                             float2* xsum_slot) {
  __half v[8];
  const bool inr = valid && k0 < p.K;
  if (p.prologue == R4Q_PRO_NONE) {
    *reinterpret_cast<uint4*>(v) = in.a;
  } else {
    float f[8];
    if (inr) {
      const __half* h = reinterpret_cast<const __half*>(&in.a);
      if (p.prologue == R4Q_PRO_SILU_FWHT) {
        const __half* hu = reinterpret_cast<const __half*>(&in.b);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          f[j] = silu_f(__half2float(h[j])) * __half2float(hu[j]);
        }
      } else if (p.prologue == R4Q_PRO_RMSNORM_FWHT) {
        const __half* hw = reinterpret_cast<const __half*>(&in.w);
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = __half2float(h[j]) * rrms * __half2float(hw[j]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = __half2float(h[j]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = 0.0f;
    }
#pragma unroll
    for (int s = 1; s < 8; s <<= 1) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if ((j & s) == 0) {
          const float a = f[j], b = f[j + s];
          f[j] = a + b;
          f[j + s] = a - b;
        }
      }
    }
#pragma unroll
    for (int s = 1; s < 4; s <<= 1) {   // k strides 8 and 16: lane q ^ s
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float o = __shfl_xor_sync(0xffffffffu, f[j], s);
        f[j] = (q & s) ? (o - f[j]) : (f[j] + o);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __float2half(f[j] * kInvSqrt32);
  }
  if constexpr (DIAG) {
    float se = 0.0f, so = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      se += __half2float(v[j]);
      so += __half2float(v[j + 1]);
    }
    se += __shfl_xor_sync(0xffffffffu, se, 1);
    so += __shfl_xor_sync(0xffffffffu, so, 1);
    se += __shfl_xor_sync(0xffffffffu, se, 2);
    so += __shfl_xor_sync(0xffffffffu, so, 2);
    if (valid && q == 0) *xsum_slot = make_float2(se + so, 1024.0f * se + 64.0f * so);
  }
  if (!valid) return;
  __half o[8];
  int sub, chunk;
  if constexpr (FMT == W_INT4) {
    o[0] = v[0]; o[1] = v[4]; o[2] = v[1]; o[3] = v[5]; o[4] = v[2]; o[5] = v[6]; o[6] = v[3]; o[7] = v[7];
    sub = q;
    chunk = blk;
  } else if constexpr (FMT == W_INT8) {
    o[0] = v[0]; o[1] = v[2]; o[2] = v[1]; o[3] = v[3]; o[4] = v[4]; o[5] = v[6]; o[6] = v[5]; o[7] = v[7];
    sub = q & 1;
    chunk = 2 * blk + (q >> 1);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = v[j];
    sub = 0;
    chunk = 4 * blk + q;
  }
  *reinterpret_cast<uint4*>(xs_col + ((long)sub * nch_pad + chunk) * 16) = *reinterpret_cast<uint4*>(o);
}

// MMAs per 16-byte chunk: INT4 8 (32 k), INT8 4 (16 k), FP16 2 (8 k).
template <int FMT> struct ChunkMma { static constexpr int N = FMT == W_INT4 ? 8 : (FMT == W_INT8 ? 4 : 2); };

// Dequantises one chunk of rows a and b into the A operands of its MMAs:
// frag[j] = {row a lo-k, row b lo-k, row a hi-k, row b hi-k} of MMA j.
template <int FMT>
__device__ __forceinline__ void chunk_dequant(const RowChunk& ra, const RowChunk& rb,
                                              uint32_t (&frag)[ChunkMma<FMT>::N][4]) {
  if constexpr (FMT == W_INT4) {
    const __half2 sza = u32_as_h2(ra.s), szb = u32_as_h2(rb.s);
    const __half2 c1024 = __float2half2_rn(1024.0f), c64 = __float2half2_rn(64.0f);
    const __half2 za = __high2half2(sza), zb = __high2half2(szb);
    const __half2 za1024 = __hadd2(za, c1024), zb1024 = __hadd2(zb, c1024);
    const __half2 nza64 = __hneg2(__hadd2(za, c64)), nzb64 = __hneg2(__hadd2(zb, c64));
    const __half2 sa = __low2half2(sza), sb = __low2half2(szb);
    const uint32_t wa[4] = {ra.w.x, ra.w.y, ra.w.z, ra.w.w};
    const uint32_t wb[4] = {rb.w.x, rb.w.y, rb.w.z, rb.w.w};
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      uint32_t A[4], Bq[4];
      deq_int4_word(wa[m], za1024, nza64, sa, A);
      deq_int4_word(wb[m], zb1024, nzb64, sb, Bq);
      frag[2 * m][0] = A[0]; frag[2 * m][1] = Bq[0]; frag[2 * m][2] = A[1]; frag[2 * m][3] = Bq[1];
      frag[2 * m + 1][0] = A[2]; frag[2 * m + 1][1] = Bq[2]; frag[2 * m + 1][2] = A[3]; frag[2 * m + 1][3] = Bq[3];
    }
  } else if constexpr (FMT == W_INT8) {
    const __half2 sa = __low2half2(u32_as_h2(ra.s)), sb = __low2half2(u32_as_h2(rb.s));
    const uint32_t wa[4] = {ra.w.x, ra.w.y, ra.w.z, ra.w.w};
    const uint32_t wb[4] = {rb.w.x, rb.w.y, rb.w.z, rb.w.w};
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      deq_int8_word(wa[m], sa, frag[m][0], frag[m][2]);
      deq_int8_word(wb[m], sb, frag[m][1], frag[m][3]);
    }
  } else {
    frag[0][0] = ra.w.x; frag[0][1] = rb.w.x; frag[0][2] = ra.w.y; frag[0][3] = rb.w.y;
    frag[1][0] = ra.w.z; frag[1][1] = rb.w.z; frag[1][2] = ra.w.w; frag[1][3] = rb.w.w;
  }
}

// MMAs of one dequantised chunk against the staged activations; MMA j uses
// activation sub-row j/2 (words x,y for even j, z,w for odd j) and
// accumulator chain j&1, so consecutive MMAs are independent.
template <int FMT, int NG>
__device__ __forceinline__ void chunk_mma_frag(const uint32_t (&frag)[ChunkMma<FMT>::N][4],
                                               const uint8_t* xs, int colstride, int nch_pad,
                                               int lchunk, const int (&colx)[NG],
                                               float (&acc)[NG][2][4]) {
  constexpr int NM = ChunkMma<FMT>::N;
#pragma unroll
  for (int cg = 0; cg < NG; ++cg) {
#pragma unroll
    for (int sub = 0; sub < NM / 2; ++sub) {
      const uint4 xf = *reinterpret_cast<const uint4*>(xs + (long)colx[cg] * colstride +
                                                       ((long)sub * nch_pad + lchunk) * 16);
      const int j = 2 * sub;
      mma16816(acc[cg][0], frag[j][0], frag[j][1], frag[j][2], frag[j][3], xf.x, xf.y);
      mma16816(acc[cg][1], frag[j + 1][0], frag[j + 1][1], frag[j + 1][2], frag[j + 1][3], xf.z, xf.w);
    }
  }
}

}  // namespace r4q
