// Row RMSNorm (+ residual) and per-head RMSNorm / RoPE / FP8 KV-cache write.
//
// rows_rmsnorm_kernel: one CTA per row, y = fp16(r * rrms * w) with r = x (+ res)
// in fp32 and rrms from the unrounded r — RMSNorm.forward (engine_utils.py:58-63),
// fused_rmsnorm (fused_ops.py:12-41), rmsnorm_ds / fused_res_norm
// (int4_decode_step.hip:795-846).
//
// head_kernel: one warp per (batch row, head).  Lane l owns elements
// l + 32 j, so the half-split RoPE partners (i, i + D/2) sit in the same lane.
// Norm and RoPE run in fp32 with a single fp16 rounding (head_rmsnorm_rope_kv,
// int4_decode_step.hip:1620-1683; qknorm_rope_kernel, fused_ops.py:89-152);
// K (after norm+RoPE) and V are written to the FP8 cache at `pos` with the
// reference encoder, optionally divided by a per-(row, kv-head) fp32 scale.
#include "r4q_common.cuh"

namespace r4q {

__global__ void rows_rmsnorm_kernel(const __half* __restrict__ x, const __half* __restrict__ res,
                                    const __half* __restrict__ w, __half* __restrict__ y,
                                    __half* __restrict__ res_out, int D, long ldx, float eps) {
  const long row = blockIdx.x;
  const __half* xr = x + row * ldx;
  const __half* rr = res ? res + row * ldx : nullptr;
  __shared__ float ws[32];
  float ss = 0.0f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float v = __half2float(xr[i]);
    if (rr) v += __half2float(rr[i]);
    ss += v * v;
  }
  ss = warp_sum(ss);
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) ws[wid] = ss;
  __syncthreads();
  if (wid == 0) {
    float v = lane < nw ? ws[lane] : 0.0f;
    v = warp_sum(v);
    if (lane == 0) ws[0] = rsqrtf(v / (float)D + eps);
  }
  __syncthreads();
  const float rrms = ws[0];
  __half* yr = y + row * (long)D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float v = __half2float(xr[i]);
    if (rr) v += __half2float(rr[i]);
    yr[i] = __float2half(v * rrms * __half2float(w[i]));
    if (res_out) res_out[row * (long)D + i] = __float2half(v);
  }
}

struct HeadArgs {
  __half *q, *k;            // inputs [B][ld_in] (q heads then separate k pointer)
  const __half* v;
  const __half *qw, *kw;
  const __half *cos_tab, *sin_tab;
  long tab_stride;          // elements between table rows
  int pos;                  // used when pos_dev is null
  const long long* pos_dev; // [B] positions (device) or null
  __half *q_out, *k_out;
  uint8_t *kc, *vc;
  const float *k_scale, *v_scale;  // [B][Hk] or null
  int B, H, Hk, D, max_seq;
  long ld_in, ld_out;
  float eps;
  int flags;
};

template <int E>  // elements per lane = D / 32
__global__ void head_kernel(const HeadArgs a) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nh = a.H + a.Hk;
  if (gw >= a.B * nh) return;
  const int b = gw / nh, h = gw - b * nh;
  const bool is_q = h < a.H;
  const int kh = h - a.H;
  const __half* src = is_q ? a.q + (long)b * a.ld_in + (long)h * a.D : a.k + (long)b * a.ld_in + (long)kh * a.D;
  const __half* wt = is_q ? a.qw : a.kw;
  float v[E];
#pragma unroll
  for (int j = 0; j < E; ++j) v[j] = __half2float(src[lane + 32 * j]);
  if (a.flags & R4Q_HEAD_NORM) {
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < E; ++j) ss += v[j] * v[j];
    ss = warp_sum(ss);
    const float rrms = rsqrtf(ss / (float)a.D + a.eps);
#pragma unroll
    for (int j = 0; j < E; ++j) v[j] = v[j] * rrms * __half2float(wt[lane + 32 * j]);
  }
  const long pos = a.pos_dev ? a.pos_dev[b] : (long)a.pos;
  if (a.flags & R4Q_HEAD_ROPE) {
    const __half* cr = a.cos_tab + pos * a.tab_stride;
    const __half* sr = a.sin_tab + pos * a.tab_stride;
#pragma unroll
    for (int j = 0; j < E / 2; ++j) {
      const int i = lane + 32 * j;
      const float c = __half2float(cr[i]), s = __half2float(sr[i]);
      const float e = v[j], o = v[j + E / 2];
      v[j] = e * c - o * s;
      v[j + E / 2] = o * c + e * s;
    }
  }
  __half* obase = is_q ? a.q_out : a.k_out;
  if (obase) {
    __half* dst = obase + (long)b * a.ld_out + (long)(is_q ? h : kh) * a.D;
#pragma unroll
    for (int j = 0; j < E; ++j) dst[lane + 32 * j] = __float2half(v[j]);
  }
  if (!is_q && (a.flags & R4Q_HEAD_KV) && pos >= 0 && pos < a.max_seq) {
    const long off = (((long)b * a.Hk + kh) * a.max_seq + pos) * a.D;
    const float ks = a.k_scale ? a.k_scale[b * a.Hk + kh] : 1.0f;
    const float vs = a.v_scale ? a.v_scale[b * a.Hk + kh] : 1.0f;
    const __half* vsrc = a.v + (long)b * a.ld_in + (long)kh * a.D;
#pragma unroll
    for (int j = 0; j < E; ++j) {
      const int i = lane + 32 * j;
      a.kc[off + i] = (uint8_t)fp8_encode(a.k_scale ? v[j] / ks : v[j]);
      const float vv = __half2float(vsrc[i]);
      a.vc[off + i] = (uint8_t)fp8_encode(a.v_scale ? vv / vs : vv);
    }
  }
}

}  // namespace r4q

using namespace r4q;

extern "C" int r4q_rmsnorm(const void* x, const void* res, const void* w, void* y, void* res_out,
                           int rows, int D, long ldx, float eps, void* stream) {
  if (!x || !w || !y || rows < 0 || D <= 0 || (rows > 0 && ldx < D))
    return set_error(R4Q_ERR_ARG, "rmsnorm: bad arguments (rows=%d D=%d ldx=%ld)", rows, D, ldx);
  if (rows == 0) return R4Q_OK;
  rows_rmsnorm_kernel<<<rows, 256, 0, (cudaStream_t)stream>>>(
      (const __half*)x, (const __half*)res, (const __half*)w, (__half*)y, (__half*)res_out, D, ldx,
      eps);
  return check_launch("rows_rmsnorm_kernel");
}

extern "C" int r4q_head_norm_rope(void* q, void* k, const void* v, const void* q_norm_w,
                                  const void* k_norm_w, const void* cos_tab, const void* sin_tab,
                                  long tab_stride, int pos, const long long* pos_dev, void* q_out,
                                  void* k_out, void* k_cache, void* v_cache, const float* k_scale,
                                  const float* v_scale, int B, int H, int Hk, int D, long ld_in,
                                  long ld_out, int max_seq, float eps, int flags, void* stream) {
  if (B < 1 || H < 0 || Hk < 0 || H + Hk == 0)
    return set_error(R4Q_ERR_ARG, "head_norm_rope: bad shape B=%d H=%d Hk=%d", B, H, Hk);
  if (D != 64 && D != 128 && D != 256)
    return set_error(R4Q_ERR_ARG, "head_norm_rope: head_dim %d not in {64,128,256}", D);
  if ((H && !q) || (Hk && !k)) return set_error(R4Q_ERR_ARG, "head_norm_rope: null q/k");
  if ((flags & R4Q_HEAD_NORM) && ((H && !q_norm_w) || (Hk && !k_norm_w)))
    return set_error(R4Q_ERR_ARG, "head_norm_rope: norm weights required");
  if ((flags & R4Q_HEAD_ROPE) && (!cos_tab || !sin_tab))
    return set_error(R4Q_ERR_ARG, "head_norm_rope: rope tables required");
  if (flags & R4Q_HEAD_KV) {
    if (!v || !k_cache || !v_cache || max_seq <= 0)
      return set_error(R4Q_ERR_ARG, "head_norm_rope: KV write needs v and both caches");
    if (!pos_dev && (pos < 0 || pos >= max_seq))
      return set_error(R4Q_ERR_CAPACITY, "head_norm_rope: pos %d outside the cache (max_seq %d)", pos, max_seq);
  }
  HeadArgs a;
  a.q = (__half*)q; a.k = (__half*)k; a.v = (const __half*)v;
  a.qw = (const __half*)q_norm_w; a.kw = (const __half*)k_norm_w;
  a.cos_tab = (const __half*)cos_tab; a.sin_tab = (const __half*)sin_tab;
  a.tab_stride = tab_stride > 0 ? tab_stride : D / 2;
  a.pos = pos; a.pos_dev = pos_dev;
  a.q_out = (__half*)q_out; a.k_out = (__half*)k_out;
  a.kc = (uint8_t*)k_cache; a.vc = (uint8_t*)v_cache;
  a.k_scale = k_scale; a.v_scale = v_scale;
  a.B = B; a.H = H; a.Hk = Hk; a.D = D; a.max_seq = max_seq;
  a.ld_in = ld_in; a.ld_out = ld_out; a.eps = eps; a.flags = flags;
  const int warps = B * (H + Hk);
  const int wpb = 4;
  dim3 grid((warps + wpb - 1) / wpb);
  cudaStream_t st = (cudaStream_t)stream;
  switch (D) {
    case 64: head_kernel<2><<<grid, wpb * 32, 0, st>>>(a); break;
    case 128: head_kernel<4><<<grid, wpb * 32, 0, st>>>(a); break;
    default: head_kernel<8><<<grid, wpb * 32, 0, st>>>(a); break;
  }
  return check_launch("head_kernel");
}
