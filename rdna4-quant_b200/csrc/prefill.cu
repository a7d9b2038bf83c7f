// Row kernels of the batched prefill (int4_prefill_logits,
// int4_decode_step.hip:2127-2320): H32 FWHT of activation rows
// (hadamard_rotate_batched, :766-792), SiLU(gate)·up (silu_mul_batched,
// :2112-2124), and the INT8 dequantisation feeding the fp16 tensor-core GEMM
// for INT8 layers (int8_quant.dequantize_int8, int8_quant.py:52-69).  All
// are HBM-bound elementwise passes: one warp per 32-element block in the
// reference's butterfly order, 16-byte vector loads elsewhere.
#include "r4q_common.cuh"

namespace r4q {
namespace {

// y[r, 32b + l] = fp16(H32 x[r, 32b + .]) — one warp per block, lane l.
__global__ void fwht_rows_kernel(const __half* __restrict__ x, long ldx, __half* __restrict__ y, long ldy,
                                 int rows, int nblk) {
  const long w = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= (long)rows * nblk) return;
  const long r = w / nblk;
  const int b = (int)(w - r * nblk);
  const float v = __half2float(x[r * ldx + b * 32 + lane]);
  y[r * ldy + b * 32 + lane] = __float2half(fwht32_lane(v, lane));
}

// y[r, i] = fp16(g / (1 + exp(-g)) * u), g = x[r, i], u = x[r, I + i].
__global__ void silu_mul_kernel(const __half* __restrict__ x, long ldx, __half* __restrict__ y, long ldy,
                                int rows, int I) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)rows * I) return;
  const long r = i / I;
  const int c = (int)(i - r * I);
  const float g = __half2float(x[r * ldx + c]);
  const float u = __half2float(x[r * ldx + I + c]);
  y[r * ldy + c] = __float2half(g / (1.0f + expf(-g)) * u);
}

// out[n, k] = fp16(q * s[n, k / 32]) for int8 q (8 values per thread).
__global__ void dequant_int8_kernel(const int8_t* __restrict__ w, const __half* __restrict__ s,
                                    __half* __restrict__ out, long n8, int K) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  const long e = i * 8;
  const long n = e / K;
  const int k = (int)(e - n * K);
  const float sc = __half2float(s[n * (K / 32) + k / 32]);
  const uint2 q = *reinterpret_cast<const uint2*>(w + e);
  const uint32_t qw[2] = {q.x, q.y};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int8_t a = (int8_t)((qw[j >> 1] >> (16 * (j & 1))) & 0xFF);
    const int8_t b = (int8_t)((qw[j >> 1] >> (16 * (j & 1) + 8)) & 0xFF);
    o[j] = h2_as_u32(__floats2half2_rn((float)a * sc, (float)b * sc));
  }
  *reinterpret_cast<uint4*>(out + e) = make_uint4(o[0], o[1], o[2], o[3]);
}

}  // namespace
}  // namespace r4q

using namespace r4q;

extern "C" int r4q_fwht_rows(const void* x, long ldx, void* y, long ldy, int rows, int K, void* stream) {
  if (!x || !y || rows < 0 || K <= 0 || K % 32 || ldx < K || ldy < K)
    return set_error(R4Q_ERR_ARG, "fwht_rows: bad arguments (rows %d K %d)", rows, K);
  if (rows == 0) return R4Q_OK;
  const long warps = (long)rows * (K / 32);
  fwht_rows_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, (cudaStream_t)stream>>>(
      (const __half*)x, ldx, (__half*)y, ldy, rows, K / 32);
  return check_launch("fwht_rows_kernel");
}

extern "C" int r4q_silu_mul(const void* x, long ldx, void* y, long ldy, int rows, int I, void* stream) {
  if (!x || !y || rows < 0 || I <= 0 || ldx < 2L * I || ldy < I)
    return set_error(R4Q_ERR_ARG, "silu_mul: bad arguments (rows %d I %d)", rows, I);
  if (rows == 0) return R4Q_OK;
  const long n = (long)rows * I;
  silu_mul_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>((const __half*)x, ldx,
                                                                                 (__half*)y, ldy, rows, I);
  return check_launch("silu_mul_kernel");
}

extern "C" int r4q_dequant_int8(const void* w, const void* s, void* out, int N, int K, void* stream) {
  if (!w || !s || !out || N < 1 || K < 32 || K % 32) return set_error(R4Q_ERR_ARG, "dequant_int8: bad arguments");
  if (!aligned(w, 8) || !aligned(out, 16)) return set_error(R4Q_ERR_ALIGN, "dequant_int8: w / out misaligned");
  const long n8 = (long)N * K / 8;
  dequant_int8_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      (const int8_t*)w, (const __half*)s, (__half*)out, n8, K);
  return check_launch("dequant_int8_kernel");
}

namespace r4q {
namespace {
// cache[row b][kv head h][start + m][d] = enc(k[m, h, d] / s) for the M prompt
// rows of batch row b (k, v: rows m with stride ld, kv heads of 128 contiguous).
__global__ void kv_write_rows_kernel(const __half* __restrict__ k, const __half* __restrict__ v, long ld,
                                     uint8_t* __restrict__ kc, uint8_t* __restrict__ vc, int M, int Hk,
                                     int max_seq, int start, int b, const float* ks, const float* vs) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;      // one thread per 4 elements
  const long n = (long)M * Hk * 32;
  if (i >= n) return;
  const int d4 = (int)(i & 31);
  const long mh = i >> 5;
  const int h = (int)(mh % Hk);
  const int m = (int)(mh / Hk);
  const float sk = ks ? ks[b * Hk + h] : 1.0f, sv = vs ? vs[b * Hk + h] : 1.0f;
  const long src = (long)m * ld + (long)h * 128 + d4 * 4;
  const long dst = (((long)b * Hk + h) * max_seq + start + m) * 128 + d4 * 4;
  uint32_t ko = 0, vo = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float kf = __half2float(k[src + j]), vf = __half2float(v[src + j]);
    ko |= fp8_encode(ks ? kf / sk : kf) << (8 * j);
    vo |= fp8_encode(vs ? vf / sv : vf) << (8 * j);
  }
  *reinterpret_cast<uint32_t*>(kc + dst) = ko;
  *reinterpret_cast<uint32_t*>(vc + dst) = vo;
}
}  // namespace
}  // namespace r4q

extern "C" int r4q_kv_write_rows(const void* k, const void* v, long ld, void* k_cache, void* v_cache, int M, int Hk,
                                 int D, int max_seq, int start_pos, int batch_row, const float* k_scale,
                                 const float* v_scale, void* stream) {
  if (!k || !v || !k_cache || !v_cache || M < 0 || Hk < 1 || D != 128 || batch_row < 0 || start_pos < 0 ||
      start_pos + M > max_seq)
    return set_error(R4Q_ERR_ARG, "kv_write_rows: bad arguments (M %d start %d max_seq %d)", M, start_pos, max_seq);
  if (M == 0) return R4Q_OK;
  const long n = (long)M * Hk * 32;
  kv_write_rows_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      (const __half*)k, (const __half*)v, ld, (uint8_t*)k_cache, (uint8_t*)v_cache, M, Hk, max_seq, start_pos,
      batch_row, k_scale, v_scale);
  return check_launch("kv_write_rows_kernel");
}
