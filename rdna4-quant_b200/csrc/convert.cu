// Format conversions: INT4 dequant to fp16, fp16 <-> FP8 with the reference codec.
#include "r4q_common.cuh"

namespace r4q {

// One thread per 32-block: 16 packed bytes + (scale, zero) -> 32 fp16.
// fp16((q - z) * s): the float product is exact, so one RN rounding gives the
// same bits as dequantize_int4_asym (int4_quant_v2.py:105-127).
__global__ void dequant_int4_kernel(const uint8_t* __restrict__ packed,
                                    const __half2* __restrict__ sz, __half* __restrict__ out,
                                    long nblocks) {
  for (long b = blockIdx.x * (long)blockDim.x + threadIdx.x; b < nblocks;
       b += (long)gridDim.x * blockDim.x) {
    const uint4 w = ldg_stream128(packed + b * 16);
    const __half2 p = sz[b];
    const float s = __low2float(p), z = __high2float(p);
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
    uint4 o[4];
    uint32_t* ov = reinterpret_cast<uint32_t*>(o);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t byte = (words[i] >> (8 * j)) & 0xFFu;
        const __half lo = __float2half_rn(((float)(byte & 0xF) - z) * s);
        const __half hi = __float2half_rn(((float)(byte >> 4) - z) * s);
        ov[i * 4 + j] = h2_as_u32(__halves2half2(lo, hi));
      }
    }
    uint4* dst = reinterpret_cast<uint4*>(out + b * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = o[i];
  }
}

__global__ void fp16_to_fp8_kernel(const __half* __restrict__ src, uint8_t* __restrict__ dst,
                                   long n, int vec) {
  const long stride = (long)gridDim.x * blockDim.x;
  const long tid = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (vec) {
    const long n8 = n / 8;
    for (long i = tid; i < n8; i += stride) {
      const uint4 q = reinterpret_cast<const uint4*>(src)[i];
      const __half* h = reinterpret_cast<const __half*>(&q);
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) lo |= fp8_encode(__half2float(h[j])) << (8 * j);
#pragma unroll
      for (int j = 0; j < 4; ++j) hi |= fp8_encode(__half2float(h[4 + j])) << (8 * j);
      reinterpret_cast<uint2*>(dst)[i] = make_uint2(lo, hi);
    }
    for (long i = n8 * 8 + tid; i < n; i += stride) dst[i] = (uint8_t)fp8_encode(__half2float(src[i]));
  } else {
    for (long i = tid; i < n; i += stride) dst[i] = (uint8_t)fp8_encode(__half2float(src[i]));
  }
}

__global__ void fp8_to_fp32_kernel(const uint8_t* __restrict__ src, float* __restrict__ dst,
                                   long n) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
       i += (long)gridDim.x * blockDim.x)
    dst[i] = fp8_decode(src[i]);
}

static int grid_for(long work, int threads) {
  long g = (work + threads - 1) / threads;
  const long cap = (long)num_sms() * 16;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace r4q

using namespace r4q;

extern "C" int r4q_dequant_int4(const void* packed, const void* sz, void* out, int N, int K,
                                void* stream) {
  if (!packed || !sz || !out) return set_error(R4Q_ERR_ARG, "dequant_int4: null pointer");
  if (N <= 0 || K <= 0 || K % 32) return set_error(R4Q_ERR_ARG, "dequant_int4: bad N=%d K=%d", N, K);
  if (!aligned(packed, 16) || !aligned(out, 16) || !aligned(sz, 4))
    return set_error(R4Q_ERR_ALIGN, "dequant_int4: packed/out need 16-byte, scales 4-byte alignment");
  const long nb = (long)N * (K / 32);
  dequant_int4_kernel<<<grid_for(nb, 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint8_t*)packed, (const __half2*)sz, (__half*)out, nb);
  return check_launch("dequant_int4_kernel");
}

extern "C" int r4q_fp16_to_fp8(const void* src, void* dst, long n, void* stream) {
  if (n < 0 || (n > 0 && (!src || !dst))) return set_error(R4Q_ERR_ARG, "fp16_to_fp8: bad args");
  if (n == 0) return R4Q_OK;
  const int vec = aligned(src, 16) && aligned(dst, 8);
  fp16_to_fp8_kernel<<<grid_for(vec ? n / 8 + 1 : n, 256), 256, 0, (cudaStream_t)stream>>>(
      (const __half*)src, (uint8_t*)dst, n, vec);
  return check_launch("fp16_to_fp8_kernel");
}

extern "C" int r4q_fp8_to_fp32(const void* src, void* dst, long n, void* stream) {
  if (n < 0 || (n > 0 && (!src || !dst))) return set_error(R4Q_ERR_ARG, "fp8_to_fp32: bad args");
  if (n == 0) return R4Q_OK;
  fp8_to_fp32_kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint8_t*)src, (float*)dst, n);
  return check_launch("fp8_to_fp32_kernel");
}
