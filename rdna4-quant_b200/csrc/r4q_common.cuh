// Common device/host helpers for the r4q B200 decode path (sm_100a only).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/r4q.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "r4q is written for sm_100a (B200) only"
#endif

namespace r4q {

// ---------------------------------------------------------------- host side
// Records a message for r4q_last_error() and returns the status.
int set_error(int status, const char* fmt, ...);
int check_launch(const char* what);
int num_sms();
inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Launch with programmatic dependent launch allowed: the kernel's CTAs may
// be scheduled while the previous kernel of the stream finishes, so the
// kernel must call pdl_wait() before touching anything that kernel writes.
// Hides the launch gap between the short kernels of a decode step.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ------------------------------------------------------------- device side
// wait for the previous kernel of the stream (complete, writes visible), then
// let the next one be scheduled
__device__ __forceinline__ void pdl_wait_trigger() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  uint32_t d;
  // (a & mask) | orv  -> immediate LUT 0xEA
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(orv));
  return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Streaming 128-bit load of read-once data (weights): bypass L1 allocation.
__device__ __forceinline__ uint4 ldg_stream128(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ldg_stream32(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ldg_stream64(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

// D(16x8,f32) += A(16x16,f16,row) * B(16x8,f16,col)
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 1/sqrt(32): the normalisation of the block-diagonal Sylvester H32.
constexpr float kInvSqrt32 = 0.17677669529663689f;

// In-register FWHT over 32 values, stage strides 1,2,4,8,16 then * 1/sqrt(32);
// v[j] <- a + b, v[j + s] <- a - b for each butterfly pair (Sylvester order).
__device__ __forceinline__ void fwht32_regs(float (&v)[32]) {
#pragma unroll
  for (int s = 1; s < 32; s <<= 1) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if ((j & s) == 0) {
        float a = v[j], b = v[j + s];
        v[j] = a + b;
        v[j + s] = a - b;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] *= kInvSqrt32;
}

// The same transform with one value per lane across a warp.
__device__ __forceinline__ float fwht32_lane(float v, int lane) {
#pragma unroll
  for (int s = 1; s < 32; s <<= 1) {
    float o = __shfl_xor_sync(0xffffffffu, v, s);
    v = (lane & s) ? (o - v) : (v + o);
  }
  return v * kInvSqrt32;
}

// SiLU with the fast exponential and division intrinsics: a few instructions
// instead of the full-precision library sequence, inlined in every prologue
// (relative error ~1e-6, far below the fp16 rounding that follows).
__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
  return v;
}

// ---------------------------------------------------------------------------
// FP8 E4M3 codec with the reference's rules (not IEEE E4M3FN, not CUDA's cvt):
//  * inputs are clamped to [-448, 448] first (NaN -> +448);
//  * magnitudes below 2^-6 (float exponent field 0 included) become signed 0;
//  * the mantissa is cut to 3 bits and rounded up when the first dropped bit is
//    set (ties away from zero), with carry into the exponent;
//  * an E4M3 exponent field >= 15 saturates to 0x7E (448) with the sign.
// Decoding composes sign | (e + 120) << 23 | m << 20 and maps |byte| == 0 to +0.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t fp8_encode(float x) {
  x = fmaxf(-448.0f, fminf(448.0f, x));
  const uint32_t f = __float_as_uint(x);
  const uint32_t sign = (f >> 24) & 0x80u;
  const int e32 = (int)((f >> 23) & 0xFFu);
  const uint32_t m32 = f & 0x7FFFFFu;
  int e = e32 - 120;
  uint32_t m = (m32 >> 20) + ((m32 >> 19) & 1u);
  e += (int)(m >> 3);        // mantissa overflow carries into the exponent
  m &= 7u;
  uint32_t r = sign | ((uint32_t)e << 3) | m;
  r = (e >= 15) ? (sign | 0x7Eu) : r;
  r = (e <= 0 || e32 == 0) ? sign : r;
  return r;
}

__device__ __forceinline__ float fp8_decode(uint32_t b) {
  const uint32_t f = ((b & 0x80u) << 24) | ((((b >> 3) & 0xFu) + 120u) << 23) | ((b & 7u) << 20);
  return (b & 0x7Fu) ? __uint_as_float(f) : 0.0f;
}

// Hardware pair conversion E4M3 -> f16x2.  Equal to fp8_decode on every byte
// the encoder above can emit (zeros, exponent fields 1..14, 0x7E/0xFE).
__device__ __forceinline__ uint32_t fp8x2_to_h2(uint16_t two) {
  uint32_t d;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(d) : "h"(two));
  return d;
}

}  // namespace r4q
