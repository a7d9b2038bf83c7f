// Device helpers shared by the TMA-fed GEMV kernels: mbarriers, bulk tensor
// loads, 32-bit shared-space loads, named barriers and the row order that
// makes the swizzled 16-byte reads conflict-free.
#pragma once
#include <cuda.h>
#include <stdint.h>

#include "gemv.cuh"

namespace r4q {

constexpr long kSpinLimit = 1L << 26;   // polls before a bounded wait gives up

// A stage (group) is a tile of rows x SK k: CPS 16-byte chunks per row in
// BOXES 128-byte TMA boxes, plus SBYTES of scales per row.
template <int FMT> struct TmaFmt;
template <> struct TmaFmt<W_INT4> {
  static constexpr int SK = 1024;        // k per stage
  static constexpr int CPS = 32;         // 16-byte chunks per row per stage
  static constexpr int BOXES = 4;        // 128-byte weight boxes per row per stage
  static constexpr int SBYTES = 128;     // (scale, zero) bytes per row per stage
  static constexpr int NS = 4;           // maximum ring depth
};
template <> struct TmaFmt<W_INT8> {
  static constexpr int SK = 512, CPS = 32, BOXES = 4, SBYTES = 32, NS = 4;
};
template <> struct TmaFmt<W_FP16> {
  static constexpr int SK = 256, CPS = 32, BOXES = 4, SBYTES = 0, NS = 4;
};


// ------------------------------------------------------------ mbarrier ---
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after `limit` polls, records the failure and
// returns false so the kernel can drain and exit instead of hanging.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, unsigned parity, int* status, long limit) {
  for (long i = 0; i < limit; ++i)
    if (mbar_try_wait(b, parity)) return true;
  if (status) atomicExch(status, 1);
  return false;
}

// L2 cache policy for data read exactly once (streamed weights).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Drain wait (producer lane at exit): try_wait lets the hardware suspend the
// lane between polls, so it takes no issue slots from the consumers.
__device__ __forceinline__ void mbar_drain(uint64_t* b, unsigned parity, int* status) {
  for (long i = 0; i < kSpinLimit; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    if (ok) return;
  }
  if (status) atomicExch(status, 1);
}

__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}


// Shared-space loads on 32-bit addresses (volatile: they must stay after the
// mbarrier wait that publishes the data).
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ float2 lds_f2(uint32_t a) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
  return v;
}

__device__ __forceinline__ void named_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void named_arrive(int id, int n) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Row order inside a 16-row m-tile: rows read by the same quarter-warp
// (groups 2q, 2q+1) differ in bit 2, so the 128-byte swizzle maps their
// chunks to disjoint banks.
__device__ __forceinline__ int row_perm(int g) { return ((g & 1) << 2) | (g >> 1); }


}  // namespace r4q
