// Prefill / batched GEMM on the 5th-generation tensor cores (tcgen05).
//
// Replaces the prefill projections of the reference, which dequantise the
// INT4 weights to fp16 (dequant_int4, int4_decode_step.hip:1973-1988, 3568-3603)
// and call rocBLAS (int4_prefill_logits, :2127-2320; int4_engine_v5.py:
// 214-266):  Y[M, N] = X[M, K] · W[N, K]ᵀ, fp16 in, fp32 accumulate, fp16 out.
//
// B200 design (one 128 x 256 output tile per CTA, 16 warps):
//  * warp 0, one lane: TMA producer.  X tiles [128 x 64] (4-stage ring) and
//    W tiles [256 x 64] (3-stage ring; fp16, K-major, 128-byte swizzle) with
//    mbarrier transaction counts; the activation ring is deeper so that the
//    L2 latency of the X tiles does not throttle the MMAs;
//  * INT4 weights (`w4` set): warps 2-15 dequantise instead of TMA-loading W
//    (fourteen warps: with six the dequantisation, not the MMA, set the pace):
//    the nibbles come in by TMA, the (scale, zero) pairs by the producer warp's
//    cp.async (8 bytes per row and stage, below TMA's 16-byte box minimum),
//    both completing on one mbarrier, in a ring of their own six stages deep
//    (refilled as soon as the dequantisers have read a slot, so the HBM
//    latency of the weights hides behind six stages of MMAs); the exact
//    reference value fp16((q - z) · s) is written into the swizzled fp16 slot
//    of the MMA ring, then fence.proxy.async makes it visible to the tensor
//    cores;
//  * warp 1, one lane: issues tcgen05.mma.cta_group::1.kind::f16 (M = 128,
//    N = 256, K = 16 per instruction, 4 per stage) from shared-memory matrix
//    descriptors into a 128 x 256 fp32 accumulator in tensor memory, and
//    tcgen05.commit releases each stage back to the producer;
//  * all 16 warps: epilogue, tcgen05.ld of their 32 accumulator lanes (= rows)
//    and a quarter of the columns, fp16 conversion, stores.
// Decode-sized M (few output tiles): the K range is split over gridDim.z so
// the grid covers the SMs; each split writes an fp32 partial and the tile's
// last CTA to arrive sums them in split order (deterministic).
// Every mbarrier wait is bounded; a timeout sets the status word and the
// kernel drains.  No multicast anywhere.
#include <cuda.h>

#include <cstdlib>
#include <mutex>

#include "r4q_common.cuh"

namespace r4q {
namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kStages = 3;                         // W (fp16) ring: TMA-filled, or the dequantisers' target
constexpr int kXS = 4;                             // activation ring (A operand), deeper than the W ring
constexpr int kNW = 5;                             // INT4: nibble/pair ring (runs ahead of the MMAs)
constexpr int kABytes = kBM * kBK * 2;             // 16 KB
constexpr int kBBytes = kBN * kBK * 2;             // 32 KB
constexpr int kW4Bytes = kBN * kBK / 2;            // 8 KB of nibbles per stage
constexpr int kPairBytes = kBN * 8;                // (scale, zero) of 2 blocks per row per stage
constexpr int kGemmThreads = 512;   // 16 warps: producer, MMA issuer, 14 dequantisers (INT4)
constexpr int kDequantThreads = kGemmThreads - 64;
constexpr long kGemmSpin = 1L << 26;

struct GemmParams {
  const uint8_t* sz;   // INT4: (scale, zero) fp16 pairs [N][K/16]
  __half* y;
  long ldy;
  int M, N, K;
  int w4;          // 1: W is INT4 (nibbles + pairs), dequantised in the kernel
  int* status;
  int splits;      // K splits (gridDim.z); > 1: fp32 partials merged by the tile's last CTA
  unsigned* cnt;   // [tiles] arrival counters (left zero)
  float* part;     // [splits][M][N] fp32 partials
};

__device__ __forceinline__ uint32_t sm_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void g_mbar_init(uint64_t* b, unsigned n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sm_u32(b)), "r"(n));
}
__device__ __forceinline__ void g_expect_tx(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sm_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void g_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sm_u32(b)) : "memory");
}
__device__ __forceinline__ bool g_wait(uint64_t* b, unsigned parity, int* status) {
  const uint32_t a = sm_u32(b);
  for (long i = 0; i < kGemmSpin; ++i) {
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                 " selp.u32 %0, 1, 0, p;\n}\n" : "=r"(ok) : "r"(a), "r"(parity) : "memory");
    if (ok) return true;
  }
  if (status) atomicExch(status, 1);
  return false;
}
__device__ __forceinline__ void g_tma2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(sm_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(sm_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows of 128
// bytes (64 fp16), 8-row groups 1024 bytes apart (stride byte offset), no
// leading byte offset, descriptor version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor of kind::f16: fp32 accumulator, fp16 A and B, both
// K-major, N = 256, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | (uint32_t(kBN >> 3) << 17) | (uint32_t(kBM >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t tmem, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
      ::"r"(tmem), "l"(da), "l"(db), "r"(kIdesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(sm_u32(bar))
               : "memory");
}

// One INT4 stage: 256 rows x 64 k.  Nibbles [256][32 B] (plain TMA box) and
// the rows' (scale, zero) pairs of blocks 2 kt, 2 kt + 1 ([256][8 B], brought
// in by the producer warp's cp.async; zero past N) -> fp16 in the 128-byte swizzled K-major layout TMA would have
// produced: element (r, k) at r * 128 + (((k >> 3) ^ (r & 7)) << 4) + (k & 7) * 2.
// The dequant threads take (row, 8-k chunk) items.  Exact reference value:
// OR-ing a nibble into 0x6400 gives the fp16 1024 + q; subtracting the fp16
// 1024 + z is exact (both integers below 2048), and the one fp16 multiply by s
// rounds (q - z) · s once, as dequantize_int4_asym does.  Rows past N get
// zero pairs.
__device__ __forceinline__ void dequant_stage(const uint8_t* w4, const uint8_t* pairs, uint8_t* bdst, int t,
                                              int nthr) {
  constexpr int kItems = (kBN * 8 + kDequantThreads - 1) / kDequantThreads;
  uint32_t wqs[kItems], prs[kItems];
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    const int item = t + i * nthr;
    const int r = item >> 3, c = item & 7;
    wqs[i] = 0u;
    prs[i] = 0u;
    if (item < kBN * 8) {
      wqs[i] = *reinterpret_cast<const uint32_t*>(w4 + r * 32 + c * 4);
      prs[i] = *reinterpret_cast<const uint32_t*>(pairs + r * 8 + (c >> 2) * 4);
    }
  }
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    const int item = t + i * nthr;
    if (item >= kBN * 8) break;
    const int r = item >> 3, c = item & 7;               // chunk c: k = 8c .. 8c+7
    const uint32_t wq = wqs[i];
    const uint32_t pair = prs[i];
    const __half2 szh = u32_as_h2(pair);
    const __half2 s2 = __half2half2(__low2half(szh));
    const __half2 z2 = __hadd2(__half2half2(__high2half(szh)), __float2half2_rn(1024.0f));
    // (k0, k4), (k1, k5), (k2, k6), (k3, k7) as 1024 + q
    const __half2 a = __hmul2(__hsub2(u32_as_h2(lop3_and_or(wq, 0x000F000Fu, 0x64006400u)), z2), s2);
    const __half2 b = __hmul2(__hsub2(u32_as_h2(lop3_and_or(wq >> 4, 0x000F000Fu, 0x64006400u)), z2), s2);
    const __half2 cc = __hmul2(__hsub2(u32_as_h2(lop3_and_or(wq >> 8, 0x000F000Fu, 0x64006400u)), z2), s2);
    const __half2 d = __hmul2(__hsub2(u32_as_h2(lop3_and_or(wq >> 12, 0x000F000Fu, 0x64006400u)), z2), s2);
    const uint4 o = make_uint4(h2_as_u32(__lows2half2(a, b)), h2_as_u32(__lows2half2(cc, d)),
                               h2_as_u32(__highs2half2(a, b)), h2_as_u32(__highs2half2(cc, d)));
    *reinterpret_cast<uint4*>(bdst + r * 128 + ((c ^ (r & 7)) << 4)) = o;
  }
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb,
                   const GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;                                        // [kXS][16 KB] activations
  uint8_t* sb = sa + kXS * kABytes;                          // [kStages][32 KB] fp16 W
  uint8_t* sw4 = sb + kStages * kBBytes;                     // [kNW][8 KB]  INT4 nibbles
  uint8_t* spr = sw4 + kNW * kW4Bytes;                       // [kNW][2 KB]  INT4 (scale, zero) pairs
  uint64_t* xfull = reinterpret_cast<uint64_t*>(spr + kNW * kPairBytes);  // [kXS]
  uint64_t* xempty = xfull + kXS;                            // [kXS] MMA commit
  uint64_t* full = xempty + kXS;                             // [kStages] fp16 W landed (TMA)
  uint64_t* empty = full + kStages;                          // [kStages] MMA commit
  uint64_t* w4full = empty + kStages;                        // [kNW] INT4 bytes landed
  uint64_t* w4empty = w4full + kNW;                          // [kNW] INT4 bytes read by the dequantisers
  uint64_t* bready = w4empty + kNW;                          // [kStages] dequantised W ready
  uint64_t* accum = bready + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  int& s_last = *reinterpret_cast<int*>(tmem_slot + 1);      // split-K: this CTA merges

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kBN, m0 = blockIdx.y * kBM;
  const int KTT = (p.K + kBK - 1) / kBK;
  const int kz = blockIdx.z;
  const int kt0 = (int)((long)kz * KTT / p.splits), KT = (int)((long)(kz + 1) * KTT / p.splits) - kt0;

  if (tid == 0) {
    for (int s = 0; s < kXS; ++s) {
      g_mbar_init(&xfull[s], 1);
      g_mbar_init(&xempty[s], 1);
    }
    for (int s = 0; s < kStages; ++s) {
      g_mbar_init(&full[s], 1);
      g_mbar_init(&empty[s], 1);
      g_mbar_init(&bready[s], kDequantThreads);
    }
    for (int s = 0; s < kNW; ++s) {
      g_mbar_init(&w4full[s], 33);               // TMA arrival + 32 lanes' cp.async
      g_mbar_init(&w4empty[s], kDequantThreads / 32);
    }
    g_mbar_init(accum, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sm_u32(tmem_slot)),
                 "r"(kBN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- producer: lane 0 issues the TMA loads; for INT4 all 32 lanes copy
    //      the stage's (scale, zero) pairs (8 bytes per row, below TMA's
    //      16-byte box minimum) with cp.async, whose completion arrives on
    //      the same mbarrier as the nibbles
    // Three rings: activations (kXS deep), fp16 W (kStages; TMA-filled, or
    // written by the dequantisers), and for INT4 the nibbles and (scale,
    // zero) pairs of stage j in slot j % kNW, kNW stages ahead of the MMAs
    // (refilled as soon as the dequantisers have read a slot).
    auto issue_w4 = [&](int j) {
      const int n = j % kNW, kt = kt0 + j;
      if (lane == 0) {
        g_expect_tx(&w4full[n], kW4Bytes);
        g_tma2d(sw4 + n * kW4Bytes, &tmb, kt * (kBK / 2), n0, &w4full[n]);
      }
      for (int r = lane; r < kBN; r += 32) {
        const bool in = n0 + r < p.N;
        const uint8_t* src = p.sz + (in ? (long)(n0 + r) * (p.K / 8) + kt * 8 : 0);
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(sm_u32(spr + n * kPairBytes + r * 8)),
                     "l"(src), "r"(in ? 8 : 0) : "memory");
      }
      asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(sm_u32(&w4full[n])) : "memory");
    };
    bool ok = true;
    if (p.w4)
      for (int j = 0; j < KT && j < kNW; ++j) issue_w4(j);
    for (int i = 0; i < KT && ok; ++i) {                // i: stage of this CTA's K range
      const int kt = kt0 + i, xs = i % kXS, s = i % kStages;
      // activations: kXS stages ahead of the MMAs
      if (i >= kXS) ok = g_wait(&xempty[xs], ((i / kXS) - 1) & 1, p.status);
      if (!ok) break;
      if (lane == 0) {
        g_expect_tx(&xfull[xs], kABytes);
        g_tma2d(sa + xs * kABytes, &tma, kt * kBK, m0, &xfull[xs]);
      }
      if (p.w4) {
        // refill the nibble slot stage i - 1 used, for stage i - 1 + kNW
        const int j = i - 1 + kNW;
        if (i >= 1 && j < KT) {
          ok = g_wait(&w4empty[(i - 1) % kNW], ((i - 1) / kNW) & 1, p.status);
          if (!ok) break;
          issue_w4(j);
        }
      } else {
        if (i >= kStages) ok = g_wait(&empty[s], ((i / kStages) - 1) & 1, p.status);
        if (!ok) break;
        if (lane == 0) {
          g_expect_tx(&full[s], kBBytes);
          g_tma2d(sb + s * kBBytes, &tmb, kt * kBK, n0, &full[s]);
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer
    bool ok = true;
    for (int i = 0; i < KT; ++i) {
      const int s = i % kStages, xs = i % kXS;
      if (ok) ok = g_wait(&xfull[xs], (i / kXS) & 1, p.status);
      if (ok) ok = g_wait(p.w4 ? &bready[s] : &full[s], (i / kStages) & 1, p.status);
      asm volatile("tcgen05.fence::after_thread_sync;");
      if (ok) {
        const uint32_t a0 = sm_u32(sa + xs * kABytes), b0 = sm_u32(sb + s * kBBytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          umma_f16(tmem, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), (i | kk) ? 1u : 0u);
      }
      umma_commit(&xempty[xs]);             // the slots are free once these MMAs have read them
      umma_commit(&empty[s]);
    }
    umma_commit(accum);
  } else if (warp >= 2 && p.w4) {
    // ---- INT4 dequantisers (warps 2-15)
    const int t = tid - 64;
    bool ok = true;
    for (int i = 0; i < KT; ++i) {
      const int s = i % kStages, n = i % kNW;
      if (ok) ok = g_wait(&w4full[n], (i / kNW) & 1, p.status);
      // the fp16 slot was last read by the MMAs of stage i - kStages
      if (ok && i >= kStages) ok = g_wait(&empty[s], ((i / kStages) - 1) & 1, p.status);
      if (ok) dequant_stage(sw4 + n * kW4Bytes, spr + n * kPairBytes, sb + s * kBBytes, t, kDequantThreads);
      __syncwarp();
      if (lane == 0) g_arrive(&w4empty[n]);             // nibble slot n may be refilled
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      g_arrive(&bready[s]);
    }
  }

  // ---- epilogue: warp w owns accumulator lanes (rows) 32 (w % 4) .. + 31
  //      and columns 128 (w / 4) .. + 127
  __syncwarp();
  const bool ok = g_wait(accum, 0, p.status);
  asm volatile("tcgen05.fence::after_thread_sync;");
  constexpr int kColGroups = kGemmThreads / 128;             // warps sharing a lane quarter
  const int quarter = warp & 3, half = warp >> 2;
  const int row = m0 + quarter * 32 + lane;
#pragma unroll 1
  for (int c0 = half * (kBN / kColGroups); c0 < (half + 1) * (kBN / kColGroups); c0 += 32) {
    uint32_t v[32];
    const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0;
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    if (!ok || row >= p.M) continue;
    const int nvalid = min(32, p.N - (n0 + c0));
    if (p.splits > 1) {                                 // this K split's fp32 partial
      float* pr = p.part + ((long)kz * p.M + row) * p.N + n0 + c0;
      if (nvalid == 32 && (p.N % 4) == 0) {
#pragma unroll
        for (int q = 0; q < 8; ++q)
          reinterpret_cast<float4*>(pr)[q] = make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                                         __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
      } else {
        for (int j = 0; j < nvalid; ++j) pr[j] = __uint_as_float(v[j]);
      }
      continue;
    }
    __half* yr = p.y + (long)row * p.ldy + n0 + c0;
    if (nvalid == 32 && (p.ldy % 8) == 0 && (reinterpret_cast<uintptr_t>(p.y) & 15) == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 o;
        o.x = h2_as_u32(__floats2half2_rn(__uint_as_float(v[8 * q]), __uint_as_float(v[8 * q + 1])));
        o.y = h2_as_u32(__floats2half2_rn(__uint_as_float(v[8 * q + 2]), __uint_as_float(v[8 * q + 3])));
        o.z = h2_as_u32(__floats2half2_rn(__uint_as_float(v[8 * q + 4]), __uint_as_float(v[8 * q + 5])));
        o.w = h2_as_u32(__floats2half2_rn(__uint_as_float(v[8 * q + 6]), __uint_as_float(v[8 * q + 7])));
        reinterpret_cast<uint4*>(yr)[q] = o;
      }
    } else {
      for (int j = 0; j < nvalid; ++j) yr[j] = __float2half(__uint_as_float(v[j]));
    }
  }
  if (p.splits > 1) {
    // the last CTA of the tile to arrive sums the partials in split order
    // (deterministic) and writes fp16; it leaves the counter zero
    const int tile = blockIdx.y * gridDim.x + blockIdx.x;
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&p.cnt[tile], 1u) == (unsigned)p.splits - 1u);
    __syncthreads();
    if (s_last) {
      __threadfence();
      // coalesced: 256 threads = 4 rows x 64 float4 columns per pass
      const int rows = min(kBM, p.M - m0), cols = min(kBN, p.N - n0);
      const bool vec = (p.N % 4) == 0 && (p.ldy % 4) == 0 && (reinterpret_cast<uintptr_t>(p.y) & 7) == 0;
      if (ok)
        for (int r = tid >> 6; r < rows; r += kGemmThreads / 64) {
          const int c = (tid & 63) * 4;
          if (c >= cols) continue;
          const long prow = (long)(m0 + r) * p.N + n0 + c;
          __half* yr = p.y + (long)(m0 + r) * p.ldy + n0 + c;
          if (vec && c + 4 <= cols) {
            float4 a4 = __ldcg(reinterpret_cast<const float4*>(p.part + prow));
            for (int q = 1; q < p.splits; ++q) {
              const float4 b4 = __ldcg(reinterpret_cast<const float4*>(p.part + (long)q * p.M * p.N + prow));
              a4.x += b4.x; a4.y += b4.y; a4.z += b4.z; a4.w += b4.w;
            }
            uint2 o;
            o.x = h2_as_u32(__floats2half2_rn(a4.x, a4.y));
            o.y = h2_as_u32(__floats2half2_rn(a4.z, a4.w));
            *reinterpret_cast<uint2*>(yr) = o;
          } else {
            for (int j = 0; j < 4 && c + j < cols; ++j) {
              float v = 0.0f;
              for (int q = 0; q < p.splits; ++q) v += __ldcg(p.part + (long)q * p.M * p.N + prow + j);
              yr[j] = __float2half(v);
            }
          }
        }
      if (tid == 0) p.cnt[tile] = 0u;
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 2) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kBN));
}

typedef CUresult (*EncodeTiledFnG)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFnG encode_g() {
  static EncodeTiledFnG fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFnG>(f);
  });
  return fn;
}

// 2-D map over [rows, cols] elements of `esize` bytes, row stride ld elements.
int map2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int esize, long rows, long cols, long ld,
          int box_cols, int box_rows, CUtensorMapSwizzle sw) {
  EncodeTiledFnG fn = encode_g();
  if (!fn) return set_error(R4Q_ERR_CUDA, "gemm: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * esize)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(R4Q_ERR_CUDA, "gemm: tensor map encode failed (%d)", (int)r);
  return R4Q_OK;
}

size_t gemm_smem() {
  return 1024 + (size_t)kXS * kABytes + (size_t)kStages * kBBytes + (size_t)kNW * (kW4Bytes + kPairBytes) +
         (2 * kXS + 3 * kStages + 2 * kNW + 1) * 8 + 16;
}

// Workspace: status word at 0, tile counters from byte 256 (split grids have
// at most kMaxSplitTiles tiles), fp32 partials from byte kPartOffset.
constexpr int kMaxSplitTiles = 1024;
constexpr size_t kPartOffset = 256 + kMaxSplitTiles * 4;

// K splits: enough CTAs to cover the SMs once when the output has few tiles
// (decode-sized M), at least 4 k-tiles per split, within the workspace.
// R4Q_GEMM_SPLIT forces the split count (measurement only).
int gemm_splits(int M, int N, int K, size_t ws_bytes) {
  const int tiles = ((N + kBN - 1) / kBN) * ((M + kBM - 1) / kBM);
  const int KT = (K + kBK - 1) / kBK;
  static const int forced = [] {
    const char* e = getenv("R4Q_GEMM_SPLIT");
    return e ? atoi(e) : 0;
  }();
  int S = forced > 0 ? (forced < KT ? forced : KT) : num_sms() / tiles;
  if (forced > 0) {
    if (tiles > kMaxSplitTiles) S = 1;
    while (S > 1 && kPartOffset + (size_t)S * M * N * 4 > ws_bytes) --S;
    return S;
  }
  if (S > KT / 4) S = KT / 4;
  if (S > 16) S = 16;
  if (tiles > kMaxSplitTiles) S = 1;
  while (S > 1 && kPartOffset + (size_t)S * M * N * 4 > ws_bytes) --S;
  return S < 1 ? 1 : S;
}

int launch_gemm(const void* x, long ldx, const void* w, const void* s, void* y, long ldy, int M, int N, int K,
                int w4, void* ws, size_t ws_bytes, cudaStream_t st) {
  CUtensorMap ta, tb;
  int rc = map2d(&ta, x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, M, K, ldx, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (w4) {
    // nibbles [N, K/2] bytes, box 32 B x 256 rows (plain layout)
    rc = map2d(&tb, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, K / 2, K / 2, kBK / 2, kBN, CU_TENSOR_MAP_SWIZZLE_NONE);
  } else {
    rc = map2d(&tb, w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, N, K, K, kBK, kBN, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (rc) return rc;
  GemmParams p{};
  p.sz = (const uint8_t*)s;
  p.y = (__half*)y;
  p.ldy = ldy;
  p.M = M;
  p.N = N;
  p.K = K;
  p.w4 = w4;
  p.status = (int*)ws;
  p.splits = gemm_splits(M, N, K, ws_bytes);
  p.cnt = reinterpret_cast<unsigned*>(reinterpret_cast<uint8_t*>(ws) + 256);
  p.part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + kPartOffset);
  const size_t smem = gemm_smem();
  static std::mutex mu;
  static bool done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 64 && !done[dev]) {
      cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      cudaGetLastError();
      done[dev] = true;
    }
  }
  dim3 grid((N + kBN - 1) / kBN, (M + kBM - 1) / kBM, p.splits);
  gemm_tc_kernel<<<grid, kGemmThreads, smem, st>>>(ta, tb, p);
  return check_launch("gemm_tc_kernel");
}

}  // namespace
}  // namespace r4q

using namespace r4q;

extern "C" int r4q_gemm_fp16(const void* x, long ldx, const void* w, void* y, long ldy, int M, int N, int K,
                             void* ws, size_t ws_bytes, void* stream) {
  if (!x || !w || !y || M < 1 || N < 1 || K < 1) return set_error(R4Q_ERR_ARG, "gemm_fp16: bad arguments");
  if (K % 8 || ldx % 8 || ldx < K || ldy < N || !aligned(x, 16) || !aligned(w, 16) || !aligned(y, 2))
    return set_error(R4Q_ERR_ALIGN, "gemm_fp16: K, ldx multiples of 8 and 16-byte aligned x, w required");
  if (!ws || ws_bytes < 4 || !aligned(ws, 16))
    return set_error(R4Q_ERR_CAPACITY, "gemm_fp16: 16-byte aligned workspace (status word) required");
  return launch_gemm(x, ldx, w, nullptr, y, ldy, M, N, K, 0, ws, ws_bytes, (cudaStream_t)stream);
}

extern "C" int r4q_gemm_int4(const void* x, long ldx, const void* w, const void* sz, void* y, long ldy, int M,
                             int N, int K, void* ws, size_t ws_bytes, void* stream) {
  if (!x || !w || !sz || !y || M < 1 || N < 1 || K < 1) return set_error(R4Q_ERR_ARG, "gemm_int4: bad arguments");
  if (K % 64 || ldx % 8 || ldx < K || ldy < N || !aligned(x, 16) || !aligned(w, 16) || !aligned(sz, 16) ||
      !aligned(y, 2))
    return set_error(R4Q_ERR_ALIGN, "gemm_int4: K % 64 == 0, ldx % 8 == 0 and 16-byte aligned x, w, sz required");
  if (!ws || ws_bytes < 4 || !aligned(ws, 16))
    return set_error(R4Q_ERR_CAPACITY, "gemm_int4: 16-byte aligned workspace (status word) required");
  return launch_gemm(x, ldx, w, sz, y, ldy, M, N, K, 1, ws, ws_bytes, (cudaStream_t)stream);
}

extern "C" size_t r4q_gemm_workspace_bytes(int M, int N, int K) {
  if (M < 1 || N < 1 || K < 1) return 256;
  const int S = gemm_splits(M, N, K, (size_t)-1);
  return S > 1 ? kPartOffset + (size_t)S * M * N * 4 : 256;
}
