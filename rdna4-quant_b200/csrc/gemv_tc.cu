// Dequant-GEMV on the 5th-generation tensor cores for batches of 3..16 rows
// (INT4 weights).  y[b, n] = sum_k x'[b, k] * fp16((q[n, k] - z) * s), where
// x' is the activation after the prologue (H32 rotation, RMSNorm, SiLU*up).
//
// Status: opt-in (R4Q_GEMV_TC=1), parity-tested, slower than the mma.sync
// kernel and therefore not the default.  Measured on B200 (global-timer trace
// per stage, gate_up 5120 -> 34816 at B = 16): each 128 x 512 stage takes
// ~4 us, bound by the MMA lane (an M = 128, N = 16, K = 16 MMA with A in
// tensor memory costs ~90 cycles whatever N, 32 of them per stage, plus one
// commit per 64-k piece) and by the tensor-memory round trip of the
// dequantised operand; 1.3 TB/s against 1.7 TB/s for gemv_tma.cu.  The
// dequantised fp16 operand is 4x the nibble bytes, and with mma.sync it goes
// from registers straight into the tensor cores: that is why the GEMV stays on
// mma.sync at these batch sizes.
//
// Design (kept for measurement): with B > 2 the mma.sync kernel issues two
// m16n8k16 MMAs and four activation-fragment loads per 512 weights per 8
// batch columns, and every CTA re-applies the prologue to the activations.
// Here:
//  * a small kernel (xprep) applies the prologue once, writing x' [B, K] in the
//    k order the dequantised weights come out in (per 8 k: 0,4,1,5,2,6,3,7);
//  * the GEMV kernel is persistent, one CTA per SM, 22 warps:
//      warp 20 (one lane): TMA producer.  A stage is 128 rows x 512 k: the
//        nibbles (2 boxes of 128 B x 128 rows, 128-byte swizzle), the
//        (scale, zero) pairs (64 B x 128 rows, 64-byte swizzle) and the x'
//        tile (8 boxes of 64 k x 16 rows fp16, 128-byte swizzle = the K-major
//        operand layout of tcgen05; rows >= B are filled with zeros by TMA);
//        tiles visit their stages in a rotated order (stage_of) so that the
//        CTAs do not all read the same slice of x' at once;
//        14 tensor-memory A buffers rotate over the pieces (1.75 stages), so
//        a buffer is rewritten only well after the MMAs that read it;
//      warps 0-15 (four warpgroups): thread = weight row; each dequantises
//        64-k pieces of its row to the exact reference value fp16((q - z) s)
//        and writes them to tensor memory (tcgen05.st) as the MMA's A operand
//        (warpgroup g takes pieces g and g + 4 of every stage);
//      warp 21 (one lane): tcgen05.mma.kind::f16 M = 128, N = 16, K = 16,
//        A from tensor memory, B (x') from shared memory, fp32 accumulator in
//        tensor memory (two accumulators, so the epilogue of one unit
//        overlaps the MMAs of the next);
//      warps 16-19: epilogue, tcgen05.ld of the accumulator (thread = row,
//        16 columns), fp16 output with optional residual and per-16-row sums
//        of squares, or fp32 outputs, or split-K partials merged by the
//        tile's last CTA in split order (deterministic);
//  * every mbarrier wait is bounded; a timeout sets the workspace status word
//    and the kernel drains instead of hanging.  No multicast.
#include <cuda.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <unordered_map>

#include "gemv_dev.cuh"
#include "tma_dev.cuh"

namespace r4q {

int make_map_f16_rows(CUtensorMap* m, const void* base, long rows, long cols, int box_cols, int box_rows);

namespace {

constexpr int kRows = 128;                       // weight rows per tile (MMA M)
constexpr int kNB = 16;                          // batch columns per MMA (N)
constexpr int kSK = 512;                         // k per stage
constexpr int kPK = 64;                          // k per tensor-memory A buffer (a "piece")
constexpr int kPieces = kSK / kPK;               // 8
constexpr int kWBytes = kRows * kSK / 2;         // 32 KB of nibbles
constexpr int kSBytes = kRows * (kSK / 32) * 4;  // 8 KB of (scale, zero) pairs
constexpr int kXBytes = kNB * kSK * 2;           // 16 KB of activations
constexpr int kStage = kWBytes + kSBytes + kXBytes;
constexpr int kNS = 3;                           // ring depth
constexpr int kDeqWarps = 16;
constexpr int kProdWarp = 20, kMmaWarp = 21;
constexpr int kThreads = 22 * 32;
__device__ __forceinline__ int dcol(int d) { return d * 32; }  // accumulator d at column 32 d
constexpr int kAcol0 = 64;                       // A buffer b at kAcol0 + 32 b
constexpr int kABuf = 14;                        // A buffers (1.75 stages of pieces)
constexpr int kTmemCols = 512;
constexpr int kMaxSplit = 16;
constexpr int kEpiBar = 3;                       // named barrier of the epilogue warpgroup

// Instruction descriptor, kind::f16: fp32 accumulator, fp16 A and B, both
// K-major, N = 16, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | (uint32_t(kNB >> 3) << 17) | (uint32_t(kRows >> 4) << 24);

struct TcParams {
  const __half* xp;     // x' [B][K] (prologue applied, permuted per 8 k)
  __half* y;
  long ldy;
  int B, N, K;
  const __half* res;
  long ldres;
  float* ss_out;
  float* y32p[8];
  int npush;
  int* status;
  long spin;
  unsigned* cnt;        // per-tile arrival counters (left zero)
  float* part;          // [S][B][N]
  int S;                // K splits
  int gt;               // CTAs per split
  int tiles, nstages;
  int dbg;              // measurement only (R4Q_GEMV_TC_DBG): 1 skip the MMAs, 2 skip the tensor-memory stores
};

// K-major operand descriptor with 128-byte swizzle: rows of 128 bytes, 8-row
// groups 1024 bytes apart, descriptor version 1, layout type 2.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(kIdesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}

// Bounded wait that naps between polls: for waiters off the critical path
// (the epilogue waits a whole unit), so their polling takes few issue slots.
__device__ __forceinline__ bool mbar_wait_nap(uint64_t* b, unsigned parity, int* status, long limit) {
  for (long i = 0; i < limit; ++i) {
    if (mbar_try_wait(b, parity)) return true;
    __nanosleep(256);
  }
  if (status) atomicExch(status, 1);
  return false;
}

// Stage order inside a unit: tile t starts at stage (t mod nst) of its K
// range and wraps around, so CTAs working on different tiles at the same time
// read different slices of x' (all CTAs reading one 16 KB slice together
// serialise on the L2 slices that hold it).  The order is fixed per tile:
// results stay deterministic.
__device__ __forceinline__ int stage_of(int t, int j, int st0, int nst) {
  int k = j + t % nst;
  if (k >= nst) k -= nst;
  return st0 + k;
}

// Units: CTA (ks, c) of the grid takes K split ks of tiles c, c + gt, ...
struct Units {
  int tiles, gt, tile, st0, st1;
  __device__ __forceinline__ bool next(int& t) {
    if (tile >= tiles) return false;
    t = tile;
    tile += gt;
    return true;
  }
};

// ------------------------------------------------------------- x prep ----
// One thread per (column, 32-block): the prologue of the mma.sync kernel
// (same code, same rounding), written as fp16 with each 8-k group in the
// order 0,4,1,5,2,6,3,7 (the order deq_int4_word's register pairs carry).
template <int PRO>
__global__ void __launch_bounds__(128) xprep_kernel(const GemvParams p, __half* __restrict__ xp) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ float s_rrms;
  const int col = blockIdx.y, tid = threadIdx.x;
  if (PRO == R4Q_PRO_RMSNORM_FWHT && col < p.B) {
    if (tid < 32) {
      float ss = 0.0f;
      if (p.ss_in) {
        for (int i0 = tid; i0 < p.ss_in_parts; i0 += 256) {
          float tv[8];
#pragma unroll
          for (int u = 0; u < 8; ++u)
            tv[u] = (i0 + 32 * u < p.ss_in_parts) ? p.ss_in[(long)(i0 + 32 * u) * p.B + col] : 0.0f;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            if (i0 + 32 * u < p.ss_in_parts) ss += tv[u];
        }
      } else {
        const __half2* xr = reinterpret_cast<const __half2*>(p.x + (long)col * p.ldx);
        for (int i = tid; i < (p.K >> 1); i += 32) {
          const float2 f = __half22float2(xr[i]);
          ss += f.x * f.x + f.y * f.y;
        }
      }
      ss = warp_sum(ss);
      if (tid == 0) s_rrms = rsqrtf(ss / (float)p.K + p.eps);
    }
    __syncthreads();
  }
  const int blk = blockIdx.x * blockDim.x + tid;
  if (blk * 32 >= p.K) return;
  uint4* dst = reinterpret_cast<uint4*>(xp + (long)col * p.K + blk * 32);
  if (col >= p.B) {                                    // padding rows of the 16-row operand
#pragma unroll
    for (int m = 0; m < 4; ++m) dst[m] = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  __half v[32];
  load_block32_t<PRO>(p, col, blk * 32, PRO == R4Q_PRO_RMSNORM_FWHT ? s_rrms : 1.0f, v);
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const int b = 8 * m;
    __half t[8] = {v[b], v[b + 4], v[b + 1], v[b + 5], v[b + 2], v[b + 6], v[b + 3], v[b + 7]};
    dst[m] = *reinterpret_cast<const uint4*>(t);
  }
}

// ---------------------------------------------------------------- GEMV ----
template <bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
    gemv_tc_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tms,
                   const __grid_constant__ CUtensorMap tmx, const TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kNS * kStage);
  uint64_t* empty = full + kNS;
  uint64_t* afull = empty + kNS;        // [kABuf]
  uint64_t* aempty = afull + kABuf;     // [kABuf]
  uint64_t* dfull = aempty + kABuf;     // [2]
  uint64_t* dempty = dfull + 2;         // [2]
  uint64_t* mdone = dempty + 2;         // the MMA lane's last commit (drain before dealloc)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);
  int* s_last = reinterpret_cast<int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ks = blockIdx.x % p.S, c0 = blockIdx.x / p.S;
  const int st0 = (int)((long)ks * p.nstages / p.S), st1 = (int)((long)(ks + 1) * p.nstages / p.S);
  const int nst = st1 - st0;

  if (tid == 0) {
    for (int i = 0; i < kNS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kDeqWarps + 1);     // dequant warps + the MMA lane's commit
    }
    for (int i = 0; i < kABuf; ++i) {
      mbar_init(&afull[i], 4);                 // the four warps of the piece's warpgroup
      mbar_init(&aempty[i], 1);                // MMA commit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&dfull[i], 1);
      mbar_init(&dempty[i], 4);                // the epilogue warps
    }
    mbar_init(mdone, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProdWarp) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmw)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tms)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmx)) : "memory");
    }
    const uint64_t pol = l2_policy_evict_first();
    // weights of the first ring's stages go out before the previous kernel
    // (the prologue pass) completes; x' after it
    int it = 0;
    bool ok = true;
    {
      Units u{p.tiles, p.gt, c0, st0, st1};
      int t;
      while (it < kNS && u.next(t)) {
        for (int j = 0; j < nst && it < kNS; ++j, ++it) {
          const int st = stage_of(t, j, st0, nst);
          if (lane == 0) {
            mbar_expect_tx(&full[it], kStage);
            uint8_t* sb = smem + it * kStage;
            tma_load_2d_hint(sb, &tmw, st * (kSK / 2), t * kRows, &full[it], pol);
            tma_load_2d_hint(sb + kWBytes / 2, &tmw, st * (kSK / 2) + 128, t * kRows, &full[it], pol);
            tma_load_2d_hint(sb + kWBytes, &tms, st * (kSK / 8), t * kRows, &full[it], pol);
          }
        }
      }
    }
    const int pre = it;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    it = 0;
    Units u{p.tiles, p.gt, c0, st0, st1};
    int t;
    while (ok && u.next(t)) {
      for (int j = 0; j < nst && ok; ++j, ++it) {
        const int st = stage_of(t, j, st0, nst);
        const int slot = it % kNS;
        uint8_t* sb = smem + slot * kStage;
        if (it >= pre) {
          if (it >= kNS) ok = __all_sync(0xffffffffu, mbar_wait(&empty[slot], ((it / kNS) - 1) & 1, p.status, p.spin));
          if (!ok) break;
          if (lane == 0) {
            mbar_expect_tx(&full[slot], kStage);
            tma_load_2d_hint(sb, &tmw, st * (kSK / 2), t * kRows, &full[slot], pol);
            tma_load_2d_hint(sb + kWBytes / 2, &tmw, st * (kSK / 2) + 128, t * kRows, &full[slot], pol);
            tma_load_2d_hint(sb + kWBytes, &tms, st * (kSK / 8), t * kRows, &full[slot], pol);
          }
        }
        if (lane == 0) {
#pragma unroll
          for (int i = 0; i < kSK / 64; ++i)
            tma_load_2d(sb + kWBytes + kSBytes + i * (kNB * 128), &tmx, st * kSK + i * 64, 0, &full[slot]);
        }
      }
    }
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // drain: no copy may still be landing in shared memory when the CTA exits
    if (lane == 0)
      for (int j = (it > kNS ? it - kNS : 0); j < it; ++j) mbar_drain(&full[j % kNS], (unsigned)(j / kNS) & 1u, p.status);
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------- MMA
    // The whole warp follows the schedule and waits (so no lane of it sits at
    // the CTA barrier below while lane 0 works); lane 0 issues.
    bool ok = true;
    int it = 0, ui = 0;
    Units u{p.tiles, p.gt, c0, st0, st1};
    int t;
    while (u.next(t)) {
      const int d = ui & 1;
      if (ok && ui >= 2) ok = __all_sync(0xffffffffu, mbar_wait(&dempty[d], ((ui >> 1) - 1) & 1, p.status, p.spin));
      fence_after();
      for (int st = 0; st < nst; ++st, ++it) {
        const int slot = it % kNS;
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&full[slot], (it / kNS) & 1, p.status, p.spin));
        const uint32_t xs = smem_u32(smem + slot * kStage + kWBytes + kSBytes);
        for (int pc = 0; pc < kPieces; ++pc) {
          // piece number g = it * kPieces + pc uses buffer g % kABuf for the (g / kABuf)-th time
          const int gpc = it * kPieces + pc, ab = gpc % kABuf, use = gpc / kABuf;
          if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&afull[ab], use & 1, p.status, p.spin));
          fence_after();
          if (lane == 0) {
            if (ok && !(p.dbg & 1)) {
#pragma unroll
              for (int kk = 0; kk < kPK / 16; ++kk)
                mma_ts(tmem + dcol(d), tmem + kAcol0 + 32 * ab + 8 * kk, desc_sw128(xs + pc * (kNB * 128) + kk * 32),
                       (st | pc | kk) ? 1u : 0u);
            }
            mma_commit(&aempty[ab]);
          }
          __syncwarp();
        }
        if (lane == 0) mma_commit(&empty[slot]);
        __syncwarp();
      }
      if (lane == 0) mma_commit(&dfull[d]);
      __syncwarp();
      ++ui;
    }
    if (lane == 0) mma_commit(mdone);
    __syncwarp();
    mbar_drain(mdone, 0, p.status);
  } else if (warp < kDeqWarps) {
    // ---------------------------------------------------------- dequant
    const int wg = warp >> 2, q = warp & 3;
    const int r = 32 * q + lane;                       // row inside the tile
    const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16);
    bool ok = true;
    int it = 0;
    Units u{p.tiles, p.gt, c0, st0, st1};
    int t;
    while (u.next(t)) {
      for (int st = 0; st < nst; ++st, ++it) {
        const int slot = it % kNS;
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&full[slot], (it / kNS) & 1, p.status, p.spin));
        const uint32_t wb = smem_u32(smem + slot * kStage), sb = wb + kWBytes;
        // this warpgroup's pieces: wg and wg + 4
        uint4 raw[2][2];
        uint2 prs[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int pc = wg + 4 * h;
          const uint32_t box = wb + (pc >> 2) * (kWBytes / 2);
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int c = (pc & 3) * 2 + j;            // 16-byte chunk (one 32-k block) of the box row
            raw[h][j] = lds128(box + r * 128 + ((c ^ (r & 7)) << 4));
          }
          // pairs of blocks 2 pc, 2 pc + 1: 16-byte unit pc >> 1, bytes (pc & 1) * 8
          prs[h] = lds64(sb + r * 64 + ((((pc >> 1) ^ ((r >> 1) & 3))) << 4) + (pc & 1) * 8);
        }
        __syncwarp();
        if (lane == 0 && ok) mbar_arrive(&empty[slot]);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int pc = wg + 4 * h;
          uint32_t a[32];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const __half2 sz = u32_as_h2(j ? prs[h].y : prs[h].x);
            const __half2 z = __high2half2(sz), s = __low2half2(sz);
            const __half2 z1024 = __hadd2(z, __float2half2_rn(1024.0f));
            const __half2 nz64 = __hneg2(__hadd2(z, __float2half2_rn(64.0f)));
            const uint32_t w4[4] = {raw[h][j].x, raw[h][j].y, raw[h][j].z, raw[h][j].w};
#pragma unroll
            for (int m = 0; m < 4; ++m) {
              uint32_t o[4];
              deq_int4_word(w4[m], z1024, nz64, s, o);
#pragma unroll
              for (int i = 0; i < 4; ++i) a[16 * j + 4 * m + i] = o[i];
            }
          }
          // the buffer is free once the MMAs of its previous piece finished
          const int gpc = it * kPieces + pc, ab = gpc % kABuf, use = gpc / kABuf;
          if (ok && use >= 1) ok = __all_sync(0xffffffffu, mbar_wait(&aempty[ab], (use - 1) & 1, p.status, p.spin));
          if (ok && !(p.dbg & 2)) tmem_st32(trow + kAcol0 + 32 * ab, a);
          else if (p.dbg & 2) asm volatile("" ::"r"(a[0] ^ a[7] ^ a[15] ^ a[31]));
          fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&afull[ab]);
        }
      }
    }
  } else {
    // --------------------------------------------------------- epilogue
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int q = warp & 3;
    const int r = 32 * q + lane;
    const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16);
    bool ok = true;
    int ui = 0;
    Units u{p.tiles, p.gt, c0, st0, st1};
    int t;
    while (u.next(t)) {
      const int d = ui & 1;
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait_nap(&dfull[d], (ui >> 1) & 1, p.status, p.spin));
      fence_after();
      uint32_t v[16];
      if (ok) tmem_ld16(trow + dcol(d), v);
      else
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0u;
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dempty[d]);
      ++ui;
      const int row = t * kRows + r;
      float acc[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i] = __uint_as_float(v[i]);
      if constexpr (SPLIT) {
        // this split's partial; the tile's last CTA sums all splits in order
        if (row < p.N)
#pragma unroll
          for (int c = 0; c < kNB; ++c)
            if (c < p.B) p.part[((long)ks * p.B + c) * p.N + row] = acc[c];
        __threadfence();
        named_sync(kEpiBar, 128);
        if (r == 0) {
          unsigned old;
          asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(p.cnt + t * 8) : "memory");
          *s_last = (old == (unsigned)p.S - 1) ? 1 : 0;
        }
        named_sync(kEpiBar, 128);
        const int last = *s_last;
        named_sync(kEpiBar, 128);                      // s_last is read before the next tile rewrites it
        if (!last) continue;
        __threadfence();
        if (row < p.N) {
#pragma unroll
          for (int c = 0; c < kNB; ++c) acc[c] = 0.0f;
          for (int j0 = 0; j0 < p.S; j0 += 2) {        // two splits' loads in flight, summed in order
            float tv[2][kNB];
#pragma unroll
            for (int jj = 0; jj < 2; ++jj)
#pragma unroll
              for (int c = 0; c < kNB; ++c)
                tv[jj][c] = (j0 + jj < p.S && c < p.B) ? __ldcg(p.part + ((long)(j0 + jj) * p.B + c) * p.N + row) : 0.0f;
#pragma unroll
            for (int jj = 0; jj < 2; ++jj)
              if (j0 + jj < p.S)
#pragma unroll
                for (int c = 0; c < kNB; ++c) acc[c] += tv[jj][c];
          }
        }
        if (r == 0) p.cnt[t * 8] = 0u;
      }
      // outputs: fp32 pushes, or fp16 (+ residual, + sums of squares per 16 rows)
      const bool inr = row < p.N;
      if (p.npush) {
        if (inr)
          for (int qq = 0; qq < p.npush; ++qq)
#pragma unroll
            for (int c = 0; c < kNB; ++c)
              if (c < p.B) p.y32p[qq][(long)c * p.ldy + row] = acc[c];
      } else {
#pragma unroll
        for (int c = 0; c < kNB; ++c) {
          float o = 0.0f;
          if (c < p.B && inr) {
            o = __half2float(__float2half(acc[c]));
            if (p.res) o += __half2float(p.res[(long)c * p.ldres + row]);
            p.y[(long)c * p.ldy + row] = __float2half(o);
          }
          if (p.ss_out) {
            float sq = o * o;
            sq += __shfl_xor_sync(0xffffffffu, sq, 1);
            sq += __shfl_xor_sync(0xffffffffu, sq, 2);
            sq += __shfl_xor_sync(0xffffffffu, sq, 4);
            sq += __shfl_xor_sync(0xffffffffu, sq, 8);
            if ((lane & 15) == 0 && c < p.B && inr) p.ss_out[(long)(row >> 4) * p.B + c] = sq;
          }
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ----------------------------------------------------------------- host ---
size_t tc_smem() { return 1024 + (size_t)kNS * kStage + (2 * kNS + 2 * kABuf + 5) * 8 + 16; }

bool set_smem_once() {
  static std::mutex mu;
  static std::unordered_map<int, bool> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  auto f = done.find(dev);
  if (f != done.end()) return f->second;
  const int sm = (int)tc_smem();
  const bool ok = cudaFuncSetAttribute(gemv_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm) ==
                      cudaSuccess &&
                  cudaFuncSetAttribute(gemv_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm) ==
                      cudaSuccess;
  cudaGetLastError();
  done[dev] = ok;
  return ok;
}

struct TcPlan {
  int S, gt;
};

// Units = (128-row tile, K split).  Minimise the busiest CTA's stages plus one
// stage per split-K merge; the partials and x' must fit the workspace.
TcPlan plan(int B, int N, int K, size_t room) {
  const int nsm = num_sms();
  const int tiles = (N + kRows - 1) / kRows;
  const int nst = (K + kSK - 1) / kSK;
  TcPlan best{0, 0};
  double best_cost = 1e30;
  static const int forced = [] {
    const char* e = getenv("R4Q_GEMV_TC_SPLIT");
    return e ? atoi(e) : 0;
  }();
  for (int S = 1; S <= kMaxSplit && S <= nst; ++S) {
    if (forced > 0 && S != forced && forced <= nst) continue;
    const int gt = nsm / S;
    if (gt < 1) break;
    if (S > 1 && (size_t)S * B * N * sizeof(float) > room) break;
    const int use = gt < tiles ? gt : tiles;
    const int rounds = (tiles + use - 1) / use;
    const int per = (nst + S - 1) / S;
    const double cost = (double)rounds * per + (S > 1 ? 1.0 * rounds : 0.0) + 0.01 * S;
    if (cost < best_cost) {
      best_cost = cost;
      best = TcPlan{S, use};
    }
  }
  return best;
}

template <int PRO>
cudaError_t launch_xprep(const GemvParams& gp, __half* xp, cudaStream_t st) {
  const int nblk = gp.K / 32;
  return launch_pdl(xprep_kernel<PRO>, dim3((nblk + 127) / 128, gp.B), dim3(128), 0, st, gp, xp);
}

}  // namespace

// x' region of the workspace: the last 16 * K * 2 bytes (rows >= B zero), 256-byte aligned.
static size_t xprep_bytes(int B, int K) {
  (void)B;
  return ((size_t)kNB * K * 2 + 255) / 256 * 256;
}

size_t gemv_tc_extra_bytes(int B, int K) { return xprep_bytes(B, K) + 256; }

bool gemv_tc_eligible(const GemvArgs& a, int fmt) {
  static const int mode = [] {
    const char* e = getenv("R4Q_GEMV_TC");
    return e ? atoi(e) : 0;
  }();
  if (mode == 0) return false;
  return fmt == W_INT4 && a.B >= 3 && a.B <= kNB && a.K % 128 == 0 && aligned(a.s, 16) && a.ws &&
         !a.tpx.nwait && !a.tpx.nsig && !a.tpx.ll_sig;
}

int launch_gemv_tc(const GemvArgs& a) {
  const size_t hdr = gemv_cnt_bytes(a.N);
  const size_t xb = xprep_bytes(a.B, a.K);
  if (a.ws_bytes < hdr + xb + 256) return R4Q_ERR_CAPACITY;
  const size_t xoff = (a.ws_bytes - xb) / 256 * 256;
  if (xoff < hdr) return R4Q_ERR_CAPACITY;
  const TcPlan pl = plan(a.B, a.N, a.K, xoff - hdr);
  if (pl.S < 1) return R4Q_ERR_CAPACITY;
  if (!set_smem_once()) return R4Q_ERR_CAPACITY;
  __half* xp = reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(a.ws) + xoff);

  CUtensorMap tmw, tms, tmx;
  int st = make_map(&tmw, a.w, a.N, a.K / 2, 128, kRows, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!st) st = make_map(&tms, a.s, a.N, a.K / 8, 64, kRows, CU_TENSOR_MAP_SWIZZLE_64B);
  if (!st) st = make_map_f16_rows(&tmx, xp, a.B, a.K, 64, kNB);
  if (st) return st;

  GemvParams gp{};
  gp.x = reinterpret_cast<const __half*>(a.x);
  gp.ldx = a.ldx;
  gp.B = a.B; gp.N = a.N; gp.K = a.K;
  gp.prologue = a.prologue;
  gp.norm_w = reinterpret_cast<const __half*>(a.norm_w);
  gp.eps = a.eps;
  gp.ss_in = a.ss_in;
  gp.ss_in_parts = a.ss_in_parts;
  cudaError_t e;
  switch (a.prologue) {
    case R4Q_PRO_FWHT: e = launch_xprep<R4Q_PRO_FWHT>(gp, xp, a.stream); break;
    case R4Q_PRO_SILU_FWHT: e = launch_xprep<R4Q_PRO_SILU_FWHT>(gp, xp, a.stream); break;
    case R4Q_PRO_RMSNORM_FWHT: e = launch_xprep<R4Q_PRO_RMSNORM_FWHT>(gp, xp, a.stream); break;
    default: e = launch_xprep<R4Q_PRO_NONE>(gp, xp, a.stream); break;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(R4Q_ERR_CUDA, "gemv_tc xprep: %s", cudaGetErrorString(e));
  }

  TcParams p{};
  p.xp = xp;
  p.y = reinterpret_cast<__half*>(a.y);
  p.ldy = a.ldy;
  p.B = a.B; p.N = a.N; p.K = a.K;
  p.res = reinterpret_cast<const __half*>(a.res);
  p.ldres = a.ldres;
  p.ss_out = a.ss_out;
  p.npush = a.npush;
  for (int i = 0; i < 8; ++i) p.y32p[i] = i < a.npush ? a.y32p[i] : nullptr;
  p.status = reinterpret_cast<int*>(a.ws);
  p.spin = gemv_spin_limit();
  p.cnt = gemv_counters(a.ws);
  p.part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(a.ws) + hdr);
  p.S = pl.S;
  p.gt = pl.gt;
  p.tiles = (a.N + kRows - 1) / kRows;
  p.nstages = (a.K + kSK - 1) / kSK;
  {
    static const int dbg = [] {
      const char* e = getenv("R4Q_GEMV_TC_DBG");
      return e ? atoi(e) : 0;
    }();
    p.dbg = dbg;
  }
  e = pl.S > 1 ? launch_pdl(gemv_tc_kernel<true>, dim3(pl.S * pl.gt), dim3(kThreads), tc_smem(), a.stream, tmw, tms,
                            tmx, p)
               : launch_pdl(gemv_tc_kernel<false>, dim3(pl.S * pl.gt), dim3(kThreads), tc_smem(), a.stream, tmw, tms,
                            tmx, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(R4Q_ERR_CUDA, "gemv_tc_kernel: %s", cudaGetErrorString(e));
  }
  return R4Q_OK;
}

// 2-D fp16 tensor map [rows, cols] (row-major), box [box_rows, box_cols],
// 128-byte swizzle; rows past `rows` read as zeros.
int make_map_f16_rows(CUtensorMap* m, const void* base, long rows, long cols, int box_cols, int box_rows) {
  typedef CUresult (*Fn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                         const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                         CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static Fn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<Fn>(f);
  });
  if (!fn) return set_error(R4Q_ERR_CUDA, "gemv_tc: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(R4Q_ERR_CUDA, "gemv_tc: tensor map encode failed (%d)", (int)r);
  return R4Q_OK;
}

}  // namespace r4q
