// Dequant-GEMV, TMA path (the default when the shape allows it).
//
// Persistent, warp-specialised kernel, one CTA per SM:
//  * warp 16 (producer): one lane streams the CTA's weight tiles — 64 rows x
//    512 k per stage for INT4 — and their (scale, zero) tiles into a
//    shared-memory ring (~120 KB) with cp.async.bulk.tensor (TMA) and mbarrier
//    transaction counts.  Weights are read from HBM exactly once and no
//    register holds data in flight.  Each row contributes >= 256 contiguous
//    bytes per stage: with 128 bytes per row per stage the TMA stream alone
//    stalls near 4.2 TB/s on B200; with 256-512 bytes it reaches the roofline;
//  * warps 0-15 (consumers): warp (m-tile, k quarter) takes 16 rows x 1/4 of
//    each stage's k, reads its 16-byte chunks with conflict-free LDS.128
//    (128-byte TMA swizzle + a row order in which rows sharing a quarter-warp
//    differ in bit 2), dequantises in registers into m16n8k16 A fragments,
//    releases the ring slot, then accumulates in fp32 on the tensor cores
//    (two independent accumulator chains) against the activations staged
//    once per CTA;
//  * units = (64-row tile, K split); each CTA owns one K split (activations are
//    staged once) and a strided set of tiles; split partials merge in the
//    last-arriving CTA of a tile (deterministic order);
//  * programmatic dependent launch: the producer starts streaming weights
//    before griddepcontrol.wait; everything that reads the previous kernel's
//    outputs (activations, sums of squares, residual) comes after it.
#include <cuda.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <unordered_map>

#include "gemv_dev.cuh"
#include "tma_dev.cuh"

namespace r4q {

constexpr int kTmaConsumers = 16;
constexpr int kTmaThreads = (kTmaConsumers + 1) * 32;
constexpr int kTileRows = 64;
constexpr int kTmaMaxSplit = 32;
constexpr int kTpPre = 3;      // staging items per thread held in registers by a TP consumer
constexpr int kStageBatch = 2; // staging rounds whose loads are in flight together
constexpr int kStagedBar = 10; // named barrier (1: consumers, 2-9: m groups): activations staged (consumers arrive, producer waits)
constexpr int kPrewait = 4;    // ring stages requested before the previous kernel completes

#ifdef R4Q_TRACE
// Development-only event trace (compiled only with -DR4Q_TRACE): per launch
// slot (eight consecutive launches), event, CTA: a global-timer stamp.
// Events: 0 CTA start, 1 griddepcontrol.wait returned, 2 activations
// staged, 3 first stage landed, 4 consumers done, 5 producer issued all,
// 6 RMSNorm scale known (staging starts), 7 first staging batch stored.
__device__ unsigned long long g_trace[8][8][256];
__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ int g_dbg_mode;  // 1: consumers only wait/release, 2: dequant without MMA
#define TRACE(slot, idx) do { if (blockIdx.x < 256) g_trace[tp.trace_par][(slot)][blockIdx.x] = gtime(); } while (0)
#define DBG_MODE g_dbg_mode
#else
#define TRACE(slot, idx) do {} while (0)
#define DBG_MODE 0
#endif  // bounded mbarrier waits (seconds of wall time)

struct TmaParams {
  GemvParams p;
  int nstages;     // stages over the whole K
  int tiles;       // 64-row tiles
  int gt;          // CTAs per K split
  int x_bytes;     // activation smem bytes
  int xsum_bytes;  // per-block activation sums (block-diagonal path)
  int ns;          // ring depth (stages), sized to the shared memory left
  int* status;     // set to 1 when a bounded wait gives up
  long spin;       // polls before a wait gives up (kSpinLimit unless lowered for a test)
  int trace_par;   // R4Q_TRACE builds: trace buffer of this launch
  int prewait;     // stages the producer requests before the previous kernel completes
};


// Floats of the k-part reduction buffer: 4 m-tiles x (P - 1) writer parts x
// NG column groups x 4 accumulators x 32 lanes (P = 8 on the block-diagonal
// path, whose warps own two m-tiles, else 4).
template <int NG, bool DIAG>
__host__ __device__ constexpr int red_floats() { return 4 * ((DIAG ? 8 : 4) - 1) * NG * 4 * 32; }  // >= any MPW's need

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kTmaConsumers * 32) : "memory");
}

// ------------------------------------------------------- work schedule ---
// A unit is a run of stages [sb, se) of one 64-row tile; contributor j of the
// n CTAs (K splits) that share the tile (n == 1: the whole tile).
struct Seg {
  int tile, sb, se, j, n;
};

// CTA (ks, c) of a K-split grid takes tiles c, c + gt, c + 2 gt, ... so that
// at any time all SMs stream neighbouring tiles.
struct SegIter {
  int tiles, gt, tile, st0, st1, ks, S;
  __device__ __forceinline__ bool next(Seg& sg) {
    if (tile >= tiles) return false;
    sg = Seg{tile, st0, st1, ks, S};
    tile += gt;
    return true;
  }
};

// ------------------------------------------------------------- kernel ----
// DIAG (INT4, B <= 2): activation column n of every MMA is (block 2n.., batch
// n & 1): lane (g, t) feeds its activations only for column g when g >> 1 == t,
// zeros otherwise, so the accumulator holds one partial sum per (row, block,
// batch).  The MMA then runs on raw biased nibbles (1024 + q for even k,
// 64 + q for odd k: one LOP3 per pair, no subtract, no scale multiply) and the
// bias, zero point and scale are applied once per block in fp32:
//   sum_k (q - z) x = C - (1024 X_even + 64 X_odd) - z X,  times s.
// PRO (the activation prologue), TPC (tensor-parallel consumer: the prologue
// reads the exchange slots) and SPLIT (K split over CTAs, merged through the
// workspace) are compile-time so that each instance carries only the code it
// runs: the kernel's once-per-CTA paths (staging, epilogue) are otherwise
// large enough to stall warps on instruction fetch (measured: 7.8 stalls per
// issue on o_proj with every variant in one instance, 0.9 without).
template <int FMT, int NG, bool DIAG, int PRO, bool TPC, bool SPLIT>
__global__ void __launch_bounds__(kTmaThreads, 1)
    gemv_tma_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tms,
                    const TmaParams tp) {
  using T = TmaFmt<FMT>;
  using F = Fmt<FMT>;
  constexpr int W_STAGE = kTileRows * T::CPS * 16;     // bytes of weights per stage
  constexpr int S_STAGE = kTileRows * T::SBYTES;
  const int NS = tp.ns;
  constexpr int V = T::CPS / 16;                       // chunks per thread per row per stage
  constexpr int NM = ChunkMma<FMT>::N;
  const GemvParams& p = tp.p;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring_w = smem;
  uint8_t* ring_s = ring_w + NS * W_STAGE;
  uint8_t* xs = ring_s + NS * S_STAGE;
  float2* xsum = reinterpret_cast<float2*>(xs + tp.x_bytes);        // [B][chunks] (X, E)
  uint8_t* zero16 = xs + tp.x_bytes + tp.xsum_bytes;
  float* red = reinterpret_cast<float*>(zero16 + 16);               // [4 m-tiles][P-1][NG*4][32]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + red_floats<NG, DIAG>());
  uint64_t* empty = full + NS;
  __shared__ float s_rrms[16];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = p.ksplit;
  const int ks = blockIdx.x % S;
  const int cta_in_split = blockIdx.x / S;
  const int st0 = (int)((long)ks * tp.nstages / S);
  const int st1 = (int)((long)(ks + 1) * tp.nstages / S);
  const int nst = st1 - st0;
  SegIter iter0{tp.tiles, tp.gt, cta_in_split, st0, st1, ks, S};

  if (tid == 0) TRACE(0, 0);
  if (tid == 0 && blockIdx.x == 0 && (p.tpx.nsig || p.tpx.ll_sig)) tp_stamp(p.tpx, 5, p.tpx.sig_idx);
  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kTmaConsumers);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  // ------------------------------------------------------------ producer
  if (warp == kTmaConsumers) {
    // The whole warp runs the schedule (its lanes poll together, so `ok`
    // stays warp-uniform); lane 0 issues the copies.
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmw)) : "memory");
      if (T::SBYTES) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tms)) : "memory");
    }
    // weights are read once: evict-first in L2, so the stream does not push
    // out the activations, norm weights and sums of squares the next kernels
    // read right after their griddepcontrol.wait
    const uint64_t l2_stream = l2_policy_evict_first();
    int it = 0;
    bool ok = true, held = false;
    SegIter iter = iter0;
    Seg sg;
    while (ok && iter.next(sg)) {
      const int tile = sg.tile;
      for (int st = sg.sb; st < sg.se && ok; ++st, ++it) {
        const int slot = it % NS;
        const unsigned ph = (unsigned)(it / NS) & 1u;
        if (it == tp.prewait) {
          // Only `prewait` stages go out before the previous kernel is done;
          // the rest wait until the consumers have staged the activations, so
          // those loads do not queue behind a full ring of weight requests
          // (with every SM's ring in flight, any new request waits ~3-4 us).
          asm volatile("griddepcontrol.wait;" ::: "memory");
          named_sync(kStagedBar, kTmaThreads);
          held = true;
        }
        if (it >= NS) ok = __all_sync(0xffffffffu, mbar_wait(&empty[slot], ph ^ 1u, tp.status, tp.spin));
        if (!ok) break;
        if (lane == 0) {
          const bool load_s = T::SBYTES && DBG_MODE != 3;
          mbar_expect_tx(&full[slot], W_STAGE + (load_s ? S_STAGE : 0));
#pragma unroll
          for (int b = 0; b < T::BOXES; ++b)
            tma_load_2d_hint(ring_w + slot * W_STAGE + b * (kTileRows * 128), &tmw,
                             st * (T::CPS * 16) + b * 128, tile * kTileRows, &full[slot], l2_stream);
          if (load_s)
            tma_load_2d_hint(ring_s + slot * S_STAGE, &tms, st * T::SBYTES, tile * kTileRows, &full[slot],
                             l2_stream);
        }
      }
    }
    if (lane == 0) TRACE(5, 0);
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (!held) named_sync(kStagedBar, kTmaThreads);   // the consumers arrive once in every case
    // Drain: the CTA must not exit while a copy into its shared memory is in
    // flight.  Consumers that gave up on a wait stop releasing slots (so no
    // slot is ever refilled before its previous copy landed); here the last
    // copy issued into each slot is awaited.  Copies complete on their own
    // within microseconds, so this wait keeps the full limit.
    if (lane == 0)
      for (int j = (it > NS ? it - NS : 0); j < it; ++j)
        mbar_drain(&full[j % NS], (unsigned)(j / NS) & 1u, tp.status);
    return;
  }

  // ------------------------------------------------------------ consumers
  // everything below may read outputs of the previous kernel in the stream
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (tid == 0) TRACE(1, 0);
  const int ctid = tid;  // 0 .. kTmaConsumers*32-1
  const int ncolx = p.B;
  const int nch_pad = nst * T::CPS;
  const int colstride = tp.x_bytes / (ncolx > 0 ? ncolx : 1);

  const bool stamp = blockIdx.x == 0 && ctid == 0;
  if (stamp && (p.tpx.nsig || p.tpx.ll_sig)) tp_stamp(p.tpx, 0, p.tpx.sig_idx);
  // tag of this GEMV's pushed words (the step counter is read after the wait)
  const unsigned ll_tag = p.tpx.ll_sig ? (unsigned)tp_epoch(p.tpx, p.tpx.sig_idx) : 0u;
  // TP consumer with the whole K staged here and at most kTpPre staging items
  // per thread: read the exchange buffer once (see below)
  const int tp_nblk = nch_pad * F::CK / 32;
  const int tp_items = ncolx * tp_nblk * 4;
  const bool tp_one = TPC && DIAG && st0 == 0 && nst == tp.nstages &&
                      tp_items <= kTmaConsumers * 32 * kTpPre;
  uint4 tp_raw[kTpPre];
  if constexpr (TPC) {
    // tensor-parallel consumer: wait for every rank's partials, then r and
    // its sum of squares straight from the exchange buffer (CTA 0 stores r)
    if (stamp) tp_stamp(p.tpx, 2, p.tpx.wait_idx);
    if (warp == 0 && !p.tpx.ll_wait) tp_wait_lane(p.tpx, lane);   // tagged words: the reads wait
    consumer_sync();
    if (stamp) tp_stamp(p.tpx, 3, p.tpx.wait_idx);
    __shared__ float s_ssp[kTmaConsumers][16];
    if (tp_one) {
      // one pass (whole K staged, B <= 2): every thread reads its staging
      // items' r values once, keeps them in registers for the staging below
      // and accumulates the sums of squares
      float ssc[2] = {0.0f, 0.0f};
#pragma unroll
      for (int r = 0; r < kTpPre; ++r) {
        const int item = warp * 32 + lane + r * (kTmaConsumers * 32);
        tp_raw[r] = make_uint4(0, 0, 0, 0);
        if (item < tp_items) {
          const int qq = item & 3, cb = item >> 2;
          const int col = cb / tp_nblk, blk = cb - col * tp_nblk;
          const int k = blk * 32 + qq * 8;
          if (k < p.K) {
            float ss = 0.0f;
            tp_raw[r] = tp_row8_ss(p, col, k, ss);
            if (col) ssc[1] += ss;
            else ssc[0] += ss;
            if (blockIdx.x == 0 && p.tpx.red_out)
              *reinterpret_cast<uint4*>(p.tpx.red_out + (long)col * p.K + k) = tp_raw[r];
          }
        }
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const float ss = warp_sum(ssc[c]);
        if (lane == 0 && c < ncolx) s_ssp[warp][c] = ss;
      }
    } else
    // every consumer thread takes 4 consecutive k of every column; partial
    // sums of squares per (warp, column) meet in shared memory
    for (int c = 0; c < ncolx; ++c) {
      const float* rb = p.tpx.red + (long)c * p.K;
      const __half* hr = p.tpx.red_res + (long)c * p.K;
      __half* ro = (blockIdx.x == 0 && p.tpx.red_out) ? p.tpx.red_out + (long)c * p.K : nullptr;
      float ss = 0.0f;
      for (int k = ctid * 4; k < p.K; k += kTmaConsumers * 128) {
        float4 a;
        if (p.tpx.ll_wait) {
          const unsigned tag = (unsigned)tp_epoch(p.tpx, p.tpx.wait_idx);
          float t4[4];
          for (int s2 = 0; s2 < p.tpx.nwait; ++s2) {
            const long i0 = (long)s2 * p.tpx.red_slot + (long)c * p.K + k;
            const ulonglong2* w2 =
                reinterpret_cast<const ulonglong2*>(reinterpret_cast<const unsigned long long*>(p.tpx.red) + i0);
            const ulonglong2 v0 = __ldcg(w2), v1 = __ldcg(w2 + 1);
            const unsigned long long w[4] = {v0.x, v0.y, v1.x, v1.y};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float f = (unsigned)(w[j] >> 32) == tag ? __uint_as_float((unsigned)w[j])
                                                             : tp_read_word(p.tpx, p.tpx.red, i0 + j, tag, s2);
              t4[j] = s2 == 0 ? f : t4[j] + f;
            }
          }
          a = make_float4(t4[0], t4[1], t4[2], t4[3]);
        } else {
          a = __ldcg(reinterpret_cast<const float4*>(rb + k));
          for (int s2 = 1; s2 < p.tpx.nwait; ++s2) {
            const float4 b = __ldcg(reinterpret_cast<const float4*>(rb + s2 * p.tpx.red_slot + k));
            a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
          }
        }
        const uint2 rr = *reinterpret_cast<const uint2*>(hr + k);
        const __half* h4 = reinterpret_cast<const __half*>(&rr);
        const float a4[4] = {a.x, a.y, a.z, a.w};
        __half o4[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float v = __half2float(__float2half(a4[j])) + __half2float(h4[j]);
          ss += v * v;
          o4[j] = __float2half(v);
        }
        if (ro) *reinterpret_cast<uint2*>(ro + k) = *reinterpret_cast<const uint2*>(o4);
      }
      ss = warp_sum(ss);
      if (lane == 0) s_ssp[warp][c] = ss;
    }
    consumer_sync();
    if (warp == 0 && lane < ncolx) {
      float ss = 0.0f;
      for (int w2 = 0; w2 < kTmaConsumers; ++w2) ss += s_ssp[w2][lane];
      s_rrms[lane] = rsqrtf(ss / (float)p.K + p.eps);
    }
    consumer_sync();
  }
  if constexpr (!TPC) {
    // One thread per (column, 32-block): the RMSNorm scale first, then each
    // thread loads its 32 activations (one memory round trip), applies the
    // prologue and the FWHT in registers (the butterfly order of the
    // reference, no shuffles) and writes the block into the permuted layout.
    if constexpr (PRO == R4Q_PRO_RMSNORM_FWHT) {
      for (int c = warp; c < ncolx; c += kTmaConsumers) {
        float ss = 0.0f;
        if (p.ss_in) {
          // eight loads in flight per lane, summed in index order
          for (int i0 = lane; i0 < p.ss_in_parts; i0 += 256) {
            float tv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
              tv[u] = (i0 + 32 * u < p.ss_in_parts) ? p.ss_in[(long)(i0 + 32 * u) * ncolx + c] : 0.0f;
#pragma unroll
            for (int u = 0; u < 8; ++u)
              if (i0 + 32 * u < p.ss_in_parts) ss += tv[u];
          }
        } else {
          const __half2* xr = reinterpret_cast<const __half2*>(p.x + (long)c * p.ldx);
          for (int i = lane; i < (p.K >> 1); i += 32) {
            const float2 f = __half22float2(xr[i]);
            ss += f.x * f.x + f.y * f.y;
          }
        }
        ss = warp_sum(ss);
        if (lane == 0) s_rrms[c] = rsqrtf(ss / (float)p.K + p.eps);
      }
      consumer_sync();
      if (ctid == 0) TRACE(6, 0);
    }
    const int nblk = nch_pad * F::CK / 32;
    const int k_base = st0 * T::SK;
    const int total = ncolx * nblk;
    for (int item = ctid; item < total; item += kTmaConsumers * 32) {
      const int col = item / nblk, blk = item - col * nblk;
      __half v[32];
      load_block32_t<PRO>(p, col, k_base + blk * 32, PRO == R4Q_PRO_RMSNORM_FWHT ? s_rrms[col] : 1.0f, v);
      if constexpr (DIAG) {
        // block sums of the even and odd k, added in the order of the
        // 4-lane form: per quarter in k order, then (q0 + q1) + (q2 + q3)
        float se[4], so[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          se[q] = 0.0f;
          so[q] = 0.0f;
#pragma unroll
          for (int jj = 0; jj < 8; jj += 2) {
            se[q] += __half2float(v[8 * q + jj]);
            so[q] += __half2float(v[8 * q + jj + 1]);
          }
        }
        const float e = (se[0] + se[1]) + (se[2] + se[3]);
        const float o = (so[0] + so[1]) + (so[2] + so[3]);
        xsum[col * nch_pad + blk] = make_float2(e + o, 1024.0f * e + 64.0f * o);
      }
      store_block32<FMT>(xs + (long)col * colstride, nch_pad, blk, v);
    }
    if (ctid == 0) TRACE(7, 0);
    if (ctid < 4) reinterpret_cast<uint32_t*>(zero16)[ctid] = 0u;
  } else
  {
    // (column, block, quarter) items, round r of thread t = item
    // t + r * 512; the loads of up to kStageBatch rounds are issued before
    // any of them is used, so staging costs one memory round trip per batch
    const int nblk = nch_pad * F::CK / 32;
    const int k_base = st0 * T::SK;
    const int total = ncolx * nblk * 4;
    const int nthr = kTmaConsumers * 32;
    const int rounds = (total + nthr - 1) / nthr;
    for (int r0 = 0; r0 < rounds; r0 += kStageBatch) {
      QuadIn in[kStageBatch];
#pragma unroll
      for (int j = 0; j < kStageBatch; ++j) {
        const int item = (r0 + j) * nthr + ctid;
        const bool valid = r0 + j < rounds && item < total;
        const int it2 = valid ? item : 0;
        const int q = it2 & 3, cb = it2 >> 2;
        const int col = cb / nblk, blk = cb - col * nblk;
        uint4 raw_in = make_uint4(0, 0, 0, 0);
        if (tp_one) {
#pragma unroll
          for (int r = 0; r < kTpPre; ++r)
            if (r == r0 + j) raw_in = tp_raw[r];
        }
        in[j] = stage_load(p, col, k_base + blk * 32, q, valid, tp_one, raw_in);
      }
#pragma unroll
      for (int j = 0; j < kStageBatch; ++j) {
        if (r0 + j >= rounds) break;                       // warp-uniform
        const int item = (r0 + j) * nthr + ctid;
        const bool valid = item < total;
        const int it2 = valid ? item : 0;
        const int q = it2 & 3, cb = it2 >> 2;
        const int col = cb / nblk, blk = cb - col * nblk;
        stage_finish<FMT, DIAG>(p, in[j], k_base + blk * 32, q,
                                p.prologue == R4Q_PRO_RMSNORM_FWHT ? s_rrms[col] : 1.0f,
                                xs + (long)col * colstride, nch_pad, blk, valid, xsum + col * nch_pad + blk);
      }
    }
    if (ctid < 4) reinterpret_cast<uint32_t*>(zero16)[ctid] = 0u;
  }
  consumer_sync();
  named_arrive(kStagedBar, kTmaThreads);                  // releases the rest of the ring
  if (ctid == 0) TRACE(2, 0);
  if (stamp && p.tpx.nwait) tp_stamp(p.tpx, 4, p.tpx.wait_idx);

  // warp -> (m group, k part); every stage is consumed by all 16 warps.  A
  // warp owns MPW m-tiles of 16 rows and 1/P of each stage's chunks; with
  // MPW = 2 (block-diagonal path) one activation fragment feeds the MMAs of
  // two m-tiles, halving the shared-memory reads of activations.
  constexpr int MPW = 1;                                    // m-tiles per warp
  constexpr int NGRP = 4 / MPW;                             // m groups per stage
  constexpr int P = kTmaConsumers / NGRP;                   // k parts
  constexpr int SPT = T::CPS / P;                           // chunks per part per row per stage
  constexpr int VV = SPT / 4;                               // chunks per lane per row per stage
  static_assert(VV >= 1, "too many k parts");
  const int g = lane >> 2, t = lane & 3;
  const int mgrp = warp % NGRP, part = warp / NGRP;
  int ra[MPW], rb[MPW];                                     // rows inside the 64-row tile
#pragma unroll
  for (int mi = 0; mi < MPW; ++mi) {
    ra[mi] = (mgrp * MPW + mi) * 16 + row_perm(g);
    rb[mi] = ra[mi] + 8;
  }
  int colx[NG];
#pragma unroll
  for (int cg = 0; cg < NG; ++cg) colx[cg] = min(cg * 8 + g, p.B - 1);
  // block-diagonal path: this lane feeds column g (= block g>>1, batch g&1)
  const bool feed = ((g >> 1) == t) && ((g & 1) < p.B);
  const uint8_t* xfeed = feed ? xs + (long)(g & 1) * colstride : nullptr;

  // Stage-invariant shared-memory offsets of this thread's chunks (the stage
  // slot base is added per stage).  Chunk c of row r sits in 128-byte box
  // c >> 3 at 16-byte unit (c & 7) ^ (r & 7) (128-byte swizzle).
  int offA[MPW][VV], offB[MPW][VV], soffA[MPW][VV], soffB[MPW][VV], cidx[VV];
#pragma unroll
  for (int v = 0; v < VV; ++v) {
    const int c = part * SPT + 4 * v + t;
    cidx[v] = c;
    const int box = c >> 3, cb = c & 7;
#pragma unroll
    for (int mi = 0; mi < MPW; ++mi) {
      const int a = ra[mi], b = rb[mi];
      offA[mi][v] = box * (kTileRows * 128) + a * 128 + ((cb ^ (a & 7)) << 4);
      offB[mi][v] = box * (kTileRows * 128) + b * 128 + ((cb ^ (b & 7)) << 4);
      if constexpr (FMT == W_INT4) {
        // 128-byte scale rows, 128-byte swizzle: (scale, zero) of block c
        soffA[mi][v] = a * 128 + (((c >> 2) ^ (a & 7)) << 4) + (c & 3) * 4;
        soffB[mi][v] = b * 128 + (((c >> 2) ^ (b & 7)) << 4) + (c & 3) * 4;
      } else if constexpr (FMT == W_INT8) {
        // 32-byte scale rows, 32-byte swizzle: fp16 scale of block c >> 1
        const int bk = c >> 1;
        soffA[mi][v] = a * 32 + (((bk >> 3) ^ ((a >> 2) & 1)) << 4) + (bk & 7) * 2;
        soffB[mi][v] = b * 32 + (((bk >> 3) ^ ((b >> 2) & 1)) << 4) + (bk & 7) * 2;
      } else {
        soffA[mi][v] = soffB[mi][v] = 0;
      }
    }
  }
  // activation pointers (block-diagonal path: lanes that feed nothing read a
  // 16-byte zero line with zero strides)
  const uint32_t xbase = DIAG ? (feed ? smem_u32(xfeed) + cidx[0] * 16 : smem_u32(zero16)) : 0u;
  const uint32_t xsub = DIAG ? (feed ? nch_pad * 16 : 0) : nch_pad * 16;   // bytes between sub-rows
  const uint32_t xstep = DIAG ? (feed ? T::CPS * 16 : 0) : T::CPS * 16;    // bytes per stage
  uint32_t xrow[NG];
#pragma unroll
  for (int cg = 0; cg < NG; ++cg) xrow[cg] = smem_u32(xs) + colx[cg] * colstride;
  const uint32_t ring_w_u = smem_u32(ring_w), ring_s_u = smem_u32(ring_s);
  const uint32_t xsum0 = smem_u32(xsum) + cidx[0] * 8, xsum1 = xsum0 + nch_pad * 8;

  int slot = 0;
  unsigned phase = 0;
  bool ok = true;
  int uidx = 0;
  SegIter iter = iter0;
  Seg sg;
  bool more = iter.next(sg);
  while (more) {
    const Seg cur = sg;
    more = iter.next(sg);                                   // is there a next unit?
    const int tile = cur.tile;
    float acc[MPW][NG][2][4];
#pragma unroll
    for (int mi = 0; mi < MPW; ++mi)
#pragma unroll
      for (int cg = 0; cg < NG; ++cg)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[mi][cg][h][i] = 0.0f;

    for (int st = cur.sb - st0; st < cur.se - st0; ++st) {  // st: stage index inside the staged x
      // warp-uniform: after a timeout the warp no longer waits and no longer
      // releases slots (the producer then stops refilling them and drains)
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&full[slot], phase, tp.status, tp.spin));
#ifdef R4Q_TRACE
      if (ctid == 0 && uidx == 0 && st == cur.sb - st0) TRACE(3, 0);
#endif
      const uint32_t wst = ring_w_u + slot * W_STAGE;
      const uint32_t sst = ring_s_u + slot * S_STAGE;
      uint64_t* emp = &empty[slot];
      if (++slot == NS) {
        slot = 0;
        phase ^= 1u;
      }
      if (DBG_MODE == 1) {
        __syncwarp();
        if (lane == 0 && ok) mbar_arrive(emp);
        continue;
      }
      if constexpr (DIAG) {
        uint4 wa[MPW][VV], wb[MPW][VV];
        uint32_t sza[MPW][VV], szb[MPW][VV];
#pragma unroll
        for (int mi = 0; mi < MPW; ++mi)
#pragma unroll
          for (int v = 0; v < VV; ++v) {
            wa[mi][v] = lds128(wst + offA[mi][v]);
            wb[mi][v] = lds128(wst + offB[mi][v]);
            sza[mi][v] = lds32(sst + soffA[mi][v]);
            szb[mi][v] = lds32(sst + soffB[mi][v]);
          }
        __syncwarp();
        if (lane == 0 && ok) mbar_arrive(emp);
        const uint32_t xst = xbase + st * xstep;
#pragma unroll
        for (int v = 0; v < VV; ++v) {
          const uint32_t xv = xst + (feed ? 4 * v * 16 : 0);
          float c0[MPW][4], c1[MPW][4];
#pragma unroll
          for (int mi = 0; mi < MPW; ++mi)
#pragma unroll
            for (int i = 0; i < 4; ++i) c0[mi][i] = c1[mi][i] = 0.0f;
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const uint4 xf = lds128(xv + m * xsub);
#pragma unroll
            for (int mi = 0; mi < MPW; ++mi) {
              const uint32_t wam = m == 0 ? wa[mi][v].x : m == 1 ? wa[mi][v].y : m == 2 ? wa[mi][v].z : wa[mi][v].w;
              const uint32_t wbm = m == 0 ? wb[mi][v].x : m == 1 ? wb[mi][v].y : m == 2 ? wb[mi][v].z : wb[mi][v].w;
              const uint32_t a8 = wam >> 8, b8 = wbm >> 8;
              const uint32_t alo = lop3_and_or(wam, 0x000F000Fu, 0x64006400u);
              const uint32_t ahi = lop3_and_or(wam, 0x00F000F0u, 0x54005400u);
              const uint32_t blo = lop3_and_or(wbm, 0x000F000Fu, 0x64006400u);
              const uint32_t bhi = lop3_and_or(wbm, 0x00F000F0u, 0x54005400u);
              const uint32_t alo2 = lop3_and_or(a8, 0x000F000Fu, 0x64006400u);
              const uint32_t ahi2 = lop3_and_or(a8, 0x00F000F0u, 0x54005400u);
              const uint32_t blo2 = lop3_and_or(b8, 0x000F000Fu, 0x64006400u);
              const uint32_t bhi2 = lop3_and_or(b8, 0x00F000F0u, 0x54005400u);
              mma16816(c0[mi], alo, blo, ahi, bhi, xf.x, xf.y);
              mma16816(c1[mi], alo2, blo2, ahi2, bhi2, xf.z, xf.w);
            }
          }
          // accumulator column 2t + b = (block of lane t, batch b)
          const uint32_t xso = (st * T::CPS + 4 * v) * 8;
          const float2 xe0 = lds_f2(xsum0 + xso);
          const float2 xe1 = p.B > 1 ? lds_f2(xsum1 + xso) : make_float2(0.f, 0.f);
#pragma unroll
          for (int mi = 0; mi < MPW; ++mi) {
            const float2 fa = __half22float2(u32_as_h2(sza[mi][v])), fb = __half22float2(u32_as_h2(szb[mi][v]));
            acc[mi][0][0][0] += fa.x * ((c0[mi][0] + c1[mi][0]) - fmaf(fa.y, xe0.x, xe0.y));
            acc[mi][0][0][2] += fb.x * ((c0[mi][2] + c1[mi][2]) - fmaf(fb.y, xe0.x, xe0.y));
            if (p.B > 1) {
              acc[mi][0][0][1] += fa.x * ((c0[mi][1] + c1[mi][1]) - fmaf(fa.y, xe1.x, xe1.y));
              acc[mi][0][0][3] += fb.x * ((c0[mi][3] + c1[mi][3]) - fmaf(fb.y, xe1.x, xe1.y));
            }
          }
        }
      } else {
        // raw chunks of every v first (the slot is free once they are in
        // registers), then dequantise and multiply one chunk at a time: only
        // one chunk's fragments are live, which keeps the B > 8 instance
        // (two column groups) out of local memory
        RowChunk A[VV], Bq[VV];
#pragma unroll
        for (int v = 0; v < VV; ++v) {
          A[v].w = lds128(wst + offA[0][v]);
          Bq[v].w = lds128(wst + offB[0][v]);
          if constexpr (FMT == W_INT4) {
            A[v].s = lds32(sst + soffA[0][v]);
            Bq[v].s = lds32(sst + soffB[0][v]);
          } else if constexpr (FMT == W_INT8) {
            A[v].s = lds16(sst + soffA[0][v]);
            Bq[v].s = lds16(sst + soffB[0][v]);
          } else {
            A[v].s = Bq[v].s = 0;
          }
        }
        __syncwarp();
        if (lane == 0 && ok) mbar_arrive(emp);
#pragma unroll
        for (int v = 0; v < VV; ++v) {
          uint32_t frag[NM][4];
          chunk_dequant<FMT>(A[v], Bq[v], frag);
          const int off = (st * T::CPS + cidx[v]) * 16;
#pragma unroll
          for (int cg = 0; cg < NG; ++cg) {
#pragma unroll
            for (int sub = 0; sub < NM / 2; ++sub) {
              const uint4 xf = lds128(xrow[cg] + off + sub * xsub);
              const int j = 2 * sub;
              mma16816(acc[0][cg][0], frag[j][0], frag[j][1], frag[j][2], frag[j][3], xf.x, xf.y);
              mma16816(acc[0][cg][1], frag[j + 1][0], frag[j + 1][1], frag[j + 1][2], frag[j + 1][3], xf.z, xf.w);
            }
          }
        }
      }
    }
    if constexpr (DIAG) {
      // the 4 lanes of a group hold different blocks: sum them
#pragma unroll
      for (int mi = 0; mi < MPW; ++mi)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float v = acc[mi][0][0][i];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          acc[mi][0][0][i] = v;
        }
    } else {
#pragma unroll
      for (int mi = 0; mi < MPW; ++mi)
#pragma unroll
        for (int cg = 0; cg < NG; ++cg)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[mi][cg][0][i] += acc[mi][cg][1][i];
    }

    // ---- combine the P k-part partials of each m-tile (fixed order).
    // Only the P warps of an m group synchronise: writers arrive on barrier
    // 2+mgrp, the reader waits on it; the reader arrives on 6+mgrp once red[]
    // is consumed, which the writers wait for before their next write.
    ++uidx;
    constexpr int GT = P * 32;                               // threads of an m group
    if (part != 0) {
      if (uidx > 1) named_sync(6 + mgrp, GT);
#pragma unroll
      for (int mi = 0; mi < MPW; ++mi)
#pragma unroll
        for (int cg = 0; cg < NG; ++cg)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            red[((((mgrp * MPW + mi) * (P - 1) + part - 1) * NG + cg) * 4 + i) * 32 + lane] = acc[mi][cg][0][i];
      named_arrive(2 + mgrp, GT);
      continue;
    }
    named_sync(2 + mgrp, GT);
    float r[MPW][NG][4];
#pragma unroll
    for (int mi = 0; mi < MPW; ++mi)
#pragma unroll
      for (int cg = 0; cg < NG; ++cg)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float v = acc[mi][cg][0][i];
#pragma unroll
          for (int q = 0; q < P - 1; ++q) v += red[((((mgrp * MPW + mi) * (P - 1) + q) * NG + cg) * 4 + i) * 32 + lane];
          r[mi][cg][i] = v;
        }
    if (more) named_arrive(6 + mgrp, GT);
#pragma unroll
    for (int mi = 0; mi < MPW; ++mi) {
      const int mt = mgrp * MPW + mi;
      const int row0 = tile * kTileRows + mt * 16;
      if (row0 >= p.N) continue;
      const int row_a = tile * kTileRows + ra[mi], row_b = tile * kTileRows + rb[mi];
      if constexpr (!SPLIT) {
#pragma unroll
        for (int cg = 0; cg < NG; ++cg) {
          float sq[2] = {0.0f, 0.0f};
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c = cg * 8 + 2 * t + h;
            if (c < p.B && p.npush) {
              for (int q = 0; q < p.npush; ++q) {
                if (p.tpx.ll_sig) {
                  tp_push_word(p.y32p[q], (long)c * p.ldy + row_a, ll_tag, r[mi][cg][h]);
                  tp_push_word(p.y32p[q], (long)c * p.ldy + row_b, ll_tag, r[mi][cg][2 + h]);
                } else {
                  p.y32p[q][(long)c * p.ldy + row_a] = r[mi][cg][h];
                  p.y32p[q][(long)c * p.ldy + row_b] = r[mi][cg][2 + h];
                }
              }
            } else if (c < p.B) {
              float va = __half2float(__float2half(r[mi][cg][h]));
              float vb = __half2float(__float2half(r[mi][cg][2 + h]));
              if (p.res) {
                va += __half2float(p.res[(long)c * p.ldres + row_a]);
                vb += __half2float(p.res[(long)c * p.ldres + row_b]);
              }
              sq[h] = va * va + vb * vb;
              p.y[(long)c * p.ldy + row_a] = __float2half(va);
              p.y[(long)c * p.ldy + row_b] = __float2half(vb);
            }
          }
          if (p.ss_out) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              float v = sq[h];
              v += __shfl_xor_sync(0xffffffffu, v, 4);
              v += __shfl_xor_sync(0xffffffffu, v, 8);
              v += __shfl_xor_sync(0xffffffffu, v, 16);
              const int c = cg * 8 + 2 * t + h;
              if (g == 0 && c < p.B) p.ss_out[(long)(row0 >> 4) * p.B + c] = v;
            }
          }
        }
      } else {
        // split K: store this split's partial for the 16 rows; the warp that
        // arrives last for this m-tile sums the partials in split order
        float* prt = p.part + (long)cur.j * p.B * p.N;
#pragma unroll
        for (int cg = 0; cg < NG; ++cg)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c = cg * 8 + 2 * t + h;
            if (c < p.B) {
              prt[(long)c * p.N + row_a] = r[mi][cg][h];
              prt[(long)c * p.N + row_b] = r[mi][cg][2 + h];
            }
          }
        __syncwarp();
        unsigned last = 0;
        if (lane == 0) {
          unsigned old;
          asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(p.cnt + (row0 >> 4)) : "memory");
          last = (old == (unsigned)cur.n - 1) ? 1u : 0u;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          // lane -> (row lane & 15, columns (lane >> 4) + 2 j): every lane
          // loads its partials of up to 4 splits at once before summing
          // them in split order, so the merge costs a few memory round trips
          // instead of one per (column, split)
          constexpr int CJ = NG * 4;
          const int rr = row0 + (lane & 15), ch = lane >> 4;
          float v[CJ];
#pragma unroll
          for (int j = 0; j < CJ; ++j) v[j] = 0.0f;
          for (int k0 = 0; k0 < cur.n; k0 += 4) {
            float tv[4][CJ];
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
#pragma unroll
              for (int j = 0; j < CJ; ++j) {
                const int c = ch + 2 * j;
                tv[kk][j] = (k0 + kk < cur.n && c < p.B)
                                ? __ldcg(p.part + ((long)(k0 + kk) * p.B + c) * p.N + rr) : 0.0f;
              }
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              if (k0 + kk < cur.n)
#pragma unroll
                for (int j = 0; j < CJ; ++j) v[j] += tv[kk][j];
          }
#pragma unroll
          for (int j = 0; j < CJ; ++j) {
            const int c = ch + 2 * j;
            float sq = 0.0f;
            if (c < p.B) {
              if (p.npush) {
                for (int q = 0; q < p.npush; ++q) {
                  if (p.tpx.ll_sig) tp_push_word(p.y32p[q], (long)c * p.ldy + rr, ll_tag, v[j]);
                  else p.y32p[q][(long)c * p.ldy + rr] = v[j];
                }
              } else {
                float o = __half2float(__float2half(v[j]));
                if (p.res) o += __half2float(p.res[(long)c * p.ldres + rr]);
                p.y[(long)c * p.ldy + rr] = __float2half(o);
                sq = o * o;
              }
            }
            if (p.ss_out && !p.npush) {
              sq += __shfl_xor_sync(0xffffffffu, sq, 1);
              sq += __shfl_xor_sync(0xffffffffu, sq, 2);
              sq += __shfl_xor_sync(0xffffffffu, sq, 4);
              sq += __shfl_xor_sync(0xffffffffu, sq, 8);
              if ((lane & 15) == 0 && c < p.B) p.ss_out[(long)(row0 >> 4) * p.B + c] = sq;
            }
          }
          if (lane == 0) p.cnt[row0 >> 4] = 0u;
        }
      }
    }
  }
  // outputs pushed into peer memory: the last CTA signals the exchange to
  // every rank once all CTAs' pushes are fenced at system scope
  if (p.tpx.nsig) {
    if (stamp) tp_stamp(p.tpx, 6, p.tpx.sig_idx);
    consumer_sync();
    if (ctid == 0) tp_signal_cta(p.tpx);
  } else if (p.npush > 1 && !p.tpx.ll_sig) {
    __threadfence_system();
  }
  if (ctid == 0) TRACE(4, 0);
}

// --------------------------------------------------------------- host ----
static std::atomic<long> g_spin_limit{kSpinLimit};
#ifdef R4Q_TRACE
static int g_trace_launch = 0;
#endif
long gemv_spin_limit() { return g_spin_limit.load(std::memory_order_relaxed); }
long gemv_set_spin_limit(long polls) {
  return g_spin_limit.exchange(polls > 0 ? polls : kSpinLimit);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

// 2-D byte tensor [rows, row_bytes] with box [box_rows, box_bytes]
int make_map(CUtensorMap* m, const void* base, long rows, long row_bytes, int box_bytes,
                    int box_rows, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(R4Q_ERR_CUDA, "gemv: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)box_bytes, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(R4Q_ERR_CUDA, "gemv: tensor map encode failed (%d)", (int)r);
  return R4Q_OK;
}

bool gemv_tma_supported(const GemvArgs& a, int fmt) {
  if (fmt == W_INT4) return a.K % 128 == 0 && aligned(a.s, 16);
  if (fmt == W_INT8) return a.K % 256 == 0 && aligned(a.s, 16);
  return a.K % 8 == 0;
}

struct TmaPlan {
  int S, gt;
  size_t smem;
  int x_bytes;
  int xsum_bytes;
  int ns;
};

// Largest dynamic shared memory this kernel may use: the per-block opt-in
// limit minus its static shared memory.  Sets the attribute once per device.
template <int FMT, int NG, bool DIAG, int PRO, bool TPC>
static size_t tma_smem_limit() {
  // both SPLIT instances have the same static shared memory
  static std::mutex mu;
  static std::unordered_map<int, size_t> lim;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  auto it = lim.find(dev);
  if (it != lim.end()) return it->second;
  int optin = 0;
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaFuncAttributes fa{};
  size_t v = 0;
  if (optin > 0 && cudaFuncGetAttributes(&fa, gemv_tma_kernel<FMT, NG, DIAG, PRO, TPC, false>) == cudaSuccess) {
    v = (size_t)optin - fa.sharedSizeBytes;
    if (cudaFuncSetAttribute(gemv_tma_kernel<FMT, NG, DIAG, PRO, TPC, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)v) != cudaSuccess ||
        cudaFuncSetAttribute(gemv_tma_kernel<FMT, NG, DIAG, PRO, TPC, true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)v) != cudaSuccess)
      v = 0;
  }
  cudaGetLastError();  // leave no error behind for the caller's runtime
  lim[dev] = v;
  return v;
}

// R4Q_GEMV_PLAN_LOG=1 prints every candidate plan (measurement only).
static bool plan_log() {
  static const bool v = [] {
    const char* e = getenv("R4Q_GEMV_PLAN_LOG");
    return e && e[0] == '1';
  }();
  return v;
}

template <int FMT, int NG, bool DIAG, int PRO, bool TPC>
static TmaPlan plan_tma(int B, int N, int K, size_t ws_bytes) {
  using T = TmaFmt<FMT>;
  using F = Fmt<FMT>;
  const int nsm = num_sms();
  const int tiles = (N + kTileRows - 1) / kTileRows;
  const int nst = (K + T::SK - 1) / T::SK;
  const size_t stage = (size_t)kTileRows * T::CPS * 16 + (size_t)kTileRows * T::SBYTES;
  const size_t fixed = 1024 + (size_t)red_floats<NG, DIAG>() * 4 + 2 * T::NS * 8 + 16;
  const size_t smem_limit = tma_smem_limit<FMT, NG, DIAG, PRO, TPC>();
  TmaPlan best{1, 1, 0, 0, 0, 0};
  double best_cost = 1e30;
  // R4Q_GEMV_SPLIT forces the K split count (measurement only)
  static const int forced_split = [] {
    const char* e = getenv("R4Q_GEMV_SPLIT");
    return e ? atoi(e) : 0;
  }();
  for (int S = 1; S <= kTmaMaxSplit && S <= nst; ++S) {
    if (forced_split > 0 && S != forced_split && forced_split <= nst) continue;
    const int gt = nsm / S;
    if (gt < 1) break;
    if (S > 1 && gemv_ws_bytes_for(B, N, S) > ws_bytes) break;
    const int per = (nst + S - 1) / S;                       // stages per unit (max)
    const int colstride = x_colstride(per * T::CPS / 4 / F::U, F::NSUB, F::U);
    const size_t xb = (size_t)colstride * B;
    const size_t xsb = DIAG ? (size_t)2 * per * T::CPS * sizeof(float2) : 0;
    if (fixed + xb + xsb + 2 * stage > smem_limit) continue;
    // the ring takes all shared memory the activations leave: under full HBM
    // load a stage takes microseconds to land, so depth is bandwidth
    int ns = (int)((smem_limit - fixed - xb - xsb) / stage);
    if (ns > T::NS) ns = T::NS;
    const int rounds = (tiles + gt - 1) / gt;
    // busiest CTA streams rounds * per stages (slower with a shallow ring);
    // S > 1 adds a partial merge per tile
    const double depth_pen = ns < 8 ? (8.0 - ns) * 0.08 : 0.0;
    // (a unit boundary with a split-K merge costs about two stages: measured
    // on B200 with forced splits at B = 1 and 16)
    const double cost = (double)rounds * per * (1.0 + depth_pen) + (S > 1 ? 2.0 * rounds : 0.0) + 0.02 * S;
    if (plan_log()) fprintf(stderr, "r4q plan B=%d N=%d K=%d S=%d gt=%d ns=%d rounds=%d per=%d cost=%.2f\n", B, N, K,
                            S, gt, ns, rounds, per, cost);
    if (cost < best_cost) {
      best_cost = cost;
      best = TmaPlan{S, gt, fixed + xb + xsb + (size_t)ns * stage, (int)xb, (int)xsb, ns};
    }
  }
  if (plan_log()) fprintf(stderr, "r4q plan B=%d N=%d K=%d -> S=%d\n", B, N, K, best.S);
  return best;
}

template <int FMT, int NG, bool DIAG, int PRO, bool TPC>
static int launch_tma_t(const GemvArgs& a) {
  using T = TmaFmt<FMT>;
  const TmaPlan pl = plan_tma<FMT, NG, DIAG, PRO, TPC>(a.B, a.N, a.K, a.ws_bytes);
  if (pl.smem == 0) return set_error(R4Q_ERR_CAPACITY, "gemv: no TMA plan fits shared memory");
  if (pl.S > 1 && !a.ws) return set_error(R4Q_ERR_CAPACITY, "gemv: workspace required");
  CUtensorMap tmw, tms;
  const long rowbytes = (FMT == W_INT4) ? a.K / 2 : (FMT == W_INT8 ? a.K : 2L * a.K);
  int st = make_map(&tmw, a.w, a.N, rowbytes, 128, kTileRows, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  if (FMT == W_INT4) st = make_map(&tms, a.s, a.N, a.K / 8, 128, kTileRows, CU_TENSOR_MAP_SWIZZLE_128B);
  else if (FMT == W_INT8) st = make_map(&tms, a.s, a.N, a.K / 16, 32, kTileRows, CU_TENSOR_MAP_SWIZZLE_32B);
  else tms = tmw;
  if (st) return st;

  TmaParams tp{};
  GemvParams& p = tp.p;
  p.x = reinterpret_cast<const __half*>(a.x);
  p.ldx = a.ldx;
  p.w = reinterpret_cast<const uint8_t*>(a.w);
  p.s = reinterpret_cast<const __half*>(a.s);
  p.y = reinterpret_cast<__half*>(a.y);
  p.ldy = a.ldy;
  p.B = a.B; p.N = a.N; p.K = a.K;
  p.mt = 4;
  p.ksplit = pl.S;
  p.prologue = a.prologue;
  p.norm_w = reinterpret_cast<const __half*>(a.norm_w);
  p.eps = a.eps;
  p.ss_in = a.ss_in;
  p.ss_in_parts = a.ss_in_parts;
  p.res = reinterpret_cast<const __half*>(a.res);
  p.ldres = a.ldres;
  p.ss_out = a.ss_out;
  p.npush = a.npush;
  for (int q = 0; q < 8; ++q) p.y32p[q] = q < a.npush ? a.y32p[q] : nullptr;
  p.tpx = a.tpx;
  p.cnt = gemv_counters(a.ws);
  p.part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(a.ws) + gemv_cnt_bytes(a.N));
  tp.nstages = (a.K + T::SK - 1) / T::SK;
  tp.tiles = (a.N + kTileRows - 1) / kTileRows;
  tp.gt = pl.gt;
  tp.x_bytes = pl.x_bytes;
  tp.xsum_bytes = pl.xsum_bytes;
  tp.ns = pl.ns;
  tp.spin = gemv_spin_limit();
  {
    // R4Q_GEMV_PREWAIT=n: request only n stages before the activations are
    // staged (measurement only; default kPrewait)
    static const int pw = [] {
      const char* e = getenv("R4Q_GEMV_PREWAIT");
      return e ? atoi(e) : -1;
    }();
    tp.prewait = pw >= 0 ? pw : kPrewait;
  }
#ifdef R4Q_TRACE
  tp.trace_par = (g_trace_launch++) & 7;
#endif
  tp.status = reinterpret_cast<int*>(a.ws);   // header word 0 (null without a workspace)

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(pl.S * pl.gt);
  cfg.blockDim = dim3(kTmaThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = a.stream;
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 1;
  cudaError_t e = pl.S > 1 ? cudaLaunchKernelEx(&cfg, gemv_tma_kernel<FMT, NG, DIAG, PRO, TPC, true>, tmw, tms, tp)
                           : cudaLaunchKernelEx(&cfg, gemv_tma_kernel<FMT, NG, DIAG, PRO, TPC, false>, tmw, tms, tp);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(R4Q_ERR_CUDA, "gemv_tma_kernel (smem %zu): %s", pl.smem, cudaGetErrorString(e));
  }
  return R4Q_OK;
}

#ifdef R4Q_TRACE
extern "C" int r4q_trace_read(unsigned long long* host) {  // [8][8][256]
  return cudaMemcpyFromSymbol(host, g_trace, sizeof(g_trace)) == cudaSuccess ? 0 : -4;
}
extern "C" int r4q_trace_mode(int m) {
  return cudaMemcpyToSymbol(g_dbg_mode, &m, sizeof(int)) == cudaSuccess ? 0 : -4;
}
extern "C" int r4q_trace_reset_counter() {
  g_trace_launch = 0;
  return 0;
}
extern "C" int r4q_trace_clear() {
  static unsigned long long z[8][8][256];
  return cudaMemcpyToSymbol(g_trace, z, sizeof(g_trace)) == cudaSuccess ? 0 : -4;
}
#endif

// Instance per (format, column groups, block-diagonal) x (prologue) and the
// tensor-parallel consumer (always an RMSNorm+FWHT prologue).
template <int FMT, int NG, bool DIAG>
static int launch_tma_pro(const GemvArgs& a) {
  if (a.tpx.nwait) {
    if (a.prologue != R4Q_PRO_RMSNORM_FWHT)
      return set_error(R4Q_ERR_ARG, "gemv: a tensor-parallel consumer needs the RMSNorm+FWHT prologue");
    return launch_tma_t<FMT, NG, DIAG, R4Q_PRO_RMSNORM_FWHT, true>(a);
  }
  switch (a.prologue) {
    case R4Q_PRO_FWHT: return launch_tma_t<FMT, NG, DIAG, R4Q_PRO_FWHT, false>(a);
    case R4Q_PRO_SILU_FWHT: return launch_tma_t<FMT, NG, DIAG, R4Q_PRO_SILU_FWHT, false>(a);
    case R4Q_PRO_RMSNORM_FWHT: return launch_tma_t<FMT, NG, DIAG, R4Q_PRO_RMSNORM_FWHT, false>(a);
    default: return launch_tma_t<FMT, NG, DIAG, R4Q_PRO_NONE, false>(a);
  }
}

int launch_gemv_tma(const GemvArgs& a, int fmt) {
  const bool two = a.B > 8;
  switch (fmt) {
    case W_INT4:
      if (a.B <= 2) return launch_tma_pro<W_INT4, 1, true>(a);
      return two ? launch_tma_pro<W_INT4, 2, false>(a) : launch_tma_pro<W_INT4, 1, false>(a);
    case W_INT8: return two ? launch_tma_pro<W_INT8, 2, false>(a) : launch_tma_pro<W_INT8, 1, false>(a);
    case W_FP16: return two ? launch_tma_pro<W_FP16, 2, false>(a) : launch_tma_pro<W_FP16, 1, false>(a);
  }
  return set_error(R4Q_ERR_ARG, "gemv: unknown weight format %d", fmt);
}

}  // namespace r4q
