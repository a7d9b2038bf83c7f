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

#include <mutex>
#include <unordered_map>

#include "gemv_dev.cuh"

namespace r4q {

constexpr int kTmaConsumers = 16;
constexpr int kTmaThreads = (kTmaConsumers + 1) * 32;
constexpr int kTileRows = 64;
constexpr int kTmaMaxSplit = 32;
constexpr long kSpinLimit = 1L << 26;  // bounded mbarrier waits (seconds of wall time)

// A stage is 64 rows x SK k.
template <int FMT> struct TmaFmt;
template <> struct TmaFmt<W_INT4> {
  static constexpr int SK = 512;         // k per stage
  static constexpr int CPS = 16;         // 16-byte chunks per row per stage
  static constexpr int BOXES = 2;        // 128-byte weight boxes per row per stage
  static constexpr int SBYTES = 64;      // (scale, zero) bytes per row per stage
  static constexpr int NS = 6;           // ring depth
};
template <> struct TmaFmt<W_INT8> {
  static constexpr int SK = 512, CPS = 32, BOXES = 4, SBYTES = 32, NS = 4;
};
template <> struct TmaFmt<W_FP16> {
  static constexpr int SK = 256, CPS = 32, BOXES = 4, SBYTES = 0, NS = 4;
};

struct TmaParams {
  GemvParams p;
  int nstages;     // stages over the whole K
  int tiles;       // 64-row tiles
  int gt;          // CTAs per K split
  int x_bytes;     // activation smem bytes
  int* status;     // set to 1 when a bounded wait gives up
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
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after kSpinLimit polls, records the failure and
// returns false so the kernel can drain and exit instead of hanging.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, unsigned parity, int* status) {
  for (long i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(b, parity)) return true;
  if (status) atomicExch(status, 1);
  return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kTmaConsumers * 32) : "memory");
}

// Row order inside a 16-row m-tile: rows read by the same quarter-warp
// (groups 2q, 2q+1) differ in bit 2, so the 128-byte swizzle maps their
// chunks to disjoint banks.
__device__ __forceinline__ int row_perm(int g) { return ((g & 1) << 2) | (g >> 1); }

// ------------------------------------------------------------- kernel ----
template <int FMT, int NG>
__global__ void __launch_bounds__(kTmaThreads, 1)
    gemv_tma_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tms,
                    const TmaParams tp) {
  using T = TmaFmt<FMT>;
  using F = Fmt<FMT>;
  constexpr int W_STAGE = kTileRows * T::CPS * 16;     // bytes of weights per stage
  constexpr int S_STAGE = kTileRows * T::SBYTES;
  constexpr int NS = T::NS;
  constexpr int V = T::CPS / 16;                       // chunks per thread per row per stage
  constexpr int NM = ChunkMma<FMT>::N;
  const GemvParams& p = tp.p;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring_w = smem;
  uint8_t* ring_s = ring_w + NS * W_STAGE;
  uint8_t* xs = ring_s + NS * S_STAGE;
  float* red = reinterpret_cast<float*>(xs + tp.x_bytes);          // [4 m-tiles][3][NG*4][32]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + 4 * 3 * NG * 4 * 32);
  uint64_t* empty = full + NS;
  __shared__ float s_rrms[16];
  __shared__ unsigned s_last;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = p.ksplit;
  const int ks = blockIdx.x % S;
  const int cta_in_split = blockIdx.x / S;
  const int st0 = (int)((long)ks * tp.nstages / S);
  const int st1 = (int)((long)(ks + 1) * tp.nstages / S);
  const int nst = st1 - st0;

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
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmw)) : "memory");
      if (T::SBYTES) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tms)) : "memory");
      int it = 0;
      bool ok = true;
      for (int tile = cta_in_split; tile < tp.tiles && ok; tile += tp.gt) {
        for (int st = st0; st < st1 && ok; ++st, ++it) {
          const int slot = it % NS;
          const unsigned ph = (unsigned)(it / NS) & 1u;
          if (it >= NS) ok = mbar_wait(&empty[slot], ph ^ 1u, tp.status);
          if (!ok) break;
          mbar_expect_tx(&full[slot], W_STAGE + S_STAGE);
#pragma unroll
          for (int b = 0; b < T::BOXES; ++b)
            tma_load_2d(ring_w + slot * W_STAGE + b * (kTileRows * 128), &tmw,
                        st * (T::CPS * 16) + b * 128, tile * kTileRows, &full[slot]);
          if (T::SBYTES)
            tma_load_2d(ring_s + slot * S_STAGE, &tms, st * T::SBYTES, tile * kTileRows, &full[slot]);
        }
      }
    }
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    return;
  }

  // ------------------------------------------------------------ consumers
  // everything below may read outputs of the previous kernel in the stream
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int ctid = tid;  // 0 .. kTmaConsumers*32-1
  const int ncolx = p.B;
  const int nch_pad = nst * T::CPS;
  const int colstride = tp.x_bytes / (ncolx > 0 ? ncolx : 1);

  if (p.prologue == R4Q_PRO_RMSNORM_FWHT) {
    for (int c = warp; c < ncolx; c += kTmaConsumers) {
      float ss = 0.0f;
      if (p.ss_in) {
        for (int i = lane; i < p.ss_in_parts; i += 32) ss += p.ss_in[(long)i * ncolx + c];
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
  }
  {
    const int nblk = nch_pad * F::CK / 32;
    const int k_base = st0 * T::SK;
    for (int item = ctid; item < ncolx * nblk; item += kTmaConsumers * 32) {
      const int col = item / nblk, blk = item - col * nblk;
      __half v[32];
      load_block32(p, col, k_base + blk * 32,
                   p.prologue == R4Q_PRO_RMSNORM_FWHT ? s_rrms[col] : 1.0f, v);
      store_block32<FMT>(xs + (long)col * colstride, nch_pad, blk, v);
    }
  }
  consumer_sync();

  // warp -> (k quarter, m-tile); every stage is consumed by all 16 warps
  const int g = lane >> 2, t = lane & 3;
  const int mt = warp & 3, part = warp >> 2;
  const int ra = mt * 16 + row_perm(g), rb = ra + 8;       // rows inside the 64-row tile
  int colx[NG];
#pragma unroll
  for (int cg = 0; cg < NG; ++cg) colx[cg] = min(cg * 8 + g, p.B - 1);

  int it0 = 0;                                              // ring index of the unit's first stage
  bool ok = true;
  for (int tile = cta_in_split; tile < tp.tiles; tile += tp.gt, it0 += nst) {
    float acc[NG][2][4];
#pragma unroll
    for (int cg = 0; cg < NG; ++cg)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[cg][h][i] = 0.0f;

    for (int st = 0; st < nst; ++st) {
      const int it = it0 + st;
      const int slot = it % NS;
      const unsigned ph = (unsigned)(it / NS) & 1u;
      if (ok) ok = mbar_wait(&full[slot], ph, tp.status);
      const uint8_t* wst = ring_w + slot * W_STAGE;
      const uint8_t* sst = ring_s + slot * S_STAGE;
      uint32_t frag[V][NM][4];
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const int c = part * (T::CPS / 4) + 4 * v + t;     // chunk within the stage row
        const int box = c >> 3, cb = c & 7;
        RowChunk A, Bq;
        A.w = *reinterpret_cast<const uint4*>(wst + box * (kTileRows * 128) + ra * 128 + ((cb ^ (ra & 7)) << 4));
        Bq.w = *reinterpret_cast<const uint4*>(wst + box * (kTileRows * 128) + rb * 128 + ((cb ^ (rb & 7)) << 4));
        if constexpr (FMT == W_INT4) {
          // 64-byte rows, 64-byte swizzle: 16-byte unit index ^= row bits 1-2
          const int ua = ((c >> 2) ^ ((ra >> 1) & 3)) << 4, ub = ((c >> 2) ^ ((rb >> 1) & 3)) << 4;
          A.s = *reinterpret_cast<const uint32_t*>(sst + ra * 64 + ua + (c & 3) * 4);
          Bq.s = *reinterpret_cast<const uint32_t*>(sst + rb * 64 + ub + (c & 3) * 4);
        } else if constexpr (FMT == W_INT8) {
          // 32-byte rows, 32-byte swizzle: 16-byte half index ^= row bit 2
          const int b = c >> 1;
          const int ha = ((b >> 3) ^ ((ra >> 2) & 1)) << 4, hb = ((b >> 3) ^ ((rb >> 2) & 1)) << 4;
          A.s = *reinterpret_cast<const uint16_t*>(sst + ra * 32 + ha + (b & 7) * 2);
          Bq.s = *reinterpret_cast<const uint16_t*>(sst + rb * 32 + hb + (b & 7) * 2);
        } else {
          A.s = Bq.s = 0;
        }
        chunk_dequant<FMT>(A, Bq, frag[v]);
      }
      // the slot is free once its bytes are in registers; the MMAs follow
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const int c = part * (T::CPS / 4) + 4 * v + t;
        chunk_mma_frag<FMT, NG>(frag[v], xs, colstride, nch_pad, st * T::CPS + c, colx, acc);
      }
    }
#pragma unroll
    for (int cg = 0; cg < NG; ++cg)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[cg][0][i] += acc[cg][1][i];

    // ---- combine the 4 k-quarter partials of each m-tile (fixed order) ----
    if (part != 0) {
#pragma unroll
      for (int cg = 0; cg < NG; ++cg)
#pragma unroll
        for (int i = 0; i < 4; ++i) red[(((mt * 3 + part - 1) * NG + cg) * 4 + i) * 32 + lane] = acc[cg][0][i];
    }
    consumer_sync();
    const int row0 = tile * kTileRows + mt * 16;
    if (part == 0 && row0 < p.N) {
      float r[NG][4];
#pragma unroll
      for (int cg = 0; cg < NG; ++cg)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float v = acc[cg][0][i];
#pragma unroll
          for (int q = 0; q < 3; ++q) v += red[(((mt * 3 + q) * NG + cg) * 4 + i) * 32 + lane];
          r[cg][i] = v;
        }
      const int row_a = tile * kTileRows + ra, row_b = tile * kTileRows + rb;
      if (S == 1) {
#pragma unroll
        for (int cg = 0; cg < NG; ++cg) {
          float sq[2] = {0.0f, 0.0f};
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c = cg * 8 + 2 * t + h;
            if (c < p.B) {
              float va = __half2float(__float2half(r[cg][h]));
              float vb = __half2float(__float2half(r[cg][2 + h]));
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
        float* prt = p.part + (long)ks * p.B * p.N;
#pragma unroll
        for (int cg = 0; cg < NG; ++cg)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c = cg * 8 + 2 * t + h;
            if (c < p.B) {
              prt[(long)c * p.N + row_a] = r[cg][h];
              prt[(long)c * p.N + row_b] = r[cg][2 + h];
            }
          }
      }
    }
    if (S > 1) {
      // the partial stores of this CTA are ordered before thread 0's gpu-scope
      // acq_rel atomic by the barrier; the last arriving CTA of the tile sums
      // the split partials in split order
      consumer_sync();
      if (ctid == 0) {
        unsigned old;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(p.cnt + tile) : "memory");
        s_last = (old == (unsigned)S - 1) ? 1u : 0u;
      }
      consumer_sync();
      if (s_last) {
        const int trow0 = tile * kTileRows;
        const int tiles16 = min(4, (p.N - trow0) >> 4);
        for (int task = warp; task < tiles16 * p.B; task += kTmaConsumers) {
          const int ti = task / p.B, col = task - ti * p.B;
          const int rr = trow0 + ti * 16 + (lane & 15);
          float v = 0.0f;
          for (int k2 = 0; k2 < S; ++k2) v += __ldcg(p.part + ((long)k2 * p.B + col) * p.N + rr);
          v = __half2float(__float2half(v));
          if (p.res) v += __half2float(p.res[(long)col * p.ldres + rr]);
          if (lane < 16) p.y[(long)col * p.ldy + rr] = __float2half(v);
          float sq = (lane < 16) ? v * v : 0.0f;
          sq = warp_sum(sq);
          if (p.ss_out && lane == 0) p.ss_out[(long)((trow0 >> 4) + ti) * p.B + col] = sq;
        }
        if (ctid == 0) p.cnt[tile] = 0u;
      }
    }
    consumer_sync();  // red[] and s_last are reused by the next tile
  }
}

// --------------------------------------------------------------- host ----
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
static int make_map(CUtensorMap* m, const void* base, long rows, long row_bytes, int box_bytes,
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
};

// Largest dynamic shared memory this kernel may use: the per-block opt-in
// limit minus its static shared memory.  Sets the attribute once per device.
template <int FMT, int NG>
static size_t tma_smem_limit() {
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
  if (optin > 0 && cudaFuncGetAttributes(&fa, gemv_tma_kernel<FMT, NG>) == cudaSuccess) {
    v = (size_t)optin - fa.sharedSizeBytes;
    if (cudaFuncSetAttribute(gemv_tma_kernel<FMT, NG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)v) != cudaSuccess)
      v = 0;
  }
  cudaGetLastError();  // leave no error behind for the caller's runtime
  lim[dev] = v;
  return v;
}

template <int FMT, int NG>
static TmaPlan plan_tma(int B, int N, int K, size_t ws_bytes) {
  using T = TmaFmt<FMT>;
  using F = Fmt<FMT>;
  const int nsm = num_sms();
  const int tiles = (N + kTileRows - 1) / kTileRows;
  const int nst = (K + T::SK - 1) / T::SK;
  const size_t fixed = 1024 + (size_t)T::NS * (kTileRows * T::CPS * 16 + kTileRows * T::SBYTES) +
                       4 * 3 * NG * 4 * 32 * 4 + 2 * T::NS * 8;
  const size_t smem_limit = tma_smem_limit<FMT, NG>();
  TmaPlan best{1, 1, 0, 0};
  double best_cost = 1e30;
  for (int S = 1; S <= kTmaMaxSplit && S <= nst; ++S) {
    const int gt = nsm / S;
    if (gt < 1) break;
    if (S > 1 && gemv_ws_bytes_for(B, N, S) > ws_bytes) break;
    const int per = (nst + S - 1) / S;                       // stages per unit (max)
    const int colstride = x_colstride(per * T::CPS / 4 / F::U, F::NSUB, F::U);
    const size_t xb = (size_t)colstride * B;
    if (fixed + xb > smem_limit) continue;
    const int rounds = (tiles + gt - 1) / gt;
    // busiest CTA streams rounds * per stages; S > 1 adds a merge per tile
    const double cost = (double)rounds * per + (S > 1 ? 0.35 * rounds : 0.0) + 0.02 * S;
    if (cost < best_cost) {
      best_cost = cost;
      best = TmaPlan{S, gt, fixed + xb, (int)xb};
    }
  }
  return best;
}

template <int FMT, int NG>
static int launch_tma_t(const GemvArgs& a) {
  using T = TmaFmt<FMT>;
  const TmaPlan pl = plan_tma<FMT, NG>(a.B, a.N, a.K, a.ws_bytes);
  if (pl.smem == 0) return set_error(R4Q_ERR_CAPACITY, "gemv: no TMA plan fits shared memory");
  if (pl.S > 1 && !a.ws) return set_error(R4Q_ERR_CAPACITY, "gemv: workspace required");
  CUtensorMap tmw, tms;
  const long rowbytes = (FMT == W_INT4) ? a.K / 2 : (FMT == W_INT8 ? a.K : 2L * a.K);
  int st = make_map(&tmw, a.w, a.N, rowbytes, 128, kTileRows, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  if (FMT == W_INT4) st = make_map(&tms, a.s, a.N, a.K / 8, 64, kTileRows, CU_TENSOR_MAP_SWIZZLE_64B);
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
  p.cnt = reinterpret_cast<unsigned*>(a.ws);
  p.part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(a.ws) + gemv_cnt_bytes(a.N));
  tp.nstages = (a.K + T::SK - 1) / T::SK;
  tp.tiles = (a.N + kTileRows - 1) / kTileRows;
  tp.gt = pl.gt;
  tp.x_bytes = pl.x_bytes;
  tp.status = a.ws ? reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(a.ws) + gemv_cnt_bytes(a.N) - 4) : nullptr;

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
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_tma_kernel<FMT, NG>, tmw, tms, tp);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(R4Q_ERR_CUDA, "gemv_tma_kernel (smem %zu): %s", pl.smem, cudaGetErrorString(e));
  }
  return R4Q_OK;
}

int launch_gemv_tma(const GemvArgs& a, int fmt) {
  const bool two = a.B > 8;
  switch (fmt) {
    case W_INT4: return two ? launch_tma_t<W_INT4, 2>(a) : launch_tma_t<W_INT4, 1>(a);
    case W_INT8: return two ? launch_tma_t<W_INT8, 2>(a) : launch_tma_t<W_INT8, 1>(a);
    case W_FP16: return two ? launch_tma_t<W_FP16, 2>(a) : launch_tma_t<W_FP16, 1>(a);
  }
  return set_error(R4Q_ERR_ARG, "gemv: unknown weight format %d", fmt);
}

}  // namespace r4q
