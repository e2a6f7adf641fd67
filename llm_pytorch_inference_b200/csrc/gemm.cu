// Dense bf16 GEMM for the decode-step projections on 5th-generation tensor cores.
//
//   Y[m, n] = sum_k X[m, k] * W[n, k]      (X: activations, m = batch; W: nn.Linear weight)
//
// Replaces the nn.Linear / cuBLAS calls of the reference decode step: q/k/v
// (models/model_cuda.py:124-126), o_proj (:180), gate_up / down (ops/mlp.py:66, :84)
// and lm_head (model_cuda.py:413).
//
// Decode GEMMs have a tiny m, so the kernel computes D^T = W X^T ("swap AB"): a
// 128-row slab of W is the UMMA M=128 operand, the whole batch is UMMA N=BN.  Both
// operands are K-major and arrive through TMA in the 128-byte swizzle layout.  The
// weight stream (the only large traffic) is split evenly over G CTAs (two per SM at batch
// <= 64, see splitk_ctas) by stream-K: CTA c owns k-blocks [c*T/G, (c+1)*T/G) of the linearised (tile, k-block)
// space.  A tile covered by several CTAs is merged by the last CTA to finish it,
// summing the fp32 partials in CTA order (deterministic).
//
// More than 256 rows (a prefill's tokens) are cut into row tiles of 256: the output tiles are the
// (weight tile, row tile) pairs, weight-major, so consecutive tiles of a CTA reuse one weight slab
// from L2.  With an even number of weight tiles they go to gemm_rows_kernel (256 x 256 tiles, below).
//
// Warp roles (192 threads):  warp 0 TMA producer, warp 1 TMEM alloc + MMA issue,
// warps 2-5 epilogue (TMEM -> registers -> global).  Accumulators are double
// buffered in TMEM so the next tile's MMAs overlap the previous tile's epilogue.
#include "common.cuh"
#include "host.h"
#include "splitk.cuh"
#include "tp.cuh"

namespace mvb {
namespace {

constexpr int BM = 128;               // UMMA M: weight rows (output features) per tile
constexpr int BK = 64;                // k per stage: one 128-byte swizzle row of bf16
constexpr int A_STAGE = BM * BK * 2;  // 16 KB
constexpr int kThreads = 192;

struct GemmArgs {
  __nv_bfloat16* y;
  int64_t ldy;
  const __nv_bfloat16* aux;
  int64_t ld_aux;
  int m, n, k;
  int tiles;     // output tiles: weight tiles x row tiles
  int mt;        // row tiles (ceil(m / BN)); 1 for decode batches
  int kblocks;   // k / BK
  int epilogue;  // MVB_EPI_*
  int inter;     // SWIGLU: rows of the gate half of W
  int maxc;      // PARTIALS: slots per tile (most contributors of any tile)
  float* partials;
  int* counters;
  unsigned* err;
};

__device__ __forceinline__ int64_t range_start(int c, int64_t total, int grid) {
  return static_cast<int64_t>(c) * total / grid;
}
// CTA whose k-block range holds linear k-block x.
__device__ __forceinline__ int cta_of(int64_t x, int64_t total, int grid) {
  return static_cast<int>(((x + 1) * grid + total - 1) / total - 1);
}

// Named barrier of the 128 threads (4 warps) that share one accumulator's epilogue.
template <int BAR = 1>
__device__ __forceinline__ void epi_bar() {
  asm volatile("bar.sync %0, 128;" ::"n"(BAR) : "memory");
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

// Final epilogue for 32 batch columns [c0, c0+32) of feature `row` of weight tile t, rows
// r0 + c0 .. of Y.
template <int BN, int BAR = 1>
__device__ __forceinline__ void epilogue_store(const GemmArgs& a, const TpGemm& tp, const float (&v)[32], int t,
                                               int row, int c0, float* xbuf, int r0) {
  if (a.epilogue == MVB_EPI_SWIGLU) {
    // TMEM lanes 0-63 hold gate features 64t + r, lanes 64-127 the matching up features.
    const bool is_up = row >= 64;
    const int r = row & 63;
    if (is_up) {
#pragma unroll
      for (int j = 0; j < 32; ++j) xbuf[r * 33 + j] = bf16_round(v[j]);
    }
    epi_bar<BAR>();
    if (!is_up) {
      const int f = 64 * t + r;
      if (f < a.inter) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int b = r0 + c0 + j;
          if (b < a.m) {
            const float g = bf16_round(v[j]);
            const float s = bf16_round(silu_f(g));
            a.y[static_cast<int64_t>(b) * a.ldy + f] = __float2bfloat16_rn(s * xbuf[r * 33 + j]);
          }
        }
      }
    }
    epi_bar<BAR>();
    return;
  }
  const int nn = t * BM + row;
  if (nn >= a.n) return;
  if (a.epilogue == MVB_EPI_RESADD) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int b = r0 + c0 + j;
      if (b < a.m) {
        const float r = __bfloat162float(a.aux[static_cast<int64_t>(b) * a.ld_aux + nn]);
        a.y[static_cast<int64_t>(b) * a.ldy + nn] = __float2bfloat16_rn(r + bf16_round(v[j]));
      }
    }
    return;
  }
  if (tp.nranks > 0 && tp.y[0] != nullptr) {
    // all-gather: this rank's output columns land in every rank's copy of the full output
    for (int q = 0; q < tp.nranks; ++q) {
      __nv_bfloat16* yq = tp.y[q];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int b = c0 + j;
        if (b < a.m) yq[static_cast<int64_t>(b) * a.ldy + nn] = __float2bfloat16_rn(v[j]);
      }
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int b = r0 + c0 + j;
    if (b < a.m) a.y[static_cast<int64_t>(b) * a.ldy + nn] = __float2bfloat16_rn(v[j]);
  }
}

// BN=64 (decode batches) keeps ~106 KB of shared memory and <= 168 registers so that two CTAs
// fit on one SM: the grid is two CTAs per SM, doubling the weight bytes in flight per SM.
template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, BN == 64 ? 2 : 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                     const GemmArgs a, const __grid_constant__ TpGemm tp) {
  constexpr int B_STAGE = BN * BK * 2;
  constexpr uint32_t STAGE_BYTES = A_STAGE + B_STAGE;
  constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulator buffers
  constexpr uint32_t IDESC = umma_idesc_bf16(BM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;  // [2]
  uint64_t* acce = accf + 2;        // [2]
  uint64_t* drain = acce + 2;       // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = abort_flag + 1;
  float* xbuf = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES + 256);  // 64 x 33 floats (SWIGLU)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int64_t total = static_cast<int64_t>(a.tiles) * a.kblocks;
  const int64_t kb_begin = range_start(blockIdx.x, total, G);
  const int64_t kb_end = range_start(blockIdx.x + 1, total, G);
  const int my_kb = static_cast<int>(kb_end - kb_begin);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *last_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) pdl_launch_dependents();

  int issued = 0;  // producer: loads issued
  if (warp == 0) {
    if (lane == 0 && my_kb > 0) {
      prefetch_tmap(&tmW);
      prefetch_tmap(&tmX);
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      const bool swiglu = a.epilogue == MVB_EPI_SWIGLU || a.epilogue == MVB_EPI_SWIGLU_PARTIALS;
      auto load_w = [&](int it) {
        const int s = it % STAGES;
        const int64_t g = kb_begin + it;
        const int lt = static_cast<int>(g / a.kblocks);  // linear tile
        const int kb = static_cast<int>(g - static_cast<int64_t>(lt) * a.kblocks);
        const int t = lt / a.mt;  // weight tile
        if (swiglu) {
          tma_load_2d(sA + s * A_STAGE, &tmW, &full[s], kb * BK, 64 * t, pol_w);
          tma_load_2d(sA + s * A_STAGE + A_STAGE / 2, &tmW, &full[s], kb * BK, a.inter + 64 * t, pol_w);
        } else {
          tma_load_2d(sA + s * A_STAGE, &tmW, &full[s], kb * BK, BM * t, pol_w);
        }
      };
      auto load_x = [&](int it) {
        const int s = it % STAGES;
        const int64_t g = kb_begin + it;
        const int t = static_cast<int>(g / a.kblocks);
        const int kb = static_cast<int>(g - static_cast<int64_t>(t) * a.kblocks);
        tma_load_2d(sB + s * B_STAGE, &tmX, &full[s], kb * BK, (t % a.mt) * BN, pol_x);  // row tile
      };
      // Weights do not depend on the previous kernel: start streaming them before the
      // grid-dependency wait, then add the activation tiles to the same stages.
      const int pro = my_kb < STAGES ? my_kb : STAGES;
      for (int it = 0; it < pro; ++it) {
        mbar_arrive_expect_tx(&full[it], STAGE_BYTES);
        load_w(it);
      }
      pdl_wait();
      if (tp.wait != nullptr) {
        // X is written by every rank (all-gathered rows): wait for all of them, then make the
        // acquired data visible to the TMA (async proxy) reads below.
        wait_counters(tp.wait, tp.nranks, static_cast<uint32_t>(*tp.epoch) * tp.wait_count, a.err);
        fence_proxy_async_global();
      }
      for (int it = 0; it < pro; ++it) load_x(it);
      issued = pro;
      for (int it = pro; it < my_kb; ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, a.err)) break;
        mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
        load_w(it);
        load_x(it);
        issued = it + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && my_kb > 0) {
      int it = 0, seg = 0;
      int64_t kb = kb_begin;
      bool ok = true;
      while (ok && kb < kb_end) {
        const int t = static_cast<int>(kb / a.kblocks);
        const int64_t seg_end = min(kb_end, static_cast<int64_t>(t + 1) * a.kblocks);
        const int ab = seg & 1;
        if (!mbar_wait(&acce[ab], ((seg >> 1) & 1) ^ 1, abort_flag, a.err)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(ab * BN);
        for (int64_t g = kb; g < seg_end; ++g, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full[s], ph, abort_flag, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = umma_desc_sw128(smem_u32(sA + s * A_STAGE));
          const uint64_t bd = umma_desc_sw128(smem_u32(sB + s * B_STAGE));
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_bf16(d, ad + 2 * kk, bd + 2 * kk, IDESC, (g > kb || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&accf[ab]);
        kb = seg_end;
        ++seg;
      }
      // Drain: every MMA issued above has completed before TMEM is released.
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, a.err);
    }
  } else {
    // Epilogue warps 2..5: warp w reads TMEM lanes 32*(w%4) .. 32*(w%4)+31.
    pdl_wait();
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int e = threadIdx.x - 64;
    int seg = 0;
    int64_t kb = kb_begin;
    while (kb < kb_end) {
      const int t = static_cast<int>(kb / a.kblocks);
      const int64_t tile_lo = static_cast<int64_t>(t) * a.kblocks;
      const int64_t seg_end = min(kb_end, tile_lo + a.kblocks);
      const int ab = seg & 1;
      if (!mbar_wait(&accf[ab], (seg >> 1) & 1, abort_flag, a.err)) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(ab * BN);
      const bool full_tile = (kb == tile_lo) && (seg_end == tile_lo + a.kblocks);
      if (a.epilogue == MVB_EPI_PARTIALS || a.epilogue == MVB_EPI_SWIGLU_PARTIALS) {
        // Every segment's fp32 accumulator goes to its (tile, contributor) slot; the consuming
        // kernel sums the slots (no fence, counter or merge here).
        const int j = static_cast<int>(blockIdx.x) - cta_of(tile_lo, total, G);
        if (tp.nranks > 0 && tp.recv[0] != nullptr) {
          // push: batch row b goes to the receive area of the rank that owns it
          const int rpr = tp.rows_per_rank;
          const int64_t base = ((static_cast<int64_t>(tp.rank) * a.tiles + t) * a.maxc + j) * rpr;
          for (int c0 = 0; c0 < BN && c0 < a.m; c0 += 32) {
            uint32_t r[32];
            tmem_ld_x32(tb + c0, r);
            tmem_ld_wait();
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) {
              const int b = c0 + jj;
              if (b < a.m) {
                const int q = b / rpr;
                tp.recv[q][(base + (b - q * rpr)) * BM + row] = __uint_as_float(r[jj]);
              }
            }
          }
        } else {
          float* part = a.partials + (static_cast<int64_t>(t) * a.maxc + j) * BN * BM;
          for (int c0 = 0; c0 < BN; c0 += 32) {
            uint32_t r[32];
            tmem_ld_x32(tb + c0, r);
            tmem_ld_wait();
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) part[(c0 + jj) * BM + row] = __uint_as_float(r[jj]);
          }
        }
      } else if (full_tile) {
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t r[32];
          tmem_ld_x32(tb + c0, r);
          tmem_ld_wait();
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          epilogue_store<BN>(a, tp, v, t / a.mt, row, c0, xbuf, (t % a.mt) * BN);
        }
      } else {
        const int slot = seg == 0 ? 2 * blockIdx.x : 2 * blockIdx.x + 1;
        float* part = a.partials + static_cast<int64_t>(slot) * BN * BM;
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t r[32];
          tmem_ld_x32(tb + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) __stcg(part + (c0 + j) * BM + row, __uint_as_float(r[j]));
        }
        __threadfence();
        epi_bar();
        if (e == 0) {
          const int c_first = cta_of(tile_lo, total, G);
          const int c_last = cta_of(tile_lo + a.kblocks - 1, total, G);
          const int old = atomicAdd(&a.counters[t], 1);
          const int last = (old == c_last - c_first);
          if (last) __threadfence();
          *last_flag = last;
        }
        epi_bar();
        if (*last_flag) {
          const int c_first = cta_of(tile_lo, total, G);
          const int c_last = cta_of(tile_lo + a.kblocks - 1, total, G);
          for (int c0 = 0; c0 < BN; c0 += 32) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.0f;
            for (int c = c_first; c <= c_last; ++c) {
              const int sl = range_start(c, total, G) >= tile_lo ? 2 * c : 2 * c + 1;
              const float* p = a.partials + static_cast<int64_t>(sl) * BN * BM;
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += __ldcg(p + (c0 + j) * BM + row);
            }
            epilogue_store<BN>(a, tp, v, t / a.mt, row, c0, xbuf, (t % a.mt) * BN);
          }
          if (e == 0) a.counters[t] = 0;
        }
        epi_bar();
      }
      tc_fence_before();
      mbar_arrive(&acce[ab]);
      kb = seg_end;
      ++seg;
    }
    if (tp.nranks > 0 && tp.signal[0] != nullptr) {
      epi_bar();  // every store of this CTA's epilogue threads
      if (e == 0) signal_ranks_once(tp.arrive, tp.arrive_total, tp.signal, tp.nranks);
    }
  }

  __syncthreads();
  if (warp == 0 && lane == 0) {
    // Wait (bounded) for the copies still in flight when a wait gave up.
    const int first = issued > STAGES ? issued - STAGES : 0;
    for (int it = first; it < issued; ++it) mbar_wait(&full[it % STAGES], (it / STAGES) & 1, nullptr, a.err);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// Prefill GEMMs (more than 256 rows, an even number of weight tiles): 256 x 256 output tiles, two
// weight tiles (UMMA M = 128 each) against one 256-row activation box.  Per k-block a CTA loads
// 64 KB for 2 x 128 x 256 x 64 multiply-adds, two thirds of the bytes per product of the 128 x 256
// tile, whose operand traffic from L2 holds the tensor pipe near 55 %.  The two accumulators fill
// TMEM (512 columns), so a tile's epilogue does not overlap the next tile's MMAs; eight epilogue
// warps (a TMEM lane quarter of one accumulator each) keep it short.  Tiles are whole and
// weight-major, a contiguous range per CTA: no split-K, no merge, the same sums on any grid.
constexpr int kRowsThreads = 320;  // warp 0 TMA, warp 1 TMEM + MMA, warps 2-9 epilogue
constexpr int kRowsStages = 3;

template <int STAGES>
__global__ void __launch_bounds__(kRowsThreads, 1)
    gemm_rows_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                     const GemmArgs a, const __grid_constant__ TpGemm tp) {
  constexpr int BN = 256;
  constexpr int B_STAGE = BN * BK * 2;                     // 32 KB
  constexpr uint32_t STAGE_BYTES = 2 * A_STAGE + B_STAGE;  // 64 KB
  constexpr uint32_t TMEM_COLS = 2 * BN;                   // accumulators of weight tiles 2tw, 2tw + 1
  constexpr uint32_t IDESC = umma_idesc_bf16(BM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                    // [stage][half] 16 KB weight boxes
  uint8_t* sB = sA + STAGES * 2 * A_STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;  // accumulators full (MMA -> epilogue)
  uint64_t* acce = accf + 1;        // accumulators drained (epilogue -> MMA)
  uint64_t* drain = acce + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xbuf = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES + 256);  // 2 x 64 x 33 floats (SWIGLU)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t_begin = static_cast<int>(range_start(blockIdx.x, a.tiles, gridDim.x));
  const int t_end = static_cast<int>(range_start(blockIdx.x + 1, a.tiles, gridDim.x));
  const int my_kb = (t_end - t_begin) * a.kblocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    mbar_init(acce, kRowsThreads - 64);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) pdl_launch_dependents();

  int issued = 0;  // producer: loads issued
  if (warp == 0) {
    if (lane == 0 && my_kb > 0) {
      prefetch_tmap(&tmW);
      prefetch_tmap(&tmX);
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      const bool swiglu = a.epilogue == MVB_EPI_SWIGLU;
      auto load_w = [&](int it) {
        const int s = it % STAGES;
        const int lt = t_begin + it / a.kblocks;
        const int kb = it % a.kblocks;
        const int tw = lt / a.mt;  // weight tiles 2tw, 2tw + 1
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint8_t* dst = sA + (s * 2 + h) * A_STAGE;
          const int t = 2 * tw + h;
          if (swiglu) {
            tma_load_2d(dst, &tmW, &full[s], kb * BK, 64 * t, pol_w);
            tma_load_2d(dst + A_STAGE / 2, &tmW, &full[s], kb * BK, a.inter + 64 * t, pol_w);
          } else {
            tma_load_2d(dst, &tmW, &full[s], kb * BK, BM * t, pol_w);
          }
        }
      };
      auto load_x = [&](int it) {
        const int s = it % STAGES;
        const int lt = t_begin + it / a.kblocks;
        const int kb = it % a.kblocks;
        tma_load_2d(sB + s * B_STAGE, &tmX, &full[s], kb * BK, (lt % a.mt) * BN, pol_x);  // row tile
      };
      // Weights do not depend on the previous kernel: start streaming them before the
      // grid-dependency wait, then add the activation boxes to the same stages.
      const int pro = my_kb < STAGES ? my_kb : STAGES;
      for (int it = 0; it < pro; ++it) {
        mbar_arrive_expect_tx(&full[it], STAGE_BYTES);
        load_w(it);
      }
      pdl_wait();
      for (int it = 0; it < pro; ++it) load_x(it);
      issued = pro;
      for (int it = pro; it < my_kb; ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, a.err)) break;
        mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
        load_w(it);
        load_x(it);
        issued = it + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && my_kb > 0) {
      int it = 0;
      bool ok = true;
      for (int lt = t_begin; ok && lt < t_end; ++lt) {
        const int seg = lt - t_begin;
        if (!mbar_wait(acce, (seg & 1) ^ 1, abort_flag, a.err)) break;
        tc_fence_after();
        for (int kb = 0; kb < a.kblocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full[s], ph, abort_flag, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t a0 = umma_desc_sw128(smem_u32(sA + (s * 2) * A_STAGE));
          const uint64_t a1 = umma_desc_sw128(smem_u32(sA + (s * 2 + 1) * A_STAGE));
          const uint64_t bd = umma_desc_sw128(smem_u32(sB + s * B_STAGE));
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
            umma_bf16(tmem_base, a0 + 2 * kk, bd + 2 * kk, IDESC, acc);
            umma_bf16(tmem_base + BN, a1 + 2 * kk, bd + 2 * kk, IDESC, acc);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(accf);
      }
      // Drain: every MMA issued above has completed before TMEM is released.
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, a.err);
    }
  } else {
    // Epilogue warps 2..9: warp w reads TMEM lanes 32*(w%4) .. +31 of accumulator h = (w-2)/4.
    pdl_wait();
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    float* xb = xbuf + h * 64 * 33;
    for (int lt = t_begin; lt < t_end; ++lt) {
      const int seg = lt - t_begin;
      if (!mbar_wait(accf, seg & 1, abort_flag, a.err)) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(h * BN);
      const int t = 2 * (lt / a.mt) + h;
      const int r0 = (lt % a.mt) * BN;
      for (int c0 = 0; c0 < BN && r0 + c0 < a.m; c0 += 32) {
        uint32_t r[32];
        tmem_ld_x32(tb + c0, r);
        tmem_ld_wait();
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if (h == 0)
          epilogue_store<BN, 1>(a, tp, v, t, row, c0, xb, r0);
        else
          epilogue_store<BN, 2>(a, tp, v, t, row, c0, xb, r0);
      }
      tc_fence_before();
      mbar_arrive(acce);
    }
  }

  __syncthreads();
  if (warp == 0 && lane == 0) {
    // Wait (bounded) for the copies still in flight when a wait gave up.
    const int first = issued > STAGES ? issued - STAGES : 0;
    for (int it = first; it < issued; ++it) mbar_wait(&full[it % STAGES], (it / STAGES) & 1, nullptr, a.err);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

size_t rows_smem() {
  return static_cast<size_t>(kRowsStages) * (2 * A_STAGE + 256 * BK * 2) + 256 + 2 * 64 * 33 * 4 + 1024;
}

int launch_gemm_rows(const CUtensorMap& tw, const CUtensorMap& tx, const GemmArgs& a, const TpGemm& tp, int grid,
                     cudaStream_t st) {
  const size_t smem = rows_smem();
  static unsigned long long done_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(done_mask & (1ull << dev))) {
    MVB_TRY(set_smem(gemm_rows_kernel<kRowsStages>, smem, "gemm: smem attribute"));
    if (dev < 64) done_mask |= 1ull << dev;
  }
  return launch("gemm_bf16_rows", gemm_rows_kernel<kRowsStages>, dim3(grid), dim3(kRowsThreads), smem, st, tw, tx,
                a, tp);
}

template <int BN>
constexpr int stages_for() {
  return BN == 64 ? 4 : (BN == 128 ? 6 : 4);
}

template <int BN>
size_t smem_for() {
  return static_cast<size_t>(stages_for<BN>()) * (A_STAGE + BN * BK * 2) + 256 + 64 * 33 * 4 + 1024;
}

int bn_for(int64_t m) { return m <= 64 ? 64 : (m <= 128 ? 128 : 256); }

bool swiglu_tiling(int epilogue) { return epilogue == MVB_EPI_SWIGLU || epilogue == MVB_EPI_SWIGLU_PARTIALS; }
bool partials_out(int epilogue) { return epilogue == MVB_EPI_PARTIALS || epilogue == MVB_EPI_SWIGLU_PARTIALS; }

int64_t tiles_for(int64_t n, int epilogue) { return swiglu_tiling(epilogue) ? (n / 2 + 63) / 64 : (n + BM - 1) / BM; }

int64_t counters_bytes(int64_t tiles) { return (tiles * 4 + 255) / 256 * 256; }

template <int BN>
int launch_gemm(const CUtensorMap& tw, const CUtensorMap& tx, const GemmArgs& a, const TpGemm& tp, int grid,
                cudaStream_t st) {
  constexpr int S = stages_for<BN>();
  const size_t smem = smem_for<BN>();
  // Once per device and instantiation, so no attribute call happens during graph capture.
  static unsigned long long done_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(done_mask & (1ull << dev))) {
    MVB_TRY(set_smem(gemm_bf16_kernel<BN, S>, smem, "gemm: smem attribute"));
    if (dev < 64) done_mask |= 1ull << dev;
  }
  return launch("gemm_bf16", gemm_bf16_kernel<BN, S>, dim3(grid), dim3(kThreads), smem, st, tw, tx, a, tp);
}

}  // namespace
}  // namespace mvb

using namespace mvb;

extern "C" int64_t mvb_gemm_workspace_bytes(int64_t m, int64_t n, int64_t k, int device) {
  (void)k;
  int sms = mvb_num_sms(device);
  if (sms <= 0) sms = 148;
  const int64_t bn = bn_for(m);
  // Counters sized for the larger of the two tilings (plain / SWIGLU pairs), times the row tiles.
  const int64_t tiles = (n + 63) / 64 * ((m + bn - 1) / bn);
  const int64_t merge = counters_bytes(tiles) + 2LL * splitk_ctas(m, sms) * bn * BM * 4 + 256;
  int64_t part = splitk_partials_bytes(splitk_plan(m, n, k, sms)) + 256;
  if (n % 2 == 0) {
    const int64_t sw = splitk_partials_bytes(splitk_plan_swiglu(m, n / 2, k, sms)) + 256;
    if (sw > part) part = sw;
  }
  return merge > part ? merge : part;
}

namespace mvb {

// Shared body of mvb_gemm_bf16 and mvb_tp_gemm_bf16; `max_ctas` > 0 caps the CTA count (the
// split-K plan follows), `grid_out` receives the CTA count.
int gemm_launch(void* y, int64_t ldy, const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t m, int64_t n,
                int64_t k, int epilogue, const void* aux, int64_t ld_aux, void* workspace, int64_t workspace_bytes,
                const TpGemm& tp, int64_t max_ctas, int* grid_out, mvb_stream_t stream) {
  MVB_REQUIRE(x && w && workspace && (y || partials_out(epilogue) || (tp.nranks > 0 && tp.y[0])),
              "mvb_gemm_bf16: null pointer");
  MVB_REQUIRE(m > 0 && m < (1LL << 24), "mvb_gemm_bf16: m=%lld", (long long)m);
  MVB_REQUIRE(m <= 256 || (!partials_out(epilogue) && tp.nranks == 0),
              "mvb_gemm_bf16: m=%lld > 256 needs a STORE, SWIGLU or RESADD epilogue on one GPU", (long long)m);
  MVB_REQUIRE(n > 0 && n < (1LL << 31) && k > 0 && k % BK == 0, "mvb_gemm_bf16: need k %% 64 == 0 (k=%lld)",
              (long long)k);
  MVB_REQUIRE(ldx >= k && ldw >= k && ldx % 8 == 0 && ldw % 8 == 0, "mvb_gemm_bf16: ldx/ldw must be >= k, %% 8");
  MVB_REQUIRE(aligned(x, 16) && aligned(w, 16), "mvb_gemm_bf16: x and w must be 16-byte aligned");
  MVB_REQUIRE(epilogue == MVB_EPI_STORE || epilogue == MVB_EPI_SWIGLU || epilogue == MVB_EPI_RESADD ||
                  partials_out(epilogue),
              "mvb_gemm_bf16: bad epilogue %d", epilogue);
  MVB_REQUIRE(epilogue != MVB_EPI_RESADD || (aux != nullptr && ld_aux >= n), "mvb_gemm_bf16: RESADD needs aux");
  MVB_REQUIRE(!swiglu_tiling(epilogue) || n % 2 == 0, "mvb_gemm_bf16: SWIGLU needs an even n (= 2*inter)");
  const int64_t out_cols = epilogue == MVB_EPI_SWIGLU ? n / 2 : n;
  MVB_REQUIRE(partials_out(epilogue) || ldy >= out_cols, "mvb_gemm_bf16: ldy < output columns");
  const int sms = current_sm_count();
  MVB_REQUIRE(sms > 0, "mvb_gemm_bf16: no device");
  const int bn = bn_for(m);
  const int64_t mt = (m + bn - 1) / bn;  // row tiles
  const int64_t tiles = tiles_for(n, epilogue) * mt;
  const int64_t kblocks = k / BK;
  const int64_t total = tiles * kblocks;
  int64_t ctas = splitk_ctas(m, sms);
  if (max_ctas > 0 && max_ctas < ctas) ctas = max_ctas;
  // The merge path's last-arriving CTA sums a tile's contributors one after another: a GEMM with
  // so few tiles that each would have more than 16 contributors (a 128-expert router: 32) is
  // spread over 8 CTAs per tile instead.
  if (!partials_out(epilogue) && ctas > tiles * 16) ctas = tiles * 8;
  const int grid = static_cast<int>(total < ctas ? total : ctas);
  // Partials at the head, tile counters at the tail of the workspace: calls of any shape
  // that share one buffer then use nested suffixes of the same (self-zeroing) counter area,
  // never bytes that another call used for partials.
  const int64_t ws_end = workspace_bytes / 256 * 256;
  const int64_t cbytes = counters_bytes((n + 63) / 64 * mt);
  SplitKPlan plan{};
  if (partials_out(epilogue)) plan = splitk_plan_ctas(m, static_cast<int>(tiles), k, ctas);
  const int64_t need = partials_out(epilogue) ? splitk_partials_bytes(plan) : cbytes + 2LL * grid * bn * BM * 4;
  MVB_REQUIRE(ws_end >= need, "mvb_gemm_bf16: workspace %lld < %lld bytes", (long long)workspace_bytes,
              (long long)need);
  MVB_REQUIRE(aligned(workspace, 256), "mvb_gemm_bf16: workspace must be 256-byte aligned");

  CUtensorMap tw, tx;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(n)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldw) * 2};
    const uint32_t box[2] = {BK, static_cast<uint32_t>(swiglu_tiling(epilogue) ? 64 : BM)};
    MVB_TRY(encode_tiled(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B));
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldx) * 2};
    const uint32_t box[2] = {BK, static_cast<uint32_t>(bn)};
    MVB_TRY(encode_tiled(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B));
  }
  GemmArgs a;
  a.y = static_cast<__nv_bfloat16*>(y);
  a.ldy = ldy;
  a.aux = static_cast<const __nv_bfloat16*>(aux);
  a.ld_aux = ld_aux;
  a.m = static_cast<int>(m);
  a.n = static_cast<int>(n);
  a.k = static_cast<int>(k);
  a.tiles = static_cast<int>(tiles);
  a.mt = static_cast<int>(mt);
  a.kblocks = static_cast<int>(kblocks);
  a.epilogue = epilogue;
  a.inter = static_cast<int>(n / 2);
  a.maxc = plan.maxc;
  a.partials = static_cast<float*>(workspace);
  a.counters = reinterpret_cast<int*>(static_cast<char*>(workspace) + ws_end - cbytes);
  a.err = device_status_ptr();
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t wtiles = tiles_for(n, epilogue);
  if (mt > 1 && wtiles % 2 == 0) {
    // Prefill rows: 256 x 256 tiles (weight tiles 2tw, 2tw + 1 against one row tile), whole.
    a.tiles = static_cast<int>(wtiles / 2 * mt);
    const int rgrid = a.tiles < sms ? a.tiles : sms;
    if (grid_out) *grid_out = rgrid;
    return launch_gemm_rows(tw, tx, a, tp, rgrid, st);
  }
  if (grid_out) *grid_out = grid;
  switch (bn) {
    case 64: return launch_gemm<64>(tw, tx, a, tp, grid, st);
    case 128: return launch_gemm<128>(tw, tx, a, tp, grid, st);
    default: return launch_gemm<256>(tw, tx, a, tp, grid, st);
  }
}

}  // namespace mvb

extern "C" int mvb_gemm_bf16(void* y, int64_t ldy, const void* x, int64_t ldx, const void* w, int64_t ldw,
                             int64_t m, int64_t n, int64_t k, int epilogue, const void* aux, int64_t ld_aux,
                             void* workspace, int64_t workspace_bytes, mvb_stream_t stream) {
  TpGemm tp{};
  return gemm_launch(y, ldy, x, ldx, w, ldw, m, n, k, epilogue, aux, ld_aux, workspace, workspace_bytes, tp, 0,
                     nullptr, stream);
}
