// Sparse mixture-of-experts MLP of one decode step (Qwen3-MoE): routing, dispatch, grouped
// expert GEMMs on tcgen05, and the weighted combine.
//
// Replaces Qwen3MoeSparseMoe.forward (models/qwen3_moe_model.py:39-65):
//   probs = softmax(gate(x)); top-k; renormalise (norm_topk_prob)
//   for each expert e (ascending) with tokens: out_e = down(silu(gate_e(x)) * up_e(x))
//     final[token] += w * out_e[token]        (model dtype, one rounding per addition)
//
//  * mvb_moe_route (one CTA): fp32 softmax of the bf16 router logits (the reference's GPU decode
//    runs under CUDA autocast, where softmax computes in fp32), top-k with ties to the lower
//    expert index, renormalisation, and the dispatch order: the (token, slot) pairs sorted by
//    expert, tokens ascending inside an expert.  Active experts are listed in ascending order.
//  * mvb_moe_gather: the rows of x in dispatch order.
//  * mvb_moe_gemm_bf16: one grouped GEMM over the active experts only.  A work unit is one
//    128-row tile of one expert's weight matrix with all of its k-blocks (no split-K: an expert
//    at decode batch sizes has a handful of tokens, so there are hundreds of units to spread
//    over the SMs); each CTA loops over units.  The expert's rows of the dispatched activations
//    are the UMMA N operand (swap-AB, as in the dense decode GEMM).  SWIGLU epilogue for
//    gate/up, plain store for down.
//  * mvb_moe_combine: per token, its experts in ascending index, acc = bf16(acc + w * out).
//
// Expert parallelism across the GPUs of a tensor-parallel group: every rank routes all tokens
// (the same router weights and the all-gathered activations give the same routing everywhere),
// runs the grouped GEMMs over its own experts only (mvb_moe_gemm_bf16_experts), and
// mvb_tp_moe_combine sums each token's slots on its experts and pushes the partial sum to the rank
// that owns the token's row, whose add+norm (mvb_tp_fused_add_rmsnorm_gemm) adds the ranks'
// partials.  No activation rows cross GPUs before the experts.
#include "common.cuh"
#include "host.h"
#include "splitk.cuh"
#include "tp.cuh"

namespace mvb {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int A_STAGE = BM * BK * 2;  // 16 KB
constexpr int kThreads = 192;
constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 16;
constexpr int kMaxRows = 256;

struct MoeGemmArgs {
  __nv_bfloat16* y;
  int64_t ldy;
  int kblocks;
  int rows_per_expert;  // rows of one expert's weight matrix (2*inter for SWIGLU)
  int n_out;            // output columns (inter for SWIGLU)
  int tiles_pe;         // work units per expert
  int swiglu;
  const int32_t* expert_off;  // [E + 1] first dispatched row of each expert
  const int32_t* active;      // [1 + E]: count, then the active experts ascending
  int first_expert;           // expert parallel: this GPU holds experts first_expert ..
  int local_experts;          //   first_expert + local_experts - 1 (weights indexed from first_expert)
  unsigned* err;
};

// Index range [i0, i1) of the ascending active list (active[1 .. n]) holding the experts
// first .. first + count - 1 (binary searches: the list is sorted).
__device__ __forceinline__ void local_active_range(const int32_t* active, int n, int first, int count, int& i0,
                                                   int& i1) {
  auto lower = [&](int v) {
    int lo = 0, hi = n;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (active[1 + mid] < v)
        lo = mid + 1;
      else
        hi = mid;
    }
    return lo;
  };
  i0 = lower(first);
  i1 = lower(first + count);
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, BN == 64 ? 2 : 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                    const MoeGemmArgs a) {
  constexpr int B_STAGE = BN * BK * 2;
  constexpr uint32_t STAGE_BYTES = A_STAGE + B_STAGE;
  constexpr uint32_t TMEM_COLS = 2 * BN;
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
  float* xbuf = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES + 256);  // 64 x 33 floats (SWIGLU)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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
  pdl_wait();  // the routing (active experts, dispatch offsets) and x come from earlier kernels
  int i0 = 0, i1 = 0;
  local_active_range(a.active, a.active[0], a.first_expert, a.local_experts, i0, i1);
  const int total = (i1 - i0) * a.tiles_pe;
  const int G = gridDim.x;

  int issued = 0;
  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmW);
      prefetch_tmap(&tmX);
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < total; u += G) {
        const int e = a.active[1 + i0 + u / a.tiles_pe];
        const int t = u % a.tiles_pe;
        const int xrow = a.expert_off[e];
        const int wrow = (e - a.first_expert) * a.rows_per_expert;
        for (int kb = 0; kb < a.kblocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, a.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          if (a.swiglu) {
            tma_load_2d(sA + s * A_STAGE, &tmW, &full[s], kb * BK, wrow + 64 * t, pol_w);
            tma_load_2d(sA + s * A_STAGE + A_STAGE / 2, &tmW, &full[s], kb * BK, wrow + a.n_out + 64 * t, pol_w);
          } else {
            tma_load_2d(sA + s * A_STAGE, &tmW, &full[s], kb * BK, wrow + BM * t, pol_w);
          }
          tma_load_2d(sB + s * B_STAGE, &tmX, &full[s], kb * BK, xrow, pol_x);
          issued = it + 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, seg = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < total; u += G, ++seg) {
        const int ab = seg & 1;
        if (!mbar_wait(&acce[ab], ((seg >> 1) & 1) ^ 1, abort_flag, a.err)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(ab * BN);
        for (int kb = 0; kb < a.kblocks; ++kb, ++it) {
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
          for (int kk = 0; kk < BK / 16; ++kk) umma_bf16(d, ad + 2 * kk, bd + 2 * kk, IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&accf[ab]);
      }
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, a.err);
    }
  } else {
    // Epilogue warps 2..5: warp w reads TMEM lanes 32*(w%4) .. +31 (weight rows of the tile).
    const int q = warp & 3;
    const int row = q * 32 + lane;
    int seg = 0;
    for (int u = blockIdx.x; u < total; u += G, ++seg) {
      const int e = a.active[1 + i0 + u / a.tiles_pe];
      const int t = u % a.tiles_pe;
      const int xrow = a.expert_off[e];
      const int n_e = a.expert_off[e + 1] - xrow;  // dispatched rows of this expert (<= BN)
      const int ab = seg & 1;
      if (!mbar_wait(&accf[ab], (seg >> 1) & 1, abort_flag, a.err)) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(ab * BN);
      for (int c0 = 0; c0 < BN && c0 < n_e; c0 += 32) {
        uint32_t r[32];
        tmem_ld_x32(tb + c0, r);
        tmem_ld_wait();
        if (a.swiglu) {
          // lanes 0-63: gate features 64t + r, lanes 64-127: the matching up features
          const bool is_up = row >= 64;
          const int rr = row & 63;
          if (is_up) {
#pragma unroll
            for (int j = 0; j < 32; ++j) xbuf[rr * 33 + j] = bf16_round(__uint_as_float(r[j]));
          }
          epi_bar();
          if (!is_up) {
            const int f = 64 * t + rr;
            if (f < a.n_out) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (c0 + j < n_e) {
                  const float g = bf16_round(__uint_as_float(r[j]));
                  const float sg = bf16_round(silu_f(g));
                  a.y[static_cast<int64_t>(xrow + c0 + j) * a.ldy + f] = __float2bfloat16_rn(sg * xbuf[rr * 33 + j]);
                }
              }
            }
          }
          epi_bar();
        } else {
          const int nn = t * BM + row;
          if (nn < a.n_out) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (c0 + j < n_e)
                a.y[static_cast<int64_t>(xrow + c0 + j) * a.ldy + nn] = __float2bfloat16_rn(__uint_as_float(r[j]));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acce[ab]);
    }
  }

  __syncthreads();
  if (warp == 0 && lane == 0) {
    const int first = issued > STAGES ? issued - STAGES : 0;
    for (int it = first; it < issued; ++it) mbar_wait(&full[it % STAGES], (it / STAGES) & 1, nullptr, a.err);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------- routing
// One CTA: every warp routes tokens (softmax, top-k, renormalisation), then the dispatch order is
// built from per-expert counts (thread e lists expert e's tokens in ascending token order).
__global__ void __launch_bounds__(1024) moe_route_kernel(const __nv_bfloat16* __restrict__ logits, int rows, int E,
                                                        int K, int norm, int32_t* topk_ids, float* topk_w,
                                                        int32_t* pair_row, int32_t* row_token, int32_t* expert_off,
                                                        int32_t* active) {
  __shared__ int s_ids[kMaxRows * kMaxTopK];
  __shared__ int s_cnt[kMaxExperts];
  __shared__ int s_off[kMaxExperts + 1];
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  constexpr int PER = kMaxExperts / 32;
  for (int b = warp; b < rows; b += nw) {
    float p[PER];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      p[i] = e < E ? __bfloat162float(logits[static_cast<int64_t>(b) * E + e]) : -INFINITY;
      m = fmaxf(m, p[i]);
    }
    m = warp_max(m);
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      p[i] = lane + 32 * i < E ? expf(p[i] - m) : 0.0f;
      sum += p[i];
    }
    sum = warp_sum(sum);
#pragma unroll
    for (int i = 0; i < PER; ++i) p[i] = lane + 32 * i < E ? p[i] / sum : -1.0f;
    float top_v[kMaxTopK];
    int top_i[kMaxTopK];
    for (int k = 0; k < K; ++k) {
      // lane-local best (lowest expert index among equals), then across the warp
      float bv = -2.0f;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < PER; ++i)
        if (p[i] > bv) {
          bv = p[i];
          bi = lane + 32 * i;
        }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      top_v[k] = bv;
      top_i[k] = bi;
#pragma unroll
      for (int i = 0; i < PER; ++i)
        if (lane + 32 * i == bi) p[i] = -1.0f;
    }
    float denom = 1.0f;
    if (norm) {
      denom = 0.0f;
      for (int k = 0; k < K; ++k) denom += top_v[k];
    }
    if (lane == 0) {
      for (int k = 0; k < K; ++k) {
        topk_ids[b * K + k] = top_i[k];
        topk_w[b * K + k] = norm ? top_v[k] / denom : top_v[k];
        s_ids[b * K + k] = top_i[k];
      }
    }
  }
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < rows * K; i += blockDim.x) atomicAdd(&s_cnt[s_ids[i]], 1);
  __syncthreads();
  if (warp == 0) {
    // Prefix sums of the counts (row offsets) and of the active flags (active list), PER experts
    // per lane, then across the warp.
    int cnt[PER], run = 0, act = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane * PER + i;
      cnt[i] = e < E ? s_cnt[e] : 0;
      run += cnt[i];
      act += cnt[i] > 0;
    }
    int incl = run, iact = act;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      const int va = __shfl_up_sync(0xffffffffu, iact, o);
      if (lane >= o) {
        incl += v;
        iact += va;
      }
    }
    int off = incl - run, n = iact - act;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane * PER + i;
      if (e < E) {
        s_off[e] = off;
        expert_off[e] = off;
        if (cnt[i] > 0) active[1 + n++] = e;
        off += cnt[i];
      }
    }
    if (lane == 31) {
      s_off[E] = incl;
      expert_off[E] = incl;
      active[0] = iact;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int r = s_off[e];
    for (int b = 0; b < rows; ++b)
      for (int k = 0; k < K; ++k)
        if (s_ids[b * K + k] == e) {
          pair_row[b * K + k] = r;
          row_token[r] = b;
          ++r;
        }
  }
}

// out[r] = x[row_token[r]], 8 bf16 per thread.
__global__ void moe_gather_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ x, int hidden,
                                  const int32_t* __restrict__ row_token) {
  pdl_launch_dependents();
  pdl_wait();
  const int r = blockIdx.x;
  const int tok = row_token[r];
  const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(tok) * hidden);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<int64_t>(r) * hidden);
  for (int i = threadIdx.x; i < hidden / 8; i += blockDim.x) dst[i] = src[i];
}

// Per token: its experts in ascending index, acc = bf16(acc + w * out) (one rounding per add,
// the reference's final[token] += w * out with fp32 routing weights).  8 features per thread.
__global__ void moe_combine_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ y,
                                   const float* __restrict__ topk_w, const int32_t* __restrict__ topk_ids,
                                   const int32_t* __restrict__ pair_row, int K, int hidden, int first_expert,
                                   int local_experts) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x;
  int ord[kMaxTopK];
  for (int k = 0; k < K; ++k) ord[k] = k;
  for (int i = 1; i < K; ++i) {  // insertion sort of the slots by expert index
    const int v = ord[i];
    int j = i - 1;
    while (j >= 0 && topk_ids[b * K + ord[j]] > topk_ids[b * K + v]) {
      ord[j + 1] = ord[j];
      --j;
    }
    ord[j + 1] = v;
  }
  for (int i = threadIdx.x * 8; i < hidden; i += blockDim.x * 8) {
    float acc[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = 0.0f;
    for (int kk = 0; kk < K; ++kk) {
      const int k = ord[kk];
      const int e = topk_ids[b * K + k];
      if (e < first_expert || e - first_expert >= local_experts) continue;   // another GPU's expert
      const float w = topk_w[b * K + k];
      const uint4 v = *reinterpret_cast<const uint4*>(y + static_cast<int64_t>(pair_row[b * K + k]) * hidden + i);
      const __nv_bfloat16* ve = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
      for (int c = 0; c < 8; ++c)  // product and sum rounded separately, as the reference's two ops
        acc[c] = bf16_round(__fadd_rn(acc[c], __fmul_rn(w, __bfloat162float(ve[c]))));
    }
    uint4 o;
    __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
    for (int c = 0; c < 8; ++c) oe[c] = __float2bfloat16_rn(acc[c]);
    *reinterpret_cast<uint4*>(out + static_cast<int64_t>(b) * hidden + i) = o;
  }
}

// Expert parallel combine: a token's slots on this GPU's experts only (ascending expert index, the
// same rounding as moe_combine_kernel), pushed as fp32 into the receive area of the row's owner
// (sk_push_offset of a one-contributor plan: tiles of 128 features, contributor 0); then every
// rank is signalled once.  A token none of whose experts live here pushes zeros.
struct MoePush {
  int nranks, rank, rpr;
  SplitKPlan plan;
  float* recv[kTpMaxRanks];
  uint32_t* signal[kTpMaxRanks];
  uint32_t* arrive;
  int first_expert, local_experts;
};

__global__ void moe_combine_push_kernel(const __nv_bfloat16* __restrict__ y, const float* __restrict__ topk_w,
                                        const int32_t* __restrict__ topk_ids, const int32_t* __restrict__ pair_row,
                                        int K, int hidden, const __grid_constant__ MoePush mp) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x;
  int ord[kMaxTopK];
  for (int k = 0; k < K; ++k) ord[k] = k;
  for (int i = 1; i < K; ++i) {  // insertion sort of the slots by expert index
    const int v = ord[i];
    int j = i - 1;
    while (j >= 0 && topk_ids[b * K + ord[j]] > topk_ids[b * K + v]) {
      ord[j + 1] = ord[j];
      --j;
    }
    ord[j + 1] = v;
  }
  const int q = b / mp.rpr, bl = b - q * mp.rpr;
  float* dst = mp.recv[q];
  for (int i = threadIdx.x * 8; i < hidden; i += blockDim.x * 8) {
    float acc[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = 0.0f;
    for (int kk = 0; kk < K; ++kk) {
      const int k = ord[kk];
      const int e = topk_ids[b * K + k];
      if (e < mp.first_expert || e >= mp.first_expert + mp.local_experts) continue;
      const float w = topk_w[b * K + k];
      const uint4 v = *reinterpret_cast<const uint4*>(y + static_cast<int64_t>(pair_row[b * K + k]) * hidden + i);
      const __nv_bfloat16* ve = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
      for (int c = 0; c < 8; ++c) acc[c] = bf16_round(__fadd_rn(acc[c], __fmul_rn(w, __bfloat162float(ve[c]))));
    }
    const int t = i / kSplitBM, r = i - t * kSplitBM;
    float4* o = reinterpret_cast<float4*>(dst + sk_push_offset(mp.plan, mp.rank, t, 0, mp.rpr, bl, r));
    o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
  __syncthreads();
  if (threadIdx.x == 0) signal_ranks_once(mp.arrive, gridDim.x, mp.signal, mp.nranks);
}

template <int BN>
constexpr int moe_stages() {
  return BN == 64 ? 4 : (BN == 128 ? 6 : 4);
}

template <int BN>
size_t moe_smem() {
  return static_cast<size_t>(moe_stages<BN>()) * (A_STAGE + BN * BK * 2) + 256 + 64 * 33 * 4 + 1024;
}

template <int BN>
int launch_moe_gemm(const CUtensorMap& tw, const CUtensorMap& tx, const MoeGemmArgs& a, int grid, cudaStream_t st) {
  constexpr int S = moe_stages<BN>();
  static unsigned long long done_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(done_mask & (1ull << dev))) {
    MVB_TRY(set_smem(moe_gemm_kernel<BN, S>, moe_smem<BN>(), "moe_gemm: smem attribute"));
    if (dev < 64) done_mask |= 1ull << dev;
  }
  return launch("moe_gemm_bf16", moe_gemm_kernel<BN, S>, dim3(grid), dim3(kThreads), moe_smem<BN>(), st, tw, tx, a);
}

}  // namespace
}  // namespace mvb

using namespace mvb;

extern "C" int mvb_moe_route(const void* logits, int64_t rows, int64_t num_experts, int64_t top_k, int norm_topk,
                             int32_t* topk_ids, float* topk_w, int32_t* pair_row, int32_t* row_token,
                             int32_t* expert_off, int32_t* active, mvb_stream_t stream) {
  MVB_REQUIRE(logits && topk_ids && topk_w && pair_row && row_token && expert_off && active,
              "mvb_moe_route: null pointer");
  MVB_REQUIRE(rows > 0 && rows <= kMaxRows && num_experts > 0 && num_experts <= kMaxExperts && top_k > 0 &&
                  top_k <= kMaxTopK && top_k <= num_experts,
              "mvb_moe_route: rows %lld (<= %d), experts %lld (<= %d), top_k %lld (<= %d)", (long long)rows, kMaxRows,
              (long long)num_experts, kMaxExperts, (long long)top_k, kMaxTopK);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // one warp per row, up to 32 warps
  const int threads = static_cast<int>((rows < 32 ? rows : 32) * 32 < 256 ? 256 : (rows < 32 ? rows : 32) * 32);
  return launch("moe_route", moe_route_kernel, dim3(1), dim3(threads), 0, st, (const __nv_bfloat16*)logits, (int)rows,
                (int)num_experts, (int)top_k, norm_topk, topk_ids, topk_w, pair_row, row_token, expert_off, active);
}

extern "C" int mvb_moe_gather(void* out, const void* x, int64_t hidden, const int32_t* row_token, int64_t nrows,
                              mvb_stream_t stream) {
  MVB_REQUIRE(out && x && row_token, "mvb_moe_gather: null pointer");
  MVB_REQUIRE(hidden > 0 && hidden % 8 == 0 && nrows > 0 && aligned(out, 16) && aligned(x, 16),
              "mvb_moe_gather: hidden %% 8 == 0 and 16-byte aligned rows required");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return launch("moe_gather", moe_gather_kernel, dim3(static_cast<unsigned>(nrows)), dim3(256), 0, st,
                (__nv_bfloat16*)out, (const __nv_bfloat16*)x, (int)hidden, row_token);
}

extern "C" int mvb_moe_gemm_bf16_experts(void* y, int64_t ldy, const void* x, int64_t ldx, const void* w,
                                         int64_t n_per_expert, int64_t k, int64_t num_experts, int64_t first_expert,
                                         int64_t local_experts, int64_t nrows, int64_t max_rows_per_expert,
                                         int epilogue, const int32_t* expert_off, const int32_t* active,
                                         mvb_stream_t stream) {
  MVB_REQUIRE(y && x && w && expert_off && active, "mvb_moe_gemm_bf16: null pointer");
  MVB_REQUIRE(first_expert >= 0 && local_experts > 0 && first_expert + local_experts <= num_experts,
              "mvb_moe_gemm_bf16: experts %lld + %lld of %lld", (long long)first_expert, (long long)local_experts,
              (long long)num_experts);
  MVB_REQUIRE(epilogue == MVB_EPI_STORE || epilogue == MVB_EPI_SWIGLU, "mvb_moe_gemm_bf16: epilogue %d", epilogue);
  MVB_REQUIRE(k > 0 && k % BK == 0 && n_per_expert > 0 && num_experts > 0 && num_experts <= kMaxExperts && nrows > 0,
              "mvb_moe_gemm_bf16: bad shape");
  MVB_REQUIRE(max_rows_per_expert > 0 && max_rows_per_expert <= 256, "mvb_moe_gemm_bf16: <= 256 rows per expert");
  const bool swiglu = epilogue == MVB_EPI_SWIGLU;
  MVB_REQUIRE(!swiglu || n_per_expert % 128 == 0, "mvb_moe_gemm_bf16: SWIGLU needs 2*inter, inter %% 64 == 0");
  const int64_t n_out = swiglu ? n_per_expert / 2 : n_per_expert;
  MVB_REQUIRE(ldy >= n_out && ldx >= k && ldx % 8 == 0 && aligned(x, 16) && aligned(w, 16),
              "mvb_moe_gemm_bf16: strides / alignment");
  const int sms = current_sm_count();
  MVB_REQUIRE(sms > 0, "mvb_moe_gemm_bf16: no device");
  const int bn = max_rows_per_expert <= 64 ? 64 : (max_rows_per_expert <= 128 ? 128 : 256);
  CUtensorMap tw, tx;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(local_experts * n_per_expert)};
    const uint64_t strides[1] = {static_cast<uint64_t>(k) * 2};
    const uint32_t box[2] = {BK, static_cast<uint32_t>(swiglu ? 64 : BM)};
    MVB_TRY(encode_tiled(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(nrows)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldx) * 2};
    const uint32_t box[2] = {BK, static_cast<uint32_t>(bn)};
    MVB_TRY(encode_tiled(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  MoeGemmArgs a;
  a.y = static_cast<__nv_bfloat16*>(y);
  a.ldy = ldy;
  a.kblocks = static_cast<int>(k / BK);
  a.rows_per_expert = static_cast<int>(n_per_expert);
  a.n_out = static_cast<int>(n_out);
  a.tiles_pe = static_cast<int>(swiglu ? (n_out + 63) / 64 : (n_out + BM - 1) / BM);
  a.swiglu = swiglu ? 1 : 0;
  a.expert_off = expert_off;
  a.active = active;
  a.first_expert = static_cast<int>(first_expert);
  a.local_experts = static_cast<int>(local_experts);
  a.err = device_status_ptr();
  // The active-expert count is known on the device only: enough CTAs for every unit of all
  // experts, two per SM at BN = 64; CTAs without a unit exit after the prologue.
  const int64_t max_units = local_experts * a.tiles_pe;
  const int64_t ctas = bn == 64 ? 2LL * sms : sms;
  const int grid = static_cast<int>(max_units < ctas ? max_units : ctas);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (bn) {
    case 64: return launch_moe_gemm<64>(tw, tx, a, grid, st);
    case 128: return launch_moe_gemm<128>(tw, tx, a, grid, st);
    default: return launch_moe_gemm<256>(tw, tx, a, grid, st);
  }
}

extern "C" int mvb_moe_gemm_bf16(void* y, int64_t ldy, const void* x, int64_t ldx, const void* w, int64_t n_per_expert,
                                 int64_t k, int64_t num_experts, int64_t nrows, int64_t max_rows_per_expert,
                                 int epilogue, const int32_t* expert_off, const int32_t* active,
                                 mvb_stream_t stream) {
  return mvb_moe_gemm_bf16_experts(y, ldy, x, ldx, w, n_per_expert, k, num_experts, 0, num_experts, nrows,
                                   max_rows_per_expert, epilogue, expert_off, active, stream);
}

extern "C" int mvb_moe_combine(void* out, const void* y, const float* topk_w, const int32_t* topk_ids,
                               const int32_t* pair_row, int64_t rows, int64_t top_k, int64_t hidden,
                               mvb_stream_t stream) {
  MVB_REQUIRE(out && y && topk_w && topk_ids && pair_row, "mvb_moe_combine: null pointer");
  MVB_REQUIRE(rows > 0 && top_k > 0 && top_k <= kMaxTopK && hidden > 0 && hidden % 8 == 0 && aligned(out, 16) &&
                  aligned(y, 16),
              "mvb_moe_combine: bad shape or alignment");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return launch("moe_combine", moe_combine_kernel, dim3(static_cast<unsigned>(rows)), dim3(256), 0, st,
                (__nv_bfloat16*)out, (const __nv_bfloat16*)y, topk_w, topk_ids, pair_row, (int)top_k, (int)hidden, 0,
                kMaxExperts);
}

extern "C" int mvb_moe_combine_experts(void* out, const void* y, const float* topk_w, const int32_t* topk_ids,
                                       const int32_t* pair_row, int64_t rows, int64_t top_k, int64_t hidden,
                                       int64_t first_expert, int64_t local_experts, mvb_stream_t stream) {
  MVB_REQUIRE(out && y && topk_w && topk_ids && pair_row, "mvb_moe_combine_experts: null pointer");
  MVB_REQUIRE(rows > 0 && top_k > 0 && top_k <= kMaxTopK && hidden > 0 && hidden % 8 == 0 && aligned(out, 16) &&
                  aligned(y, 16) && first_expert >= 0 && local_experts > 0,
              "mvb_moe_combine_experts: bad shape, alignment or expert range");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return launch("moe_combine", moe_combine_kernel, dim3(static_cast<unsigned>(rows)), dim3(256), 0, st,
                (__nv_bfloat16*)out, (const __nv_bfloat16*)y, topk_w, topk_ids, pair_row, (int)top_k, (int)hidden,
                (int)first_expert, (int)local_experts);
}

extern "C" int mvb_tp_moe_combine(mvb_tp_comm* comm, const void* y, const float* topk_w, const int32_t* topk_ids,
                                  const int32_t* pair_row, int64_t rows, int64_t top_k, int64_t hidden,
                                  int64_t first_expert, int64_t local_experts, int64_t recv_offset, int signal_point,
                                  mvb_stream_t stream) {
  MVB_REQUIRE(comm && y && topk_w && topk_ids && pair_row, "mvb_tp_moe_combine: null pointer");
  const int nr = comm->nranks;
  MVB_REQUIRE(rows > 0 && rows <= kMaxRows && rows % nr == 0 && top_k > 0 && top_k <= kMaxTopK && hidden > 0 &&
                  hidden % kSplitBM == 0 && aligned(y, 16),
              "mvb_tp_moe_combine: rows %lld (a multiple of %d ranks), hidden %lld (a multiple of %d)",
              (long long)rows, nr, (long long)hidden, kSplitBM);
  MVB_REQUIRE(first_expert >= 0 && local_experts > 0, "mvb_tp_moe_combine: expert range");
  MVB_REQUIRE(signal_point >= 0 && signal_point < kTpMaxPoints, "mvb_tp_moe_combine: signal point");
  const int sms = current_sm_count();
  MVB_REQUIRE(sms > 0, "mvb_tp_moe_combine: no device");
  MoePush mp{};
  mp.nranks = nr;
  mp.rank = comm->rank;
  mp.rpr = static_cast<int>(rows / nr);
  mp.plan = splitk_plan_push(rows, hidden, kSplitBK, sms, nr);   // one k-block: one contributor per tile
  MVB_REQUIRE(recv_offset >= kTpSignalBytes && recv_offset % 16 == 0 &&
                  recv_offset + splitk_push_bytes(mp.plan, nr, mp.rpr) <= comm->heap_bytes,
              "mvb_tp_moe_combine: receive area outside the heap");
  for (int q = 0; q < nr; ++q) {
    mp.recv[q] = reinterpret_cast<float*>(comm->base[q] + recv_offset);
    mp.signal[q] = comm->signal_slot(q, signal_point);
  }
  mp.arrive = comm->arrive_slot(signal_point);
  mp.first_expert = static_cast<int>(first_expert);
  mp.local_experts = static_cast<int>(local_experts);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MVB_TRY(launch("tp_moe_combine", moe_combine_push_kernel, dim3(static_cast<unsigned>(rows)), dim3(256), 0, st,
                 (const __nv_bfloat16*)y, topk_w, topk_ids, pair_row, (int)top_k, (int)hidden, mp));
  comm->point_count[signal_point] = 1;   // one signal per rank per step
  return MVB_OK;
}
