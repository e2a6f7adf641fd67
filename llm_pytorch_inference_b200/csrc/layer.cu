// Fused decoder-layer kernel: everything of a dense decode layer after its attention, plus the
// next layer's q|k|v projection, in one persistent launch.
//
// The unfused step runs, per layer, o_proj GEMM -> residual add + RMSNorm -> gate_up GEMM ->
// SwiGLU finalize -> down GEMM -> residual add + RMSNorm -> (next layer) q|k|v GEMM -> QK-norm +
// RoPE + KV write, eight launches whose boundaries each cost a few microseconds of ramp, drain and
// dependency wait while HBM idles.  Here one persistent grid (two CTAs per SM) runs them as phases
// (models/model.py:315-328 with model.py:154-243 of the next layer):
//
//   GEMM phase  o_proj  (X = attention output)      -> fp32 split-K partials
//   consumer    residual += o_proj; xn = RMSNorm(residual; post_attention_layernorm)
//   GEMM phase  gate_up (X = xn, SwiGLU-paired rows) -> h = silu(gate) * up, by each tile's
//               contributor 0 in its epilogue (no separate pass)
//   GEMM phase  down    (X = h)                     -> partials
//   consumer    residual += down;  xn = RMSNorm(residual; next input_layernorm | final norm)
//   GEMM phase  q|k|v of the next layer (X = xn)    -> partials      (absent after the last layer)
//   consumer    QK-norm + RoPE + paged KV write of the next layer
//
// Phases are separated by grid-wide barriers (all CTAs are resident: two per SM).  The TMA
// producer streams the weights of a phase as soon as shared-memory stages free
// up -- weights do not depend on the previous phase -- and only the activation tiles wait for the
// barrier, so HBM keeps streaming through the barriers and consumers.  Each GEMM phase is a
// stream-K split over the grid (splitk_plan_ctas) with fp32 partials per contributor, summed by the
// consumers in contributor order (deterministic); the results agree with the unfused kernels to
// bf16 rounding (a different split and a different order of the sum of squares).
//
// Tensor parallel (mvb_tp_decoder_layer_tail): the same phases on a rank's shards; o_proj and
// down_proj are row-parallel, so each tile's contributor 0 pushes the rank's sum of the tile to
// the owners of its batch rows, the owners add and normalise their rows and write them into
// every rank's xn, and signal points (system-scope release / acquire) order the ranks.
//
// Every wait is bounded (mbarrier waits, grid barriers, contributor flags, other ranks' signals):
// a wait that runs out sets the kDevWaitTimeout status bit, the CTA unwinds, waits for its copies
// in flight and frees its TMEM.
#include <algorithm>

#include "common.cuh"
#include "host.h"
#include "qk_rope.cuh"
#include "splitk.cuh"
#include "tp.cuh"

namespace mvb {
namespace {

constexpr int LBM = 128;               // UMMA M: weight rows per tile
constexpr int LBK = 64;                // k per stage
constexpr int LBN = 64;                // UMMA N: batch columns (decode batches of <= 64 rows)
constexpr int LSTAGES = 4;         // two CTAs per SM: 2 x 4 x 16 KB of weights in flight per SM
constexpr int LA = LBM * LBK * 2;      // 16 KB of weights per stage
constexpr int LB = LBN * LBK * 2;      // 8 KB of activations per stage
constexpr uint32_t LSTAGE = LA + LB;
constexpr int kLayerThreads = 192;     // warp 0 TMA, warp 1 TMEM + MMA, warps 2-5 epilogue + consumers
constexpr int kMaxPhases = 4;
constexpr int kLayerMaxHidden = 4096;  // add+norm rows held in the 128 epilogue threads' registers

// What follows a GEMM phase: residual add + RMSNorm over the grid; SwiGLU in the epilogue of each
// tile's contributor 0 (no consumer pass); QK-norm + RoPE + KV write over the grid; tensor
// parallel: partials pushed to the ranks that own the batch rows, the owners' residual add +
// RMSNorm of their rows written into every rank's activations.
enum : int { kConsAddNorm = 0, kConsSwiglu = 1, kConsQk = 2, kConsTpAddNorm = 3 };

struct LayerPhase {
  SplitKPlan plan;   // stream-K split over the launch's grid (plan.grid <= gridDim.x)
  float* partials;   // this phase's partial slots
  int swiglu;        // W rows paired: tile t = gate rows 64t.. | up rows inter + 64t..
  int inter;         // SwiGLU: gate rows of W
  int consumer;      // kCons*
};

struct LayerArgs {
  int m;                          // batch rows
  int nphase;
  LayerPhase ph[kMaxPhases];
  // residual stream and activations
  __nv_bfloat16* residual;        // [m, hidden]
  __nv_bfloat16* xn;              // [m, hidden]: the next GEMM's input
  __nv_bfloat16* h;               // [m, inter]
  int hidden;
  int inter;
  const __nv_bfloat16* norm_w[2]; // RMSNorm weights of the two add+norm consumers
  float eps;
  float* ss;                      // [m * kNormChunks] per-chunk sums of squares
  unsigned* flags;                // [tiles][maxc] of a reduced phase: partial written (launch + phase stamp)
  // QK-norm + RoPE + KV write of the next layer
  __nv_bfloat16* q_out;
  __nv_bfloat16* kv;
  const __nv_bfloat16* qnw;
  const __nv_bfloat16* knw;
  const __nv_bfloat16* cos_t;
  const __nv_bfloat16* sin_t;
  int64_t table_len;
  const int32_t* positions;
  const int32_t* block_tables;
  int64_t max_blocks;
  int nq, nkv;
  int64_t next_layer;
  int64_t num_blocks;
  int bs;
  // grid barrier: uint32 arrival count at bar[0], the launch's base count at bar[32] (separate
  // 128-byte lines)
  unsigned* bar;
  unsigned* err;
  // tensor parallel (nranks > 0): row-parallel o_proj / down_proj push their partials to the
  // owners of the batch rows (rows_per_rank each); each owner adds and normalises its rows and
  // writes them into every rank's xn; four signal points per launch (0: o_proj pushed, 1: rows
  // gathered, 2: down_proj pushed, 3: rows gathered), each signalled once per rank per step.
  int nranks, rank, rpr;
  const float* recv[2];                   // this rank's receive areas (o_proj, down_proj)
  float* push[2][kTpMaxRanks];            // every rank's receive area of the two pushes
  SplitKPlan push_plan[2];                // their layout: one (summed) contribution per rank and tile
  __nv_bfloat16* xn_all[kTpMaxRanks];     // every rank's xn
  uint32_t* signal[4][kTpMaxRanks];       // rank q's counter [point][this rank]
  const uint32_t* wait[4];                // this rank's counters [point][0..nranks)
  const int32_t* epoch;                   // the step counter (signals per point so far)
};

struct LayerMaps {
  CUtensorMap w[kMaxPhases];
  CUtensorMap x[kMaxPhases];
};

__device__ __forceinline__ uint32_t ld_acquire_gpu(const unsigned* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_gpu(unsigned* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid barriers count arrivals on one word that only grows: every CTA adds 1 (a release) per
// barrier, and barrier n of a launch is complete once the count reaches base + n * ctas, where
// base is the count when the launch started.  CTA 0 publishes the next launch's base (bar[32]) once
// the launch's last barrier is complete; the next launch reads it only after this one has ended.

// Bounded wait until the arrival count reaches `target` (wrap-around compare).  Relaxed polls
// (one thread per CTA), then one acquire fence.
__device__ __forceinline__ bool wait_count(const unsigned* count, uint32_t target, volatile int* abort_flag,
                                           unsigned* err) {
  const unsigned long long t0 = globaltimer_ns();
  unsigned polls = 0;
  while (static_cast<int32_t>(ld_relaxed_gpu(count) - target) < 0) {
    __nanosleep(32);
    if ((++polls & 15u) == 0) {
      if (abort_flag != nullptr && *abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        report(err, kDevWaitTimeout);
        if (abort_flag != nullptr) *abort_flag = 1;
        return false;
      }
    }
  }
  fence_acq_rel_gpu();
  return true;
}

// One thread per CTA, after a barrier over the CTA's stores: arrive (the release covers the CTA's
// stores ordered before it by that barrier) and wait for all CTAs.
__device__ __forceinline__ bool grid_barrier(unsigned* count, uint32_t target, volatile int* abort_flag,
                                             unsigned* err) {
  asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(count) : "memory");
  return wait_count(count, target, abort_flag, err);
}

// Named barrier of the 128 epilogue threads.
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Residual add + RMSNorm (model semantics, model.py:19-25, :319) from the partials of `plan`, in
// two passes over work units u = (row b, chunk c) of the row's 128-feature tiles, one unit per CTA
// at a time (kNormChunks chunks per row, so 4 x 64 rows keep 256 CTAs busy):
//   pass 1: v = bf16(sum of partials), residual = bf16(residual + v) stored, the chunk's sum of
//           squares to ss[u];
//   (grid barrier)
//   pass 2: r = 1 / sqrt(sum of the row's chunk sums in chunk order / hidden + eps),
//           out = bf16(w * (residual * r)).
constexpr int kNormChunks = 4;

__device__ __forceinline__ int norm_chunks(int tiles) { return tiles < kNormChunks ? tiles : kNormChunks; }

__device__ void add_norm_pass1(const LayerArgs& a, const SplitKPlan& p, const float* partials, int u, int warp4,
                               int lane, float* red) {
  const int T = a.hidden / kSplitBM, C = norm_chunks(T), tpc = (T + C - 1) / C;
  const int b = u / C, c = u - b * C;
  const int t_end = min(T, (c + 1) * tpc);
  __nv_bfloat16* res = a.residual + static_cast<int64_t>(b) * a.hidden;
  float ss = 0.0f;
  for (int t = c * tpc + warp4; t < t_end; t += 8) {
    const int t2 = t + 4;
    float4 s1, s2;
    sk_sum4_x2(partials, p, t, b, 4 * lane, t2, b, 4 * lane, t2 < t_end, s1, s2);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int tt = k == 0 ? t : t2;
      if (tt >= t_end) break;
      const float4 sv = k == 0 ? s1 : s2;
      const int i = tt * kSplitBM + 4 * lane;
      const uint2 rr = __ldcg(reinterpret_cast<const uint2*>(res + i));
      const __nv_bfloat162 r01 = *reinterpret_cast<const __nv_bfloat162*>(&rr.x);
      const __nv_bfloat162 r23 = *reinterpret_cast<const __nv_bfloat162*>(&rr.y);
      const float v0 = bf16_round(__low2float(r01) + bf16_round(sv.x));
      const float v1 = bf16_round(__high2float(r01) + bf16_round(sv.y));
      const float v2 = bf16_round(__low2float(r23) + bf16_round(sv.z));
      const float v3 = bf16_round(__high2float(r23) + bf16_round(sv.w));
      __nv_bfloat162 o01 = __floats2bfloat162_rn(v0, v1);
      __nv_bfloat162 o23 = __floats2bfloat162_rn(v2, v3);
      uint2 ov;
      ov.x = *reinterpret_cast<uint32_t*>(&o01);
      ov.y = *reinterpret_cast<uint32_t*>(&o23);
      __stcg(reinterpret_cast<uint2*>(res + i), ov);
      ss += v0 * v0 + v1 * v1 + v2 * v2 + v3 * v3;
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp4] = ss;
  epi_sync();
  if (warp4 == 0 && lane == 0) a.ss[u] = red[0] + red[1] + red[2] + red[3];
  epi_sync();   // red is reused by the next unit
}

__device__ void add_norm_pass2(const LayerArgs& a, const __nv_bfloat16* w, int u, int warp4, int lane) {
  const int T = a.hidden / kSplitBM, C = norm_chunks(T), tpc = (T + C - 1) / C;
  const int b = u / C, c = u - b * C;
  const int t_end = min(T, (c + 1) * tpc);
  float total = 0.0f;
  for (int k = 0; k < C; ++k) total += __ldcg(a.ss + b * C + k);
  const float rr = 1.0f / sqrtf(total / static_cast<float>(a.hidden) + a.eps);
  const __nv_bfloat16* res = a.residual + static_cast<int64_t>(b) * a.hidden;
  __nv_bfloat16* out = a.xn + static_cast<int64_t>(b) * a.hidden;
  for (int t = c * tpc + warp4; t < t_end; t += 4) {
    const int i = t * kSplitBM + 4 * lane;
    const uint2 rv = __ldcg(reinterpret_cast<const uint2*>(res + i));
    const uint2 wv = *reinterpret_cast<const uint2*>(w + i);
    const __nv_bfloat162 r01 = *reinterpret_cast<const __nv_bfloat162*>(&rv.x);
    const __nv_bfloat162 r23 = *reinterpret_cast<const __nv_bfloat162*>(&rv.y);
    const __nv_bfloat162 w01 = *reinterpret_cast<const __nv_bfloat162*>(&wv.x);
    const __nv_bfloat162 w23 = *reinterpret_cast<const __nv_bfloat162*>(&wv.y);
    __nv_bfloat162 o01 = __floats2bfloat162_rn(bf16_round(__low2float(w01) * (__low2float(r01) * rr)),
                                               bf16_round(__high2float(w01) * (__high2float(r01) * rr)));
    __nv_bfloat162 o23 = __floats2bfloat162_rn(bf16_round(__low2float(w23) * (__low2float(r23) * rr)),
                                               bf16_round(__high2float(w23) * (__high2float(r23) * rr)));
    uint2 ov;
    ov.x = *reinterpret_cast<uint32_t*>(&o01);
    ov.y = *reinterpret_cast<uint32_t*>(&o23);
    __stcg(reinterpret_cast<uint2*>(out + i), ov);
  }
}

__device__ __forceinline__ float silu_l(float x) { return x / (1.0f + expf(-x)); }

// Bounded wait until a contributor flag holds `want` (the launch's stamp).
__device__ __forceinline__ bool wait_flag(const unsigned* flag, uint32_t want, volatile int* abort_flag, unsigned* err) {
  const unsigned long long t0 = globaltimer_ns();
  unsigned polls = 0;
  while (ld_relaxed_gpu(flag) != want) {
    __nanosleep(32);
    if ((++polls & 15u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        report(err, kDevWaitTimeout);
        *abort_flag = 1;
        return false;
      }
    }
  }
  fence_acq_rel_gpu();
  return true;
}

// The producer's bounded wait until the epilogue has passed `target` grid barriers.
__device__ __forceinline__ bool wait_passed(volatile uint32_t* nbar_s, uint32_t target, volatile int* abort_flag,
                                            unsigned* err) {
  const unsigned long long t0 = globaltimer_ns();
  unsigned polls = 0;
  while (*nbar_s < target) {
    __nanosleep(20);
    if ((++polls & 15u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        report(err, kDevWaitTimeout);
        *abort_flag = 1;
        return false;
      }
    }
  }
  __threadfence_block();
  return true;
}

// Bounded wait until every rank's counter counters[0..n) reaches `target` (signals from other
// GPUs: system-scope acquire polls; a system-scope fence here would cost microseconds per CTA).
__device__ __forceinline__ bool wait_ranks(const uint32_t* counters, int n, uint32_t target, volatile int* abort_flag,
                                           unsigned* err) {
  const unsigned long long t0 = globaltimer_ns();
  for (int s = 0; s < n; ++s) {
    unsigned polls = 0;
    while (static_cast<int32_t>(ld_acquire_sys(counters + s) - target) < 0) {
      __nanosleep(64);
      if ((++polls & 15u) == 0) {
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          report(err, kDevWaitTimeout);
          *abort_flag = 1;
          return false;
        }
      }
    }
  }
  return true;
}

// Tensor parallel: the owner's residual add + RMSNorm of its owned row `bl` (batch row
// rank * rpr + bl), one CTA's 128 epilogue threads per row: the pushed partials summed over
// source ranks, then contributors (the order of norm.cu's tensor-parallel fused_add_rmsnorm),
// residual += bf16(sum), out = bf16(w * (residual * r)) stored into every rank's xn.  The new
// residual row waits in shared memory (vs, bf16 [hidden]) for the row's 1 / rms.
constexpr int kTpNormRuns = kLayerMaxHidden / (4 * 128);

__device__ void tp_add_norm_row(const LayerArgs& a, const SplitKPlan& p, const float* __restrict__ recv,
                                const __nv_bfloat16* __restrict__ w, int bl, int e, float* red,
                                __nv_bfloat16* vs) {
  const int b = a.rank * a.rpr + bl;
  __nv_bfloat16* res = a.residual + static_cast<int64_t>(b) * a.hidden;
  const int runs = a.hidden / 4;
  float ss = 0.0f;
  for (int k0 = 0; k0 < kTpNormRuns; k0 += 2) {
    float4 acc[2];
    uint2 rv[2];
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      const int run = e + 128 * (k0 + kk);
      acc[kk] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (run < runs) {
        const int i = run * 4;
        const int t = i / kSplitBM, r = i - t * kSplitBM;
        const int nc = sk_count(p, t);
        rv[kk] = __ldcg(reinterpret_cast<const uint2*>(res + i));
        for (int src = 0; src < a.nranks; ++src)
          for (int j = 0; j < nc; ++j) {
            const float4 q =
                __ldcg(reinterpret_cast<const float4*>(recv + sk_push_offset(p, src, t, j, a.rpr, bl, r)));
            acc[kk].x += q.x;
            acc[kk].y += q.y;
            acc[kk].z += q.z;
            acc[kk].w += q.w;
          }
      }
    }
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      const int run = e + 128 * (k0 + kk);
      if (run < runs) {
        const int i = run * 4;
        const __nv_bfloat162 r01 = *reinterpret_cast<const __nv_bfloat162*>(&rv[kk].x);
        const __nv_bfloat162 r23 = *reinterpret_cast<const __nv_bfloat162*>(&rv[kk].y);
        const float v0 = bf16_round(__low2float(r01) + bf16_round(acc[kk].x));
        const float v1 = bf16_round(__high2float(r01) + bf16_round(acc[kk].y));
        const float v2 = bf16_round(__low2float(r23) + bf16_round(acc[kk].z));
        const float v3 = bf16_round(__high2float(r23) + bf16_round(acc[kk].w));
        __nv_bfloat162 o01 = __floats2bfloat162_rn(v0, v1);
        __nv_bfloat162 o23 = __floats2bfloat162_rn(v2, v3);
        uint2 ov;
        ov.x = *reinterpret_cast<uint32_t*>(&o01);
        ov.y = *reinterpret_cast<uint32_t*>(&o23);
        __stcg(reinterpret_cast<uint2*>(res + i), ov);
        *reinterpret_cast<uint2*>(vs + i) = ov;
        ss += v0 * v0 + v1 * v1 + v2 * v2 + v3 * v3;
      }
    }
  }
  ss = warp_sum(ss);
  if ((e & 31) == 0) red[e >> 5] = ss;
  epi_sync();
  const float total = red[0] + red[1] + red[2] + red[3];
  const float rs = 1.0f / sqrtf(total / static_cast<float>(a.hidden) + a.eps);
  for (int run = e; run < runs; run += 128) {
    const int i = run * 4;
    const uint2 vv = *reinterpret_cast<const uint2*>(vs + i);
    const uint2 wv = *reinterpret_cast<const uint2*>(w + i);
    const __nv_bfloat162 v01 = *reinterpret_cast<const __nv_bfloat162*>(&vv.x);
    const __nv_bfloat162 v23 = *reinterpret_cast<const __nv_bfloat162*>(&vv.y);
    const __nv_bfloat162 w01 = *reinterpret_cast<const __nv_bfloat162*>(&wv.x);
    const __nv_bfloat162 w23 = *reinterpret_cast<const __nv_bfloat162*>(&wv.y);
    __nv_bfloat162 o01 = __floats2bfloat162_rn(bf16_round(__low2float(w01) * (__low2float(v01) * rs)),
                                               bf16_round(__high2float(w01) * (__high2float(v01) * rs)));
    __nv_bfloat162 o23 = __floats2bfloat162_rn(bf16_round(__low2float(w23) * (__low2float(v23) * rs)),
                                               bf16_round(__high2float(w23) * (__high2float(v23) * rs)));
    uint2 ov;
    ov.x = *reinterpret_cast<uint32_t*>(&o01);
    ov.y = *reinterpret_cast<uint32_t*>(&o23);
    const int64_t off = static_cast<int64_t>(b) * a.hidden + i;
    for (int q = 0; q < a.nranks; ++q) *reinterpret_cast<uint2*>(a.xn_all[q] + off) = ov;
  }
  epi_sync();   // red and vs are reused by the next row
}

// SwiGLU of one gate_up tile (64 gate rows | the 64 matching up rows, 64 batch columns) by the
// tile's contributor 0 in its epilogue: each epilogue thread holds one tile row, sums its
// accumulator (TMEM) and the other contributors' partials in contributor order (the order of
// sk_sum4, so the sums equal the unfused path's), the up rows pass bf16(u) to the gate rows
// through shared memory (xs), the gate rows put h = bf16(silu(bf16 g) * bf16 u)
// (elementwise.cu's swiglu_gemm_kernel) into a [64 batch rows][64 features] tile (hs), and all
// 128 threads store it as 16-byte row pieces.  Every thread runs the four epi_sync calls whatever
// `go` is.
// Contributor 0's sum of tile row `row`, batch columns c0 .. c0 + 15: its own accumulator (TMEM)
// first, then contributors 1 .. n-1 in order (the order of sk_sum4), two contributors' loads in
// flight together.  Sixteen columns at a time keep the sum and the loads in registers.
__device__ __forceinline__ void reduce_chunk16(const LayerPhase& ph, int t, int n, int c0, int row, uint32_t tb,
                                               float* v) {
  uint32_t r[16];
  tmem_ld_x16(tb + c0, r);
  tmem_ld_wait();
#pragma unroll
  for (int jj = 0; jj < 16; ++jj) {
    v[jj] = 0.0f;
    v[jj] += __uint_as_float(r[jj]);
  }
  const float* base = ph.partials + (static_cast<int64_t>(t) * ph.plan.maxc * LBN + c0) * LBM + row;
  constexpr int64_t kContrib = static_cast<int64_t>(LBN) * LBM;
  for (int q = 1; q < n; q += 2) {
    const bool two = q + 1 < n;
    float x0[16], x1[16];
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) x0[jj] = __ldcg(base + q * kContrib + jj * LBM);
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) x1[jj] = two ? __ldcg(base + (q + 1) * kContrib + jj * LBM) : 0.0f;
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) v[jj] += x0[jj];
    if (two) {
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) v[jj] += x1[jj];
    }
  }
}

// Columns c0 .. c0 + 31 (two 16-column sums).
__device__ __forceinline__ void reduce_chunk(const LayerPhase& ph, int t, int n, int c0, int row, uint32_t tb,
                                             float (&v)[32]) {
  reduce_chunk16(ph, t, n, c0, row, tb, v);
  reduce_chunk16(ph, t, n, c0 + 16, row, tb, v + 16);
}

__device__ __forceinline__ void swiglu_tile(const LayerArgs& a, const LayerPhase& ph, int t, int n, uint32_t tb,
                                            int row, int e, bool go, __nv_bfloat16* xs, __nv_bfloat16* hs) {
  for (int c0 = 0; c0 < LBN; c0 += 32) {
    float v[32];
    if (go) {
      reduce_chunk(ph, t, n, c0, row, tb, v);
      if (row >= 64) {
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) xs[jj * 64 + row - 64] = __float2bfloat16_rn(v[jj]);
      }
    }
    epi_sync();
    if (go && row < 64) {
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const float g = bf16_round(silu_l(bf16_round(v[jj])));
        hs[(c0 + jj) * 64 + row] = __float2bfloat16_rn(g * __bfloat162float(xs[jj * 64 + row]));
      }
    }
    epi_sync();   // xs is reused; after the second chunk, hs is complete
  }
  if (go) {
    // 64 rows x 128 bytes: 512 pieces of 16 bytes, 4 per thread
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int idx = e + 128 * k, b = idx >> 3, piece = idx & 7;
      if (b < a.m)
        *reinterpret_cast<uint4*>(a.h + static_cast<int64_t>(b) * a.inter + t * 64 + piece * 8) =
            reinterpret_cast<const uint4*>(hs)[idx];
    }
  }
}

// Tensor parallel: contributor 0 of a row-parallel tile sums the tile over this rank's
// contributors and pushes the sum of every batch row to the receive area of the row's owner
// (one-contributor layout `pp`), so NVLink carries one tile per rank, not one per contributor.
__device__ __forceinline__ void push_tile(const LayerArgs& a, const LayerPhase& ph, const SplitKPlan& pp,
                                          float* const* dst, int t, int n, uint32_t tb, int row) {
  for (int c0 = 0; c0 < LBN; c0 += 16) {
    float v[16];
    reduce_chunk16(ph, t, n, c0, row, tb, v);
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) {
      const int b = c0 + jj;
      if (b < a.m) {
        const int q = b / a.rpr, bl = b - q * a.rpr;
        dst[q][sk_push_offset(pp, a.rank, t, 0, a.rpr, bl, row)] = v[jj];
      }
    }
  }
}

// Stream-K range of phase p for this CTA: k-blocks [kb0, kb0 + nkb) of the linear (tile, k-block)
// space, empty when the phase's split uses fewer CTAs than the grid.
__device__ __forceinline__ void phase_range(const SplitKPlan& p, int cta, int64_t& kb0, int& nkb) {
  const int64_t total = static_cast<int64_t>(p.tiles) * p.kblocks;
  if (cta >= p.grid) {
    kb0 = 0;
    nkb = 0;
    return;
  }
  kb0 = sk_range_start(cta, total, p.grid);
  nkb = static_cast<int>(sk_range_start(cta + 1, total, p.grid) - kb0);
}

// Grid barriers of phase p: its partials are complete (not for SwiGLU, finished per tile); for an
// add+norm consumer, its first pass is complete; except after the last phase, the phase's output
// is complete.
__device__ __forceinline__ uint32_t phase_bars(const LayerArgs& a, int p) {
  const int c = a.ph[p].consumer;
  const bool last = p + 1 == a.nphase;
  if (c == kConsSwiglu) return last ? 0u : 1u;
  if (c == kConsTpAddNorm) return 2u;   // pushes issued; gathered rows written
  return 1u + (c == kConsAddNorm ? 1u : 0u) + (last ? 0u : 1u);
}
// Synchronisation points of phase p: its grid barriers, and for a tensor-parallel add+norm the
// waits for every rank's signal (pushed; unless last, gathered).  The producer loads a phase's
// activations once the epilogue has passed every point before it.
__device__ __forceinline__ uint32_t phase_syncs(const LayerArgs& a, int p) {
  return phase_bars(a, p) + (a.ph[p].consumer == kConsTpAddNorm ? (p + 1 == a.nphase ? 1u : 2u) : 0u);
}
__device__ __forceinline__ uint32_t bars_before(const LayerArgs& a, int p) {
  uint32_t n = 0;
  for (int q = 0; q < p; ++q) n += phase_bars(a, q);
  return n;
}
__device__ __forceinline__ uint32_t syncs_before(const LayerArgs& a, int p) {
  uint32_t n = 0;
  for (int q = 0; q < p; ++q) n += phase_syncs(a, q);
  return n;
}

__global__ void __launch_bounds__(kLayerThreads, 2)
    layer_kernel(const __grid_constant__ LayerMaps maps, const __grid_constant__ LayerArgs a) {
  constexpr uint32_t IDESC = umma_idesc_bf16(LBM, LBN);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + LSTAGES * LA;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + LSTAGES * LB);
  uint64_t* empty = full + LSTAGES;
  uint64_t* accf = empty + LSTAGES;  // [2]
  uint64_t* acce = accf + 2;         // [2]
  uint64_t* drain = acce + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // synchronisation points the epilogue has passed (written by its thread 0 after a CTA-scope
  // fence; the producer polls it instead of the global count)
  volatile uint32_t* nbar_s = reinterpret_cast<volatile uint32_t*>(abort_flag + 1);
  volatile int* leave = reinterpret_cast<volatile int*>(nbar_s + 1);   // thread 0's decision, read after a barrier
  volatile int* go_s = leave + 1;                                      // SwiGLU reducer: partials seen
  float* red = reinterpret_cast<float*>(smem + LSTAGES * LSTAGE + 256);   // [4]
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(red + 4);           // [32][64] SwiGLU bf16(up)
  __nv_bfloat16* hs = xs + 32 * 64;   // [64][64] SwiGLU output tile; tensor parallel: a residual row
  static_assert(64 * 64 >= kLayerMaxHidden, "a residual row fits in hs");
  static_assert((2 * LSTAGES + 5) * 8 + 5 * 4 <= 256, "barrier area");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const uint32_t G = gridDim.x;
  unsigned* const count = a.bar;    // grid-barrier arrivals
  unsigned* const epoch = a.bar + 32;  // the count when this launch started

  if (threadIdx.x == 0) {
    for (int s = 0; s < LSTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *nbar_s = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * LBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  int64_t kb0[kMaxPhases];
  int nkb[kMaxPhases];
  int total_it = 0;
#pragma unroll
  for (int p = 0; p < kMaxPhases; ++p) {
    if (p < a.nphase) {
      phase_range(a.ph[p].plan, cta, kb0[p], nkb[p]);
    } else {
      kb0[p] = 0;
      nkb[p] = 0;
    }
    total_it += nkb[p];
  }

  int w_it = 0, x_it = 0;  // producer: weight / activation loads issued
  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      for (int p = 0; p < a.nphase; ++p) {
        prefetch_tmap(&maps.w[p]);
        prefetch_tmap(&maps.x[p]);
      }
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      auto locate = [&](int it, int& p, int& t, int& kb) {
        p = 0;
        while (p < kMaxPhases - 1 && it >= nkb[p]) {
          it -= nkb[p];
          ++p;
        }
        const int64_t g = kb0[p] + it;
        t = static_cast<int>(g / a.ph[p].plan.kblocks);
        kb = static_cast<int>(g - static_cast<int64_t>(t) * a.ph[p].plan.kblocks);
      };
      int ready = -1;          // activation tiles of phases <= ready may be loaded
      auto issue_w = [&]() -> bool {   // the weights of stage w_it, once the MMA has freed the stage
        const int s = w_it % LSTAGES;
        if (!mbar_wait(&empty[s], ((w_it / LSTAGES) & 1) ^ 1, abort_flag, a.err)) return false;
        mbar_arrive_expect_tx(&full[s], LSTAGE);
        int p, t, kb;
        locate(w_it, p, t, kb);
        if (a.ph[p].swiglu) {
          tma_load_2d(sA + s * LA, &maps.w[p], &full[s], kb * LBK, 64 * t, pol_w);
          tma_load_2d(sA + s * LA + LA / 2, &maps.w[p], &full[s], kb * LBK, a.ph[p].inter + 64 * t, pol_w);
        } else {
          tma_load_2d(sA + s * LA, &maps.w[p], &full[s], kb * LBK, LBM * t, pol_w);
        }
        ++w_it;
        return true;
      };
      bool ok = true;
      while (ok && x_it < total_it) {
        int p, t, kb;
        locate(x_it, p, t, kb);
        if (p > ready) {
          // The activations of phase p are not ready yet: stream this phase's first weight tiles
          // into the free stages meanwhile, then wait.  (Each stage frees once the MMA has
          // consumed the previous phase's tile in it, whose activations are already issued.)
          while (ok && w_it < total_it && w_it < x_it + LSTAGES) ok = issue_w();
          if (!ok) break;
          if (ready < 0) pdl_wait();   // phase 0's activations come from the previous kernel
          if (p > 0) {
            if (!wait_passed(nbar_s, syncs_before(a, p), abort_flag, a.err)) break;
            fence_proxy_async_global();   // the consumer's generic stores, read by TMA below
          }
          ready = p;
        }
        if (w_it == x_it && !(ok = issue_w())) break;   // steady state: weights and activations together
        tma_load_2d(sB + (x_it % LSTAGES) * LB, &maps.x[p], &full[x_it % LSTAGES], kb * LBK, 0, pol_x);
        ++x_it;
      }
      if (x_it < w_it) {
        // Unwinding: complete the stages whose weights are in flight with an activation tile
        // (any in-bounds one), so that every copy can be waited for below.
        for (int it = x_it; it < w_it; ++it)
          tma_load_2d(sB + (it % LSTAGES) * LB, &maps.x[0], &full[it % LSTAGES], 0, 0, pol_x);
        x_it = w_it;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int it = 0, seg = 0;
      bool ok = true;
      for (int p = 0; ok && p < a.nphase; ++p) {
        const int kbl = a.ph[p].plan.kblocks;
        int64_t kb = kb0[p];
        const int64_t kb_end = kb0[p] + nkb[p];
        while (ok && kb < kb_end) {
          const int t = static_cast<int>(kb / kbl);
          const int64_t seg_end = min(kb_end, static_cast<int64_t>(t + 1) * kbl);
          const int ab = seg & 1;
          if (!mbar_wait(&acce[ab], ((seg >> 1) & 1) ^ 1, abort_flag, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + static_cast<uint32_t>(ab * LBN);
          for (int64_t g = kb; g < seg_end; ++g, ++it) {
            const int s = it % LSTAGES;
            if (!mbar_wait(&full[s], (it / LSTAGES) & 1, abort_flag, a.err)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t ad = umma_desc_sw128(smem_u32(sA + s * LA));
            const uint64_t bd = umma_desc_sw128(smem_u32(sB + s * LB));
#pragma unroll
            for (int kk = 0; kk < LBK / 16; ++kk)
              umma_bf16(d, ad + 2 * kk, bd + 2 * kk, IDESC, (g > kb || kk > 0) ? 1u : 0u);
            umma_commit(&empty[s]);
          }
          if (!ok) break;
          umma_commit(&accf[ab]);
          kb = seg_end;
          ++seg;
        }
      }
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, a.err);
    }
  } else {
    // ------------------------------------------------------------ epilogue + consumers
    // The 128 threads meet on named barrier 1 (epi_sync), which has no time limit, so they always
    // reach the same barriers: a warp whose wait gives up skips its remaining work (the abort
    // flag is raised) and the CTA's threads leave together at the next meeting point, on a
    // decision thread 0 takes and publishes between two barriers.
    const int e = threadIdx.x - 64;
    const int row = (warp & 3) * 32 + lane;
    pdl_wait();
    uint32_t gen0 = 0, tp_target = 0;
    if (e == 0) {
      gen0 = ld_acquire_gpu(epoch);   // published by the previous launch, which has ended
      if (a.nranks > 0) tp_target = static_cast<uint32_t>(*a.epoch);
    }
    int seg = 0;
    uint32_t nbar = 0;   // grid barriers passed (thread 0)
    uint32_t nsync = 0;  // synchronisation points passed (thread 0)
    bool dead = false;   // warp-uniform
    for (int p = 0; p < a.nphase; ++p) {
      const LayerPhase& ph = a.ph[p];
      const int kbl = ph.plan.kblocks;
      const int64_t total = static_cast<int64_t>(ph.plan.tiles) * kbl;
      int64_t kb = kb0[p];
      const int64_t kb_end = kb0[p] + nkb[p];
      // tiles finished in contributor 0's epilogue: SwiGLU, or (tensor parallel) the push of the
      // rank's sum of a row-parallel tile
      const bool fix = ph.consumer == kConsSwiglu || ph.consumer == kConsTpAddNorm;
      const uint32_t stamp = gen0 + 1 + static_cast<uint32_t>(p);   // this launch's, this phase's flags
      while (kb < kb_end) {
        // A warp whose wait gave up (dead) skips the work of the remaining segments but still
        // takes part in their epi_sync calls, which every thread of the 128 must reach.
        const int t = static_cast<int>(kb / kbl);
        const int64_t seg_end = min(kb_end, static_cast<int64_t>(t + 1) * kbl);
        const int ab = seg & 1;
        if (!dead && !__all_sync(0xffffffffu, mbar_wait(&accf[ab], (seg >> 1) & 1, abort_flag, a.err))) {
          dead = true;
          *abort_flag = 1;
        }
        if (!dead) tc_fence_after();
        const uint32_t tb = tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16) + static_cast<uint32_t>(ab * LBN);
        const int j = cta - sk_cta_of(static_cast<int64_t>(t) * kbl, total, ph.plan.grid);
        if (fix && j == 0) {
          // the other contributors' partials of tile t, then SwiGLU or the push
          const int n = sk_count(ph.plan, t);
          if (e == 0) {
            bool ok = !*abort_flag;
            for (int q = 1; ok && q < n; ++q)
              ok = wait_flag(a.flags + static_cast<int64_t>(t) * ph.plan.maxc + q, stamp, abort_flag, a.err);
            *go_s = ok;
          }
          epi_sync();
          if (ph.consumer == kConsSwiglu) {
            swiglu_tile(a, ph, t, n, tb, row, e, *go_s && !dead, xs, hs);
          } else if (*go_s && !dead) {
            const int pi = p == 0 ? 0 : 1;
            push_tile(a, ph, a.push_plan[pi], a.push[pi], t, n, tb, row);
          }
        } else {
          if (!dead) {
            float* part = ph.partials + (static_cast<int64_t>(t) * ph.plan.maxc + j) * LBN * LBM;
            for (int c0 = 0; c0 < LBN; c0 += 32) {
              uint32_t r[32];
              tmem_ld_x32(tb + c0, r);
              tmem_ld_wait();
#pragma unroll
              for (int jj = 0; jj < 32; ++jj) __stcg(part + (c0 + jj) * LBM + row, __uint_as_float(r[jj]));
            }
          }
          if (fix) {
            // the tile's reducer may read this partial once the flag holds the launch's stamp
            epi_sync();
            if (e == 0 && !*abort_flag)
              st_release_gpu(a.flags + static_cast<int64_t>(t) * ph.plan.maxc + j, stamp);
          }
        }
        if (!dead) {
          tc_fence_before();
          mbar_arrive(&acce[ab]);
        }
        kb = seg_end;
        ++seg;
      }
      // every CTA's partials of this phase, then the consumer
      auto meet = [&](bool fence_async) -> bool {   // grid barrier of the CTA's 128 epilogue threads
        if (fence_async) fence_proxy_async_global();
        epi_sync();
        if (e == 0) {
          ++nbar;
          ++nsync;
          if (!*abort_flag && !grid_barrier(count, gen0 + nbar * G, abort_flag, a.err)) *abort_flag = 1;
          if (cta == 0 && nbar == bars_before(a, a.nphase) && !*abort_flag)
            st_release_gpu(epoch, gen0 + nbar * G);   // every arrival of this launch is in
          if (!*abort_flag) {
            __threadfence_block();   // the acquire above, then the count the producer reads
            *nbar_s = nsync;
          }
          *leave = *abort_flag;
        }
        epi_sync();
        return !*leave;
      };
      // Tensor parallel, right after a grid barrier: CTA 0 signals point k to every rank (one
      // system-scope release fence, cumulative over every CTA's stores that the barrier ordered
      // before it, then a relaxed increment per rank); with `wait`, every CTA then waits for
      // point k's signal from every rank.
      auto xrank = [&](int k, bool wait) -> bool {
        epi_sync();   // every thread has read the last decision before thread 0 writes the next
        if (e == 0) {
          if (cta == 0 && !*abort_flag) {
            fence_acq_rel_sys();
            for (int q = 0; q < a.nranks; ++q) signal_add_relaxed_sys(a.signal[k][q]);
          }
          if (wait && !*abort_flag) {
            if (wait_ranks(a.wait[k], a.nranks, tp_target, abort_flag, a.err)) {
              ++nsync;
              __threadfence_block();
              *nbar_s = nsync;
            }
          }
          *leave = *abort_flag;
        }
        epi_sync();
        return !*leave;
      };
      if (ph.consumer == kConsTpAddNorm) {
        const int k0 = p == 0 ? 0 : 2;
        if (!meet(false)) break;          // every CTA's pushes issued
        if (!xrank(k0, true)) break;      // ... and every rank's arrived
        if (p == 0 && e == 0) pdl_launch_dependents();
        for (int bl = cta; bl < a.rpr; bl += G)
          tp_add_norm_row(a, a.push_plan[p == 0 ? 0 : 1], a.recv[p == 0 ? 0 : 1], a.norm_w[p == 0 ? 0 : 1], bl, e,
                          red, hs);
        if (!meet(true)) break;           // this rank's owned rows written into every rank's xn
        if (!xrank(k0 + 1, p + 1 < a.nphase)) break;   // ... and every owner's (read by TMA next)
        continue;
      }
      if (!fix && !meet(false)) break;
      if (p == 0 && e == 0) pdl_launch_dependents();   // every CTA is resident: the next kernel may queue
      const int warp4 = warp - 2;
      if (ph.consumer == kConsAddNorm) {
        const int T = a.hidden / kSplitBM;
        const int units = a.m * norm_chunks(T);
        for (int u = cta; u < units; u += G) add_norm_pass1(a, ph.plan, ph.partials, u, warp4, lane, red);
        if (!meet(false)) break;
        const __nv_bfloat16* w = a.norm_w[p == 0 ? 0 : 1];
        for (int u = cta; u < units; u += G) add_norm_pass2(a, w, u, warp4, lane);
      } else if (ph.consumer == kConsQk) {
        // one warp per (row, head), two heads' partial sums in flight together (head dim 128: a
        // head is one 128-feature tile, the lane's 4 features at tile row 4 * lane)
        const int heads = a.nq + 2 * a.nkv;
        const int tasks = a.m * heads;
        const int W = static_cast<int>(G) * 4;
        for (int task = cta * 4 + warp4; task < tasks; task += 2 * W) {
          int tt[2], bb[2], rr[2];
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int k = task + i * W < tasks ? task + i * W : task;
            bb[i] = k / heads;
            tt[i] = k - bb[i] * heads;
            rr[i] = 4 * lane;
          }
          float4 sv[2];
          sk_sum4_n<2>(ph.partials, ph.plan, tt, bb, rr, task + W < tasks ? 2 : 1, sv);
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            if (i == 1 && task + W >= tasks) break;
            float x[4] = {bf16_round(sv[i].x), bf16_round(sv[i].y), bf16_round(sv[i].z), bf16_round(sv[i].w)};
            qk_norm_rope_kv_x<128>(bb[i], tt[i], lane, x, a.q_out, a.kv, a.qnw, a.knw, a.cos_t, a.sin_t, a.table_len,
                                   a.positions, a.block_tables, a.max_blocks, a.nq, a.nkv, a.next_layer,
                                   a.num_blocks, a.bs, a.eps, 0, a.err);
          }
        }
      }
      // the consumer's output is the next phase's activations (read by TMA)
      if (p + 1 < a.nphase && !meet(true)) break;
    }
  }

  __syncthreads();
  if (warp == 0 && lane == 0) {
    // Wait (bounded) for the copies still in flight.
    const int first = x_it > LSTAGES ? x_it - LSTAGES : 0;
    for (int it = first; it < x_it; ++it) mbar_wait(&full[it % LSTAGES], (it / LSTAGES) & 1, nullptr, a.err);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * LBN);
  }
}


size_t layer_smem() { return static_cast<size_t>(LSTAGES) * LSTAGE + 256 + 16 + (32 + 64) * 64 * 2 + 1024; }

int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, uint32_t box_rows) {
  const uint64_t dims[2] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(rows)};
  const uint64_t strides[1] = {static_cast<uint64_t>(ld) * 2};
  const uint32_t box[2] = {LBK, box_rows};
  return encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// The CTAs of one launch: two per SM, all resident (the grid barriers need every CTA running).
// The kernel's 168 registers and ~100 KB of shared memory fit twice on an SM (the same budget as
// the standalone decode GEMM, whose CTAs run two per SM); if a CTA could not become resident, the
// grid barriers would run out of time and report MVB_DEV_WAIT_TIMEOUT instead of hanging.
int layer_grid(int sms) {
  static bool done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return -1;
  if (!done[dev]) {
    if (set_smem(layer_kernel, layer_smem(), "decoder_layer_tail: smem attribute") != MVB_OK) return -1;
    done[dev] = true;
  }
  return 2 * sms;
}

}  // namespace
}  // namespace mvb

using namespace mvb;

extern "C" int64_t mvb_decoder_layer_workspace_bytes(int64_t m, int64_t hidden, int64_t q_dim, int64_t inter,
                                                     int64_t qkv_dim, int device) {
  int sms = mvb_num_sms(device);
  if (sms <= 0) sms = 148;
  const int64_t G = 2LL * sms;
  int64_t best = 0;
  const SplitKPlan plans[4] = {
      splitk_plan_ctas(m, static_cast<int>((hidden + LBM - 1) / LBM), q_dim, G),
      splitk_plan_ctas(m, static_cast<int>((inter + 63) / 64), hidden, G),
      splitk_plan_ctas(m, static_cast<int>((hidden + LBM - 1) / LBM), inter, G),
      splitk_plan_ctas(m, static_cast<int>((qkv_dim + LBM - 1) / LBM), hidden, G)};
  int64_t nflags = 0;
  for (const SplitKPlan& p : plans) {
    best = std::max(best, splitk_partials_bytes(p));
    nflags = std::max(nflags, static_cast<int64_t>(p.tiles) * p.maxc);
  }
  return (best + 255) / 256 * 256 + (m * kNormChunks * 4 + 255) / 256 * 256 + (nflags * 4 + 255) / 256 * 256;
}

namespace {

// Tensor-parallel arguments of a launch (null: one GPU).
struct TpLayerCall {
  mvb_tp_comm* comm;
  int64_t recv_o, recv_down, xn;   // heap offsets
  int layer;                       // signal points 4 * layer .. 4 * layer + 3
};

int layer_tail_impl(const TpLayerCall* tp, const void* attn, int64_t attn_stride, const void* wo, const void* ln2,
                    const void* wgu, const void* wdown, const void* ln_next, const void* wqkv_next,
                    const void* q_norm_next, const void* k_norm_next, void* residual, void* xn, void* h,
                    void* q_out, void* kv_cache, const void* cos, const void* sin, int64_t table_len,
                    const int32_t* positions, const int32_t* block_tables, int64_t max_blocks, int64_t m,
                    int64_t hidden, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim, int64_t inter,
                    int64_t num_layers, int64_t next_layer, int64_t num_blocks, int64_t block_size, float eps,
                    void* workspace, int64_t workspace_bytes, void* barrier, mvb_stream_t stream) {
  MVB_REQUIRE(attn && wo && ln2 && wgu && wdown && ln_next && residual && xn && h && workspace && barrier,
              "mvb_decoder_layer_tail: null pointer");
  MVB_REQUIRE(m > 0 && m <= LBN, "mvb_decoder_layer_tail: batch %lld must be in [1, %d]", (long long)m, LBN);
  MVB_REQUIRE(head_dim == 128 && num_q_heads > 0 && num_kv_heads > 0 && num_q_heads % num_kv_heads == 0,
              "mvb_decoder_layer_tail: head_dim 128 and whole GQA groups");
  const int64_t q_dim = num_q_heads * head_dim, qkv_dim = (num_q_heads + 2 * num_kv_heads) * head_dim;
  MVB_REQUIRE(hidden % LBK == 0 && hidden % 4 == 0 && hidden <= kLayerMaxHidden && inter % 64 == 0 && inter > 0 &&
                  q_dim % LBK == 0,
              "mvb_decoder_layer_tail: hidden %lld (multiple of 64, <= %d), intermediate %lld (multiple of 64)",
              (long long)hidden, kLayerMaxHidden, (long long)inter);
  MVB_REQUIRE(attn_stride >= q_dim && attn_stride % 8 == 0, "mvb_decoder_layer_tail: attn_stride");
  MVB_REQUIRE(aligned(attn, 16) && aligned(xn, 16) && aligned(h, 16) && aligned(wo, 16) && aligned(wgu, 16) &&
                  aligned(wdown, 16) && aligned(residual, 8) && aligned(workspace, 256) && aligned(barrier, 128),
              "mvb_decoder_layer_tail: alignment");
  const bool next = wqkv_next != nullptr;
  if (next) {
    MVB_REQUIRE(q_out && kv_cache && cos && sin && positions && block_tables,
                "mvb_decoder_layer_tail: the next layer's QK-norm/RoPE/KV-write inputs");
    MVB_REQUIRE((q_norm_next == nullptr) == (k_norm_next == nullptr),
                "mvb_decoder_layer_tail: pass both norm weights or neither");
    MVB_REQUIRE(next_layer >= 0 && next_layer < num_layers && num_blocks > 0 && block_size > 0 && max_blocks > 0,
                "mvb_decoder_layer_tail: bad cache geometry");
    MVB_REQUIRE(aligned(wqkv_next, 16), "mvb_decoder_layer_tail: alignment");
  }
  const int sms = current_sm_count();
  MVB_REQUIRE(sms > 0, "mvb_decoder_layer_tail: no device");
  const int G = layer_grid(sms);
  MVB_REQUIRE(G > 0, "mvb_decoder_layer_tail: the kernel does not fit on an SM");

  LayerArgs a{};
  LayerMaps maps{};
  a.m = static_cast<int>(m);
  a.nphase = next ? 4 : 3;
  a.ph[0].plan = splitk_plan_ctas(m, static_cast<int>((hidden + LBM - 1) / LBM), q_dim, G);
  a.ph[0].consumer = kConsAddNorm;
  a.ph[1].plan = splitk_plan_ctas(m, static_cast<int>(inter / 64), hidden, G);
  a.ph[1].swiglu = 1;
  a.ph[1].inter = static_cast<int>(inter);
  a.ph[1].consumer = kConsSwiglu;
  a.ph[2].plan = splitk_plan_ctas(m, static_cast<int>((hidden + LBM - 1) / LBM), inter, G);
  a.ph[2].consumer = kConsAddNorm;
  if (next) {
    a.ph[3].plan = splitk_plan_ctas(m, static_cast<int>(qkv_dim / LBM), hidden, G);
    a.ph[3].consumer = kConsQk;
  }
  int points[4] = {0, 0, 0, 0};
  if (tp) {
    // row-parallel o_proj / down_proj: the whole grid's stream-K split (as one GPU), each tile
    // summed over this rank's contributors by its contributor 0, which pushes one fp32 tile per
    // rank (a one-k-block plan's layout, which fits the receive areas mvb_tp_recv_bytes sizes for
    // the per-kernel path's push split)
    mvb_tp_comm* c = tp->comm;
    const int nr = c->nranks;
    MVB_REQUIRE(m % nr == 0, "mvb_tp_decoder_layer_tail: batch %lld not a multiple of %d ranks", (long long)m, nr);
    a.nranks = nr;
    a.rank = c->rank;
    a.rpr = static_cast<int>(m / nr);
    a.ph[0].consumer = kConsTpAddNorm;
    a.ph[2].consumer = kConsTpAddNorm;
    const int64_t off[2] = {tp->recv_o, tp->recv_down};
    for (int k = 0; k < 2; ++k) {
      a.push_plan[k] = splitk_plan_push(m, hidden, kSplitBK, sms, nr);
      MVB_REQUIRE(a.push_plan[k].maxc == 1, "mvb_tp_decoder_layer_tail: push layout");
      const int64_t bytes = splitk_push_bytes(a.push_plan[k], nr, a.rpr);
      MVB_REQUIRE(off[k] >= kTpSignalBytes && off[k] % 16 == 0 && off[k] + bytes <= c->heap_bytes,
                  "mvb_tp_decoder_layer_tail: receive area outside the heap");
      a.recv[k] = reinterpret_cast<const float*>(c->base[c->rank] + off[k]);
      for (int q = 0; q < nr; ++q) a.push[k][q] = reinterpret_cast<float*>(c->base[q] + off[k]);
    }
    MVB_REQUIRE(tp->xn >= kTpSignalBytes && tp->xn % 16 == 0 && tp->xn + m * hidden * 2 <= c->heap_bytes,
                "mvb_tp_decoder_layer_tail: xn outside the heap");
    for (int q = 0; q < nr; ++q) a.xn_all[q] = reinterpret_cast<__nv_bfloat16*>(c->base[q] + tp->xn);
    MVB_REQUIRE(tp->layer >= 0 && 4 * tp->layer + 3 < kTpMaxPoints, "mvb_tp_decoder_layer_tail: layer %d",
                tp->layer);
    for (int k = 0; k < 4; ++k) {
      points[k] = 4 * tp->layer + k;
      for (int q = 0; q < nr; ++q) a.signal[k][q] = c->signal_slot(q, points[k]);
      a.wait[k] = c->wait_row(points[k]);
    }
    a.epoch = c->epoch;
  }
  int64_t need = 0, nflags = 0;
  for (int p = 0; p < a.nphase; ++p) {
    a.ph[p].partials = static_cast<float*>(workspace);
    need = std::max(need, splitk_partials_bytes(a.ph[p].plan));
    nflags = std::max(nflags, static_cast<int64_t>(a.ph[p].plan.tiles) * a.ph[p].plan.maxc);
  }
  const int64_t ss_off = (need + 255) / 256 * 256;
  const int64_t flags_off = ss_off + (m * kNormChunks * 4 + 255) / 256 * 256;
  need = flags_off + nflags * 4;
  MVB_REQUIRE(workspace_bytes >= need, "mvb_decoder_layer_tail: workspace %lld < %lld bytes",
              (long long)workspace_bytes, (long long)need);
  a.ss = reinterpret_cast<float*>(static_cast<char*>(workspace) + ss_off);
  a.flags = reinterpret_cast<unsigned*>(static_cast<char*>(workspace) + flags_off);
  MVB_TRY(make_map(&maps.w[0], wo, hidden, q_dim, q_dim, LBM));
  MVB_TRY(make_map(&maps.x[0], attn, m, q_dim, attn_stride, LBN));
  MVB_TRY(make_map(&maps.w[1], wgu, 2 * inter, hidden, hidden, 64));
  MVB_TRY(make_map(&maps.x[1], xn, m, hidden, hidden, LBN));
  MVB_TRY(make_map(&maps.w[2], wdown, hidden, inter, inter, LBM));
  MVB_TRY(make_map(&maps.x[2], h, m, inter, inter, LBN));
  if (next) {
    MVB_TRY(make_map(&maps.w[3], wqkv_next, qkv_dim, hidden, hidden, LBM));
    MVB_TRY(make_map(&maps.x[3], xn, m, hidden, hidden, LBN));
  }
  a.residual = static_cast<__nv_bfloat16*>(residual);
  a.xn = static_cast<__nv_bfloat16*>(xn);
  a.h = static_cast<__nv_bfloat16*>(h);
  a.hidden = static_cast<int>(hidden);
  a.inter = static_cast<int>(inter);
  a.norm_w[0] = static_cast<const __nv_bfloat16*>(ln2);
  a.norm_w[1] = static_cast<const __nv_bfloat16*>(ln_next);
  a.eps = eps;
  a.q_out = static_cast<__nv_bfloat16*>(q_out);
  a.kv = static_cast<__nv_bfloat16*>(kv_cache);
  a.qnw = static_cast<const __nv_bfloat16*>(q_norm_next);
  a.knw = static_cast<const __nv_bfloat16*>(k_norm_next);
  a.cos_t = static_cast<const __nv_bfloat16*>(cos);
  a.sin_t = static_cast<const __nv_bfloat16*>(sin);
  a.table_len = table_len;
  a.positions = positions;
  a.block_tables = block_tables;
  a.max_blocks = max_blocks;
  a.nq = static_cast<int>(num_q_heads);
  a.nkv = static_cast<int>(num_kv_heads);
  a.next_layer = next_layer;
  a.num_blocks = num_blocks;
  a.bs = static_cast<int>(block_size);
  a.bar = static_cast<unsigned*>(barrier);
  a.err = device_status_ptr();
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MVB_TRY(launch(tp ? "tp_decoder_layer_tail" : "decoder_layer_tail", layer_kernel, dim3(static_cast<unsigned>(G)),
                 dim3(kLayerThreads), layer_smem(), st, maps, a));
  if (tp)
    for (int k = 0; k < 4; ++k) tp->comm->point_count[points[k]] = 1;   // one signal per rank per step
  return MVB_OK;
}

}  // namespace

extern "C" int mvb_decoder_layer_tail(const void* attn, int64_t attn_stride, const void* wo, const void* ln2,
                                      const void* wgu, const void* wdown, const void* ln_next, const void* wqkv_next,
                                      const void* q_norm_next, const void* k_norm_next, void* residual, void* xn,
                                      void* h, void* q_out, void* kv_cache, const void* cos, const void* sin,
                                      int64_t table_len, const int32_t* positions, const int32_t* block_tables,
                                      int64_t max_blocks, int64_t m, int64_t hidden, int64_t num_q_heads,
                                      int64_t num_kv_heads, int64_t head_dim, int64_t inter, int64_t num_layers,
                                      int64_t next_layer, int64_t num_blocks, int64_t block_size, float eps,
                                      void* workspace, int64_t workspace_bytes, void* barrier, mvb_stream_t stream) {
  return layer_tail_impl(nullptr, attn, attn_stride, wo, ln2, wgu, wdown, ln_next, wqkv_next, q_norm_next,
                         k_norm_next, residual, xn, h, q_out, kv_cache, cos, sin, table_len, positions, block_tables,
                         max_blocks, m, hidden, num_q_heads, num_kv_heads, head_dim, inter, num_layers, next_layer,
                         num_blocks, block_size, eps, workspace, workspace_bytes, barrier, stream);
}

extern "C" int mvb_tp_decoder_layer_tail(mvb_tp_comm* comm, int layer, const void* attn, int64_t attn_stride,
                                         const void* wo, const void* ln2, const void* wgu, const void* wdown,
                                         const void* ln_next, const void* wqkv_next, const void* q_norm_next,
                                         const void* k_norm_next, void* residual, int64_t xn_offset, void* h,
                                         void* q_out, void* kv_cache, const void* cos, const void* sin,
                                         int64_t table_len, const int32_t* positions, const int32_t* block_tables,
                                         int64_t max_blocks, int64_t m, int64_t hidden, int64_t num_q_heads,
                                         int64_t num_kv_heads, int64_t head_dim, int64_t inter, int64_t num_layers,
                                         int64_t next_layer, int64_t num_blocks, int64_t block_size, float eps,
                                         int64_t recv_o_offset, int64_t recv_down_offset, void* workspace,
                                         int64_t workspace_bytes, void* barrier, mvb_stream_t stream) {
  MVB_REQUIRE(comm, "mvb_tp_decoder_layer_tail: null communicator");
  MVB_REQUIRE(xn_offset >= 0 && xn_offset < comm->heap_bytes, "mvb_tp_decoder_layer_tail: xn offset");
  const TpLayerCall tp{comm, recv_o_offset, recv_down_offset, xn_offset, layer};
  return layer_tail_impl(&tp, attn, attn_stride, wo, ln2, wgu, wdown, ln_next, wqkv_next, q_norm_next, k_norm_next,
                         residual, comm->base[comm->rank] + xn_offset, h, q_out, kv_cache, cos, sin, table_len,
                         positions, block_tables, max_blocks, m, hidden, num_q_heads, num_kv_heads, head_dim, inter,
                         num_layers, next_layer, num_blocks, block_size, eps, workspace, workspace_bytes, barrier,
                         stream);
}
