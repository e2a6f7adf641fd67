// Paged-attention decode: one query token per sequence, K/V read straight out of the
// reference's paged pool through the block table.
//
// Replaces, for decode, Attention._read_kv_cache_batch + GQA expand + SDPA with a
// padding mask (models/model.py:191-221; models/model_cuda.py:145-177;
// models/gemma3_model.py:169-195 for head_dim 256):
//   out[b, h] = softmax(q[b, h] . K[b, lo_b:ctx_b]^T * scale) V[b, lo_b:ctx_b]
// with lo_b = 0, or ctx_b - window under a sliding window of the newest `window` keys, and
// optionally soft-capped scores s -> cap * tanh(s / cap) (Gemma-2's attention softcap).
// Pool layout (engine/kv_cache.py:24-29): [L, 2, num_blocks, block_size=16, Hkv, D], D 128 or 256.
//
// Work split: the KV heads are cut into head groups of HKV heads (all of them at D = 128; two
// at D = 256, whose blocks are twice as large).  The (sequence x head group, block) pairs of the
// whole batch are laid end to end and divided evenly over the persistent CTAs (split-KV across
// the GPU).  A sequence that spans several CTAs is merged by the last CTA to finish it,
// combining the partial (max, sum, output) triples in CTA order, so results are deterministic.
//
// CTA = 8 consumer warps (4 at D = 256 and for D = 128 groups of <= 2 heads) + 1 producer warp.  The producer streams each block's
// K and V (the head group's heads) through TMA into a 128-byte-swizzled image of 128-byte lines
// (head_dim split into parts of 64).  It issues one copy per (K|V, part), image
// [kv][part][head][token][64]; only for D = 128 blocks of one or two heads (tensor-parallel
// shards, 4-8 KB) is the per-copy cost worth saving, with one 5-D copy per block, image
// [kv][token][head, part][64].  Consumer warp (h, w) serves KV head h -- its GROUP query heads
// are the columns of an m16n8 tile -- and with W = (consumer warps) / HKV warps per head takes every
// W-th block of the CTA's range, so a GPU holding few KV heads (tensor parallelism) still runs
// every consumer warp; the W partial softmax states of a head are combined in shared memory at
// each sequence boundary.
// Both products run transposed on mma.sync m16n8k16 (bf16 in, fp32 accumulate) so that the
// query heads fill the n = 8 side instead of wasting 16-row tiles: S^T = K Q^T (tokens x heads),
// then O^T = V^T P^T (dims x heads), P^T reaching the B operand through one 8x8 transpose
// (movmatrix) per 8 tokens.  The softmax is the online (running max / running sum) form in the
// exp2 domain, kept per head column.
#include <mutex>

#include "common.cuh"
#include "host.h"
#include "mma_sync.cuh"

namespace mvb {
namespace {

constexpr int BS = 16;       // tokens per block (the reference's block_size)
constexpr int HALF_BYTES_PER_HEAD = BS * 64 * 2;  // 2 KB: 16 tokens x 64 dims (one part of a head)
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kEarlyBlocks = 4;  // see the early arrival-count read in the consumer loop

struct AttnArgs {
  __nv_bfloat16* out;
  int64_t out_stride;
  const __nv_bfloat16* q;
  int64_t q_stride;
  const int32_t* block_tables;
  int64_t max_blocks;
  const int32_t* ctx_lens;
  int batch;
  int nhg;           // head groups per sequence (KV heads / HKV)
  int window;        // > 0: attend to the newest `window` keys only
  int64_t layer;
  int64_t num_blocks;
  float scale_log2;  // scale * log2(e)
  float cap_scale;   // softcap > 0: scale / softcap
  float cap_log2;    // softcap * log2(e); 0 = no soft-capping
  float* partial_o;  // [2*G][GROUP*HKV][D]
  float2* partial_ml;  // [2*G][GROUP*HKV]  (running max in log2 units, running sum)
  int* counters;     // [batch * nhg]
  unsigned* err;
};

// First block of a sequence of ctx keys that the window reaches.
__device__ __forceinline__ int window_first_block(int ctx, int window) {
  return (window > 0 && ctx > window) ? (ctx - window) / 16 : 0;
}

__device__ __forceinline__ int64_t range_start(int c, int64_t total, int grid) {
  return static_cast<int64_t>(c) * total / grid;
}
__device__ __forceinline__ int cta_of(int64_t x, int64_t total, int grid) {
  return static_cast<int>(((x + 1) * grid + total - 1) / total - 1);
}

template <int NCW>
__device__ __forceinline__ void consumer_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory");
}

// Barrier of the W consumer warps of KV head h (named barriers 2 .. 2 + Hkv - 1).
template <int W>
__device__ __forceinline__ void head_bar(int h) {
  asm volatile("bar.sync %0, %1;" ::"r"(2 + h), "n"(W * 32) : "memory");
}

// Consumer warps per CTA: 8 at D = 128.  At D = 256 the bandwidth is set by the bytes the
// stages keep in flight, and 4 warps (2 per KV head of a two-head group) let the stage count be
// a multiple of 2 instead of 4: 6 stages of 32 KB instead of 4.
template <int D>
__host__ __device__ constexpr int attn_consumer_warps() {
  return D == 128 ? 8 : 4;
}

// Consumer warps per KV head: all consumer warps of the CTA shared by its HKV heads, as long as
// the merge's per-thread share (GROUP * D / (W * 32) outputs) stays whole.  Blocks of one or two
// D = 128 heads (4-8 KB) take 4 consumer warps instead of 8: each warp then owns twice as many
// stages ahead of it (25.7 instead of 27.4 us at one KV head, batch 64, context 2049).
template <int GROUP, int HKV, int D>
__host__ __device__ constexpr int attn_wph() {
  constexpr int cw = (D == 128 && HKV <= 2) ? 4 : attn_consumer_warps<D>();
  return (cw / HKV) < GROUP * (D / 32) ? (cw / HKV) : GROUP * (D / 32);
}

// CTAs per SM: two for D = 128 groups of one or two KV heads (tensor-parallel shards) when the
// launch has at most kDualMaxPairs (sequence, head group) pairs, each CTA with about half the
// stage memory; two producers and two consumer sets per SM overlap one CTA's ramp, merges and
// tail with the other's streaming, and the finer split of the block ranges evens out when the
// CTAs finish.  One for the rest.
constexpr int kDualMaxPairs = 512;
__host__ __device__ constexpr bool attn_dual_for(int hkv, int d) { return d == 128 && hkv <= 2; }

// One TMA copy per block (D = 128 blocks of <= 2 heads) or one per (K|V, part).  Several small
// copies keep more requests in flight than one large multi-dimensional box: at D = 256 the split
// form streams at 6.7 TB/s where one 32 KB box per stage reached 3.9 TB/s.
__host__ __device__ constexpr bool attn_one_copy_for(int hkv, int d) { return d == 128 && hkv <= 2; }
template <int HKV, int D>
__host__ __device__ constexpr bool attn_one_copy() {
  return attn_one_copy_for(HKV, D);
}

// 128-byte line of (kv, part, head, token) in a stage image of either layout.
template <int HKV, int D>
__device__ __forceinline__ int attn_line(int kv, int part, int h, int tok) {
  constexpr int NP = D / 64;
  if constexpr (attn_one_copy<HKV, D>()) return (kv * BS + tok) * (NP * HKV) + h * NP + part;
  return ((kv * NP + part) * HKV + h) * BS + tok;
}

// Shared memory of the per-head combine: every consumer warp's (m, l, o) for its GROUP rows.
template <int GROUP, int HKV, int D>
__host__ __device__ constexpr int attn_combine_bytes() {
  return attn_wph<GROUP, HKV, D>() > 1 ? HKV * attn_wph<GROUP, HKV, D>() * GROUP * (D + 2) * 4 : 0;
}

// CAP: soft-capped scores (a compile-time switch: the tanh would otherwise be evaluated for
// every score of every launch).
template <int GROUP, int HKV, int STAGES, int D, bool CAP, int CPS>
__global__ void __launch_bounds__((HKV * attn_wph<GROUP, HKV, D>() + 1) * 32, CPS)
    paged_attention_kernel(const __grid_constant__ CUtensorMap tm, const AttnArgs a) {
  constexpr int NP = D / 64;                                      // 64-dim parts of a head
  constexpr int STAGE_BYTES = 2 * NP * HKV * HALF_BYTES_PER_HEAD;  // K and V parts of HKV heads
  constexpr int W = attn_wph<GROUP, HKV, D>();                    // consumer warps per KV head
  constexpr int HQ = GROUP * HKV;                                 // query heads of a head group
  constexpr int NCW = HKV * W;                                // consumer warps
  static_assert(STAGES % W == 0, "a stage must always serve the same warp of each head");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + STAGES);
  volatile int* last_flag = abort_flag + 1;
  const int nv = a.batch * a.nhg;  // virtual sequences: (sequence, head group), head groups adjacent
  int* cu = const_cast<int*>(abort_flag + 2);  // [nv + 1] block prefix sums
  // per-head combine (W > 1), 16-byte aligned
  float* combine_smem = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(cu + nv + 1) + 15) & ~uintptr_t(15));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], HKV);
    }
    *abort_flag = 0;
    *last_flag = 0;
    fence_barrier_init();
  }
  // Programmatic dependent launch: only q and the newest token's K/V (always in the last block of
  // its sequence) come from the previous kernel.  Lengths and block tables are step metadata, so
  // the prologue and the TMA copies of every other block run before the grid-dependency wait; the
  // producer waits before issuing a sequence's last block, the consumers before reading q.
  if (threadIdx.x == 0) pdl_launch_dependents();
  // Per-(sequence, head group) block counts -> prefix sums (warp 0, 32 at a time).
  if (warp == 0) {
    int carry = 0;
    for (int base = 0; base < nv; base += 32) {
      const int v = base + lane;
      int n = 0;
      if (v < nv) {
        const int ctx = a.ctx_lens[v / a.nhg];
        n = ctx > 0 ? (ctx + BS - 1) / BS : 0;
        if (n > a.max_blocks) {
          report(a.err, kDevBadPosition);
          n = static_cast<int>(a.max_blocks);
        }
        n -= window_first_block(ctx, a.window);
        if (n < 0) n = 0;
      }
      int incl = n;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int x = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += x;
      }
      if (v < nv) cu[v + 1] = carry + incl;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) cu[0] = 0;
  }
  __syncthreads();
  const int64_t total = cu[nv];
  // Effective grid: never more CTAs than blocks, so every CTA in [0, G) owns at least
  // one block and the contributor count of a sequence is exact.
  const int G = static_cast<int>(total < gridDim.x ? total : gridDim.x);
  if (static_cast<int>(blockIdx.x) >= G) return;
  const int64_t g_begin = range_start(blockIdx.x, total, G);
  const int64_t g_end = range_start(blockIdx.x + 1, total, G);
  int b0 = 0;
  {  // first virtual sequence with cu[v+1] > g_begin
    int lo = 0, hi = nv - 1;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (cu[mid + 1] > g_begin) hi = mid; else lo = mid + 1;
    }
    b0 = lo;
  }

  int issued = 0;
  if (warp == NCW) {
    // ---------------------------------------------------------------- producer
    // The whole warp fetches the next 32 block ids at once (one per lane, one round trip of
    // latency per 32 blocks); lane 0 then issues the TMA copies from the shuffled ids.
    if (g_end > g_begin) {
      if (lane == 0) prefetch_tmap(&tm);
      const uint64_t pol = l2_policy_evict_first();
      const int64_t P = a.num_blocks;
      int b_lane = b0;
      bool ok = true;
      bool waited = false;  // lane 0: grid-dependency wait done
      for (int64_t g0 = g_begin; ok && g0 < g_end; g0 += 32) {
        const int64_t g = g0 + lane;
        int blk = 0, last = 0;
        if (g < g_end) {
          while (g >= cu[b_lane + 1]) ++b_lane;
          const int bs = b_lane / a.nhg;
          const int j = static_cast<int>(g - cu[b_lane]) + window_first_block(a.ctx_lens[bs], a.window);
          last = g == cu[b_lane + 1] - 1;
          blk = a.block_tables[static_cast<int64_t>(bs) * a.max_blocks + j];
          if (blk < 0 || blk >= P) {
            report(a.err, kDevBadBlock);
            blk = 0;  // stay in bounds; the sequence's output is not trusted (status word set)
          }
        }
        const int n = static_cast<int>(g_end - g0 < 32 ? g_end - g0 : 32);
        for (int i = 0; i < n; ++i) {
          const int bi = __shfl_sync(0xffffffffu, blk, i);
          const int li = __shfl_sync(0xffffffffu, last, i);
          // head group of the block (at D = 128 a stage holds all KV heads: one group)
          const int hg = D == 128 ? 0 : __shfl_sync(0xffffffffu, b_lane, i) % a.nhg;
          int good = 1;
          if (lane == 0) {
            if (li && !waited) {  // this block holds the token the previous kernel wrote
              pdl_wait();
              waited = true;
            }
            const int it = static_cast<int>(g0 - g_begin) + i;
            const int s = it % STAGES;
            const uint32_t ph = (it / STAGES) & 1;
            if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, a.err)) {
              good = 0;
            } else {
              mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
              uint8_t* st = smem + s * STAGE_BYTES;
              if constexpr (attn_one_copy<HKV, D>()) {
                tma_load_5d(st, &tm, &full[s], 0, hg * HKV * NP, 0, bi, static_cast<int>(a.layer * 2), pol);
              } else {
                for (int kv = 0; kv < 2; ++kv) {
                  const int row = static_cast<int>((a.layer * 2 + kv) * P + bi);
                  for (int part = 0; part < NP; ++part)
                    tma_load_4d(st + (kv * NP + part) * HKV * HALF_BYTES_PER_HEAD, &tm, &full[s], part * 64, 0,
                                hg * HKV, row, pol);
                }
              }
              issued = it + 1;
            }
          }
          if (!__shfl_sync(0xffffffffu, good, 0)) {
            ok = false;
            break;
          }
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- consumers
    pdl_wait();  // q, and the partial / counter workspace the previous launch may still use
    const int h = warp / W, w = warp - (warp / W) * W;  // KV head, and this warp's turn among its W
    const int g = lane >> 2, t = lane & 3;
    const bool row_valid = g < GROUP;
    const uint32_t sbase = smem_u32(smem);
    int vs = b0;  // virtual sequence: (sequence b, head group hg)
    int64_t gpos = g_begin;
    while (gpos < g_end) {
      while (gpos >= cu[vs + 1]) ++vs;
      const int b = vs / a.nhg, hg = vs - (vs / a.nhg) * a.nhg;
      const int64_t seq_lo = cu[vs], seq_hi = cu[vs + 1];
      const int64_t seg_end = min(g_end, seq_hi);
      const bool whole = (gpos == seq_lo) && (seg_end == seq_hi);
      // Thread 0 of a split segment reads the sequence's arrival count a few blocks before the
      // segment ends (kEarlyBlocks per consumer warp of a head): if every other contributor has
      // already arrived, this CTA is the last one and merges without the fence and the atomic.
      // The CTA whose range begins a sequence is its usual last arriver, long after the CTAs that
      // took the sequence's later blocks at the start of their ranges.
      bool early_read = false;
      uint32_t early_count = 0;
      const int ctx = a.ctx_lens[b];
      const int blk0 = window_first_block(ctx, a.window);
      const int lo_tok = a.window > 0 ? ctx - a.window : 0;
      const int hq0 = (hg * HKV + h) * GROUP;  // first query head of KV head h (global index)
      // Q fragments (rows = the GROUP query heads of this KV head; rows >= GROUP are zero).
      uint32_t qa[D / 16][2];
      {
        const __nv_bfloat16* qp = a.q + static_cast<int64_t>(b) * a.q_stride + static_cast<int64_t>(hq0 + g) * D;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          if (row_valid) {
            qa[kk][0] = *reinterpret_cast<const uint32_t*>(qp + kk * 16 + 2 * t);
            qa[kk][1] = *reinterpret_cast<const uint32_t*>(qp + kk * 16 + 8 + 2 * t);
          } else {
            qa[kk][0] = qa[kk][1] = 0u;
          }
        }
      }
      // O^T accumulators, one m16n8 tile per 16 dims: o[mt] = {O^T[dim 16mt+g][head 2t],
      // [16mt+g][2t+1], [16mt+g+8][2t], [16mt+g+8][2t+1]} (heads = this KV head's GROUP query heads).
      float o[D / 16][4];
#pragma unroll
      for (int n = 0; n < D / 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
      // Softmax state of this thread's two query heads 2t and 2t+1 (the S^T / O^T columns): running
      // max (log2 units, equal across the g lanes) and this thread's share of the denominator.
      float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.0f, l_b = 0.0f;

      // This warp's blocks of the segment: iterations it = gg - g_begin with it % W == w.
      const int64_t off = (gpos - g_begin) % W;
      for (int64_t gg = gpos + (w - off + W) % W; gg < seg_end; gg += W) {
        const int it = static_cast<int>(gg - g_begin);
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        // A wait that gives up has reported the timeout and raised the abort flag; the warp
        // carries on (on stale data) so that every warp still meets every barrier below.
        mbar_wait(&full[s], ph, abort_flag, a.err);
        if (threadIdx.x == 0 && !whole && !early_read && seg_end - gg <= kEarlyBlocks * W) {
          early_count = ld_relaxed_gpu(reinterpret_cast<const unsigned*>(a.counters + vs));
          early_read = true;
        }
        const int j = blk0 + static_cast<int>(gg - seq_lo);  // block index within the sequence
        // 128-byte lines of the stage image (attn_line); 16-byte chunks are XOR-swizzled with the
        // line index mod 8 (the stage is 1024-byte aligned).
        const uint32_t stage_base = sbase + s * STAGE_BYTES;
        // S^T = K Q^T for 16 tokens (m = 16 tokens, n = 8 query heads, k = 16 dims per step), in four
        // independent accumulator chains.  A = K from a plain ldmatrix.x4: matrices (tokens 0-7 |
        // 8-15) x (dims 0-7 | 8-15) in the fragment order a0 a1 a2 a3; B = Q^T is the q fragment.
        float sacc[4][4];
#pragma unroll
        for (int c = 0; c < 4; ++c) sacc[c][0] = sacc[c][1] = sacc[c][2] = sacc[c][3] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int part = kk >> 2;
          const int mi = lane >> 3;
          const int tok = (mi & 1) * 8 + (lane & 7);
          const int chunk = (kk & 3) * 2 + (mi >> 1);
          const int line = attn_line<HKV, D>(0, part, h, tok);
          const uint32_t addr = stage_base + line * 128 + ((chunk ^ (line & 7)) << 4);
          uint32_t k0, k1, k2, k3;
          ldsm_x4(addr, k0, k1, k2, k3);
          mma_bf16_16816(sacc[kk & 3], k0, k1, k2, k3, qa[kk][0], qa[kk][1]);
        }
        // x = S^T[token g][head 2t], [g][2t+1], [g+8][2t], [g+8][2t+1]: scaled (and soft-capped)
        // into the log2 domain; tokens past the context or before the window masked.
        const int tok0 = j * BS;
        const int tka = tok0 + g, tkb = tok0 + g + 8;
        const bool ka = tka < ctx && tka >= lo_tok, kb = tkb < ctx && tkb >= lo_tok;
        float x[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float raw = sacc[0][c] + sacc[1][c] + sacc[2][c] + sacc[3][c];
          float sc;
          if constexpr (CAP) {
            sc = a.cap_log2 * tanhf(raw * a.cap_scale);
          } else {
            sc = raw * a.scale_log2;
          }
          x[c] = (c < 2 ? ka : kb) ? sc : -INFINITY;
        }
        // Column (head) maxima over the 16 tokens: this thread's two rows, then the 8 g lanes.
        float mxa = fmaxf(x[0], x[2]), mxb = fmaxf(x[1], x[3]);
#pragma unroll
        for (int o_ = 4; o_ < 32; o_ <<= 1) {
          mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, o_));
          mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, o_));
        }
        const float mna = fmaxf(m_a, mxa), mnb = fmaxf(m_b, mxb);
        const float alpha_a = exp2f(m_a - mna), alpha_b = exp2f(m_b - mnb);
        float p[4];
        p[0] = exp2f(x[0] - mna);
        p[1] = exp2f(x[1] - mnb);
        p[2] = exp2f(x[2] - mna);
        p[3] = exp2f(x[3] - mnb);
        l_a = l_a * alpha_a + (p[0] + p[2]);
        l_b = l_b * alpha_b + (p[1] + p[3]);
        m_a = mna;
        m_b = mnb;
#pragma unroll
        for (int n = 0; n < D / 16; ++n) {
          o[n][0] *= alpha_a;
          o[n][1] *= alpha_b;
          o[n][2] *= alpha_a;
          o[n][3] *= alpha_b;
        }
        // O^T += V^T P^T (m = 16 dims, n = 8 heads, k = 16 tokens).  The P^T values of this thread
        // are [token g | g+8][heads 2t, 2t+1], the layout of an 8x8 fragment; one transpose per 8
        // tokens turns them into the B fragment P[head g][tokens 2t, 2t+1 | 8+2t, 9+2t].
        uint32_t pb0, pb1;
        movmatrix_trans(pack_bf16(p[0], p[1]), pb0);
        movmatrix_trans(pack_bf16(p[2], p[3]), pb1);
        // A = V^T, one transposed ldmatrix.x4 per 16 dims: matrices (dims 0-7 | 8-15) x
        // (tokens 0-7 | 8-15) in the fragment order a0 a1 a2 a3.
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) {
          const int part = mt >> 2;
          const int mi = lane >> 3;
          const int tok = (mi >> 1) * 8 + (lane & 7);
          const int chunk = (mt & 3) * 2 + (mi & 1);
          const int line = attn_line<HKV, D>(1, part, h, tok);
          const uint32_t addr = stage_base + line * 128 + ((chunk ^ (line & 7)) << 4);
          uint32_t v0, v1, v2, v3;
          ldsm_x4_t(addr, v0, v1, v2, v3);
          mma_bf16_16816(o[mt], v0, v1, v2, v3, pb0, pb1);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }

      // Segment done: finish this warp's GROUP heads.  This thread's O^T columns are heads 2t and
      // 2t+1; their denominators are summed over the 8 g lanes.
#pragma unroll
      for (int o_ = 4; o_ < 32; o_ <<= 1) {
        l_a += __shfl_xor_sync(0xffffffffu, l_a, o_);
        l_b += __shfl_xor_sync(0xffffffffu, l_b, o_);
      }
      const int ha = 2 * t, hb = 2 * t + 1;
      const bool va = ha < GROUP, vb = hb < GROUP;
      float ma = m_a, la = l_a, mb = m_b, lb = l_b;
      if constexpr (W > 1) {
        // Combine the W warps of head h: each publishes (m, l, o) of its GROUP heads as rows of
        // D + 2 floats (a warp that had no block in the segment contributes m = -inf, l = 0,
        // o = 0), then each merges a share of the dims.
        constexpr int RS = D + 2;
        float* mine = combine_smem + static_cast<int64_t>(warp) * GROUP * RS;
        if (g == 0) {
          if (va) {
            mine[ha * RS] = ma;
            mine[ha * RS + 1] = la;
          }
          if (vb) {
            mine[hb * RS] = mb;
            mine[hb * RS + 1] = lb;
          }
        }
#pragma unroll
        for (int n = 0; n < D / 16; ++n) {
          const int d0 = 16 * n + g;
          if (va) {
            mine[ha * RS + 2 + d0] = o[n][0];
            mine[ha * RS + 2 + d0 + 8] = o[n][2];
          }
          if (vb) {
            mine[hb * RS + 2 + d0] = o[n][1];
            mine[hb * RS + 2 + d0 + 8] = o[n][3];
          }
        }
        head_bar<W>(h);
        // Every warp merges the dims it owns (m-tiles n with n % W == w) for the head's GROUP query
        // heads; the per-head max and denominator are formed redundantly by all W warps.
        const float* base = combine_smem + static_cast<int64_t>(h * W) * GROUP * RS;
        float Ma = -INFINITY, Mb = -INFINITY;
#pragma unroll
        for (int ww = 0; ww < W; ++ww) {
          if (va) Ma = fmaxf(Ma, base[ww * GROUP * RS + ha * RS]);
          if (vb) Mb = fmaxf(Mb, base[ww * GROUP * RS + hb * RS]);
        }
        float La = 0.0f, Lb = 0.0f;
#pragma unroll 1
        for (int ww = 0; ww < W; ++ww) {
          const float* r = base + ww * GROUP * RS;
          if (va && r[ha * RS] != -INFINITY) La += r[ha * RS + 1] * exp2f(r[ha * RS] - Ma);
          if (vb && r[hb * RS] != -INFINITY) Lb += r[hb * RS + 1] * exp2f(r[hb * RS] - Mb);
        }
#pragma unroll
        for (int n = 0; n < D / 16; ++n) {
          if (n % W != w) continue;
          float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
#pragma unroll 1
          for (int ww = 0; ww < W; ++ww) {
            const float* r = base + ww * GROUP * RS;
            if (va && r[ha * RS] != -INFINITY) {
              const float sc = exp2f(r[ha * RS] - Ma);
              s0 += r[ha * RS + 2 + 16 * n + g] * sc;
              s2 += r[ha * RS + 2 + 16 * n + g + 8] * sc;
            }
            if (vb && r[hb * RS] != -INFINITY) {
              const float sc = exp2f(r[hb * RS] - Mb);
              s1 += r[hb * RS + 2 + 16 * n + g] * sc;
              s3 += r[hb * RS + 2 + 16 * n + g + 8] * sc;
            }
          }
          o[n][0] = s0;
          o[n][1] = s1;
          o[n][2] = s2;
          o[n][3] = s3;
        }
        ma = Ma;
        la = La;
        mb = Mb;
        lb = Lb;
        head_bar<W>(h);  // the area is rewritten by the next segment
      }
      // m-tiles this warp writes: all of them, or after a W-warp combine those with n % W == w.
      auto owns = [&](int n) { return W == 1 || n % W == w; };
      if (whole) {
        __nv_bfloat16* op = a.out + static_cast<int64_t>(b) * a.out_stride + static_cast<int64_t>(hq0) * D;
        const float ia = va ? 1.0f / la : 0.0f, ib = vb ? 1.0f / lb : 0.0f;
#pragma unroll
        for (int n = 0; n < D / 16; ++n) {
          if (!owns(n)) continue;
          const int d0 = 16 * n + g;
          if (va) {
            op[ha * D + d0] = __float2bfloat16_rn(o[n][0] * ia);
            op[ha * D + d0 + 8] = __float2bfloat16_rn(o[n][2] * ia);
          }
          if (vb) {
            op[hb * D + d0] = __float2bfloat16_rn(o[n][1] * ib);
            op[hb * D + d0 + 8] = __float2bfloat16_rn(o[n][3] * ib);
          }
        }
      } else {
        const int slot = (g_begin >= seq_lo) ? 2 * blockIdx.x : 2 * blockIdx.x + 1;
        const int c_first = cta_of(seq_lo, total, G);
        const int nc = cta_of(seq_hi - 1, total, G) - c_first + 1;  // contributors of the sequence
        // Thread 0 only: every other contributor had arrived when the count was read, so this
        // CTA is the last one.  The fence turns that relaxed read into an acquire of their
        // partials; it comes before this thread's own stores, so it has nothing to wait for.
        const bool known_last = early_read && early_count == static_cast<uint32_t>(nc - 1);
        if (known_last) fence_acq_rel_gpu();
        // query heads h*GROUP + ha / hb within the head group
        float* po = a.partial_o + (static_cast<int64_t>(slot) * HQ + h * GROUP) * D;
        const float ia = va ? 1.0f / la : 0.0f, ib = vb ? 1.0f / lb : 0.0f;
#pragma unroll
        for (int n = 0; n < D / 16; ++n) {
          if (!owns(n)) continue;
          const int d0 = 16 * n + g;
          if (va) {
            __stcg(po + ha * D + d0, o[n][0] * ia);
            __stcg(po + ha * D + d0 + 8, o[n][2] * ia);
          }
          if (vb) {
            __stcg(po + hb * D + d0, o[n][1] * ib);
            __stcg(po + hb * D + d0 + 8, o[n][3] * ib);
          }
        }
        float2* pml = a.partial_ml + static_cast<int64_t>(slot) * HQ + h * GROUP;
        if (w == 0 && g == 0) {
          if (va) __stcg(pml + ha, make_float2(ma, la));
          if (vb) __stcg(pml + hb, make_float2(mb, lb));
        }
        // Arrival: after the barrier, thread 0's fence orders the whole CTA's partial stores before
        // its relaxed increment (a release), and a last arriver's second fence acquires the other
        // contributors' partials.  A known last arriver neither increments nor fences again (the
        // merge below reads this CTA's own partial after the CTA barriers).
        consumer_bar<NCW>();
        if (threadIdx.x == 0) {
          int last = 1;
          if (!known_last) {
            fence_acq_rel_gpu();
            const int old = atomicAdd(&a.counters[vs], 1);
            last = old == nc - 1;
            if (last) fence_acq_rel_gpu();
          }
          *last_flag = last;
        }
        consumer_bar<NCW>();
        if (*last_flag) {
          // Merge the sequence's nc partials in contributor order (deterministic).  Thread t owns
          // PER consecutive dims of query head t / TPH and folds the contributors in with an online
          // softmax (running max, denominator and weighted sum of the normalised partials), loading
          // JB contributors' (m, l) pairs and dims at a time: one round of global loads per JB
          // contributors, no shared memory and no barrier.
          constexpr int NT = NCW * 32;
          constexpr int PER = HQ * D / NT;
          constexpr int TPH = D / PER;  // threads per query head
          static_assert(PER * NT == HQ * D && TPH * PER == D, "merge share must be whole");
          // Contributors per round of loads, as many as the registers allow without spilling.
          constexpr int JB = (PER >= 32 || (CPS == 2 && PER >= 16)) ? 1
                             : (PER >= 16 ? 2 : (16 / PER > 4 ? 4 : 16 / PER));
          const int hh = threadIdx.x / TPH;
          const int d0 = (threadIdx.x - hh * TPH) * PER;
          auto slot_of = [&](int j) {
            const int c = c_first + j;
            return range_start(c, total, G) >= seq_lo ? 2 * c : 2 * c + 1;
          };
          float M = -INFINITY, den = 0.0f;
          float acc[PER];
#pragma unroll
          for (int k = 0; k < PER; ++k) acc[k] = 0.0f;
          for (int j0 = 0; j0 < nc; j0 += JB) {
            float2 ml[JB];
            float ov[JB][PER];
#pragma unroll
            for (int jj = 0; jj < JB; ++jj) {
              if (j0 + jj < nc) {
                const int64_t sl = slot_of(j0 + jj);
                ml[jj] = __ldcg(a.partial_ml + sl * HQ + hh);
                const float* po = a.partial_o + (sl * HQ + hh) * D + d0;
                if constexpr (PER % 4 == 0) {
#pragma unroll
                  for (int k = 0; k < PER; k += 4) {
                    const float4 v = __ldcg(reinterpret_cast<const float4*>(po + k));
                    ov[jj][k] = v.x;
                    ov[jj][k + 1] = v.y;
                    ov[jj][k + 2] = v.z;
                    ov[jj][k + 3] = v.w;
                  }
                } else {
#pragma unroll
                  for (int k = 0; k < PER; ++k) ov[jj][k] = __ldcg(po + k);
                }
              }
            }
#pragma unroll
            for (int jj = 0; jj < JB; ++jj) {
              if (j0 + jj < nc) {
                const float Mn = fmaxf(M, ml[jj].x);
                const float keep = exp2f(M - Mn);  // 0 for the first contributor
                const float wj = ml[jj].y * exp2f(ml[jj].x - Mn);
                den = den * keep + wj;
#pragma unroll
                for (int k = 0; k < PER; ++k) acc[k] = acc[k] * keep + wj * ov[jj][k];
                M = Mn;
              }
            }
          }
          const float inv = 1.0f / den;
          __nv_bfloat16* og = a.out + static_cast<int64_t>(b) * a.out_stride +
                              static_cast<int64_t>(hg) * HQ * D + hh * D + d0;
          if constexpr (PER % 2 == 0) {
#pragma unroll
            for (int k = 0; k < PER; k += 2)
              *reinterpret_cast<__nv_bfloat162*>(og + k) = __floats2bfloat162_rn(acc[k] * inv, acc[k + 1] * inv);
          } else {
#pragma unroll
            for (int k = 0; k < PER; ++k) og[k] = __float2bfloat16_rn(acc[k] * inv);
          }
          if (threadIdx.x == 0) a.counters[vs] = 0;
        }
        consumer_bar<NCW>();
      }
      gpos = seg_end;
    }
  }

  __syncthreads();
  if (warp == NCW && lane == 0) {
    const int first = issued > STAGES ? issued - STAGES : 0;
    for (int it = first; it < issued; ++it) mbar_wait(&full[it % STAGES], (it / STAGES) & 1, nullptr, a.err);
  }
}

// Most (sequence, head group) pairs one launch takes: their block prefix sums live in shared
// memory, so at D = 256 (32 KB stages) the bound is lower to leave room for a sixth stage, and
// the two-CTA form (CPS = 2) keeps kDualMaxPairs.
template <int D, int CPS>
constexpr int attn_max_pairs() {
  return CPS == 2 ? kDualMaxPairs : (D == 128 ? 4096 : 1024);
}

// Shared memory other than the stages, at the largest batch: barriers, the block prefix sums,
// the per-head combine and the 1 KB alignment slack.
template <int GROUP, int HKV, int D, int CPS>
constexpr int attn_fixed_smem() {
  return 2 * 8 * 32 + 16 + 4 * (attn_max_pairs<D, CPS>() + 1) + 16 + attn_combine_bytes<GROUP, HKV, D>() + 1024;
}

// As many stages as fit next to the rest (at most 24) in 227 KB, or in 112 KB when two CTAs share
// an SM (CPS = 2), rounded down to a multiple of
// the warps per head: iteration `it` uses stage it % STAGES and warp it % W of each head, so with
// STAGES % W == 0 a stage only ever serves the same warp of each head, in iteration order.  A warp
// therefore never waits on a stage more than one phase ahead of its last use, where the
// mbarrier's parity would alias a stale phase as complete.
template <int GROUP, int HKV, int D, int CPS>
constexpr int attn_stages() {
  constexpr int stage = 2 * (D / 64) * HKV * HALF_BYTES_PER_HEAD;
  constexpr int W = attn_wph<GROUP, HKV, D>();
  constexpr int budget = CPS == 2 ? 112 * 1024 : 227 * 1024;
  constexpr int n = (budget - attn_fixed_smem<GROUP, HKV, D, CPS>()) / stage;
  constexpr int c = n > 24 ? 24 : n;
  return c / W * W;
}

template <int GROUP, int HKV, int D, int CPS>
size_t attn_smem(int nv) {
  return static_cast<size_t>(attn_stages<GROUP, HKV, D, CPS>()) * 2 * (D / 64) * HKV * HALF_BYTES_PER_HEAD +
         2 * 8 * 32 + 16 + 4 * (nv + 1) + 16 + attn_combine_bytes<GROUP, HKV, D>() + 1024;
}

template <int GROUP, int HKV, int D, bool CAP, int CPS>
int launch_attn_cps(const CUtensorMap& tm, const AttnArgs& a, int grid, cudaStream_t st) {
  constexpr int S = attn_stages<GROUP, HKV, D, CPS>();
  static_assert(S >= 2, "two stages must fit");
  constexpr int NT = (HKV * attn_wph<GROUP, HKV, D>() + 1) * 32;
  const size_t smem = attn_smem<GROUP, HKV, D, CPS>(a.batch * a.nhg);
  // Raise the kernel's dynamic-smem limit once per device (to the largest pair count), so no
  // attribute call happens while a stream is being captured into a graph.
  static unsigned long long done_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(done_mask & (1ull << dev))) {
    MVB_TRY(set_smem(paged_attention_kernel<GROUP, HKV, S, D, CAP, CPS>,
                     attn_smem<GROUP, HKV, D, CPS>(attn_max_pairs<D, CPS>()), "paged_attention: smem attribute"));
    if (dev < 64) done_mask |= 1ull << dev;
  }
  return launch("paged_attention_decode", paged_attention_kernel<GROUP, HKV, S, D, CAP, CPS>, dim3(grid), dim3(NT),
                smem, st, tm, a);
}

template <int GROUP, int HKV, int D, bool CAP>
int launch_attn_cap(const CUtensorMap& tm, const AttnArgs& a, int grid, bool dual, cudaStream_t st) {
  if constexpr (attn_dual_for(HKV, D)) {
    if (dual) return launch_attn_cps<GROUP, HKV, D, CAP, 2>(tm, a, grid, st);
  }
  return launch_attn_cps<GROUP, HKV, D, CAP, 1>(tm, a, grid, st);
}

template <int GROUP, int HKV, int D>
int launch_attn(const CUtensorMap& tm, const AttnArgs& a, int grid, bool dual, cudaStream_t st) {
  return a.cap_log2 > 0.0f ? launch_attn_cap<GROUP, HKV, D, true>(tm, a, grid, dual, st)
                           : launch_attn_cap<GROUP, HKV, D, false>(tm, a, grid, dual, st);
}

template <int HKV, int D>
int dispatch_group(int group, const CUtensorMap& tm, const AttnArgs& a, int grid, bool dual, cudaStream_t st) {
  switch (group) {
    case 1: return launch_attn<1, HKV, D>(tm, a, grid, dual, st);
    case 2: return launch_attn<2, HKV, D>(tm, a, grid, dual, st);
    case 4: return launch_attn<4, HKV, D>(tm, a, grid, dual, st);
    case 8: return launch_attn<8, HKV, D>(tm, a, grid, dual, st);
    default: return fail(MVB_ERR_UNSUPPORTED, "paged attention: %d query heads per KV head", group);
  }
}

int64_t attn_counters_bytes(int64_t batch) { return (batch * 4 + 255) / 256 * 256; }

// KV heads one CTA stage holds (a head group): all of them at D = 128, two (or one) at D = 256.
int64_t attn_heads_per_group(int64_t hkv, int64_t d) { return d == 128 ? hkv : (hkv % 2 == 0 ? 2 : 1); }

// The KV-pool tensor map.  One-copy layout: dims (innermost first) 64 dims of a part, NP*Hkv
// (head, part) lines of 128 bytes, 16 tokens, blocks, layer*2 + kv; one box = K and V of one
// block for the hs heads of a head group.  Split layout (D = 128): dims 128 dims, 16 tokens,
// Hkv heads (strides permuted so a box lands as [head][token][64]), rows = (layer*2 + kv)*P +
// block; one box = one part of K or V of hs heads.
int encode_kv_map(CUtensorMap* m, const void* kv, int64_t hkv, int64_t d, int64_t hs, int64_t num_blocks,
                  int64_t num_layers, bool one_copy) {
  const uint64_t block_bytes = static_cast<uint64_t>(BS * hkv * d * 2);
  if (one_copy) {
    const uint64_t dims[5] = {64, static_cast<uint64_t>(d / 64 * hkv), static_cast<uint64_t>(BS),
                              static_cast<uint64_t>(num_blocks), static_cast<uint64_t>(2 * num_layers)};
    const uint64_t strides[4] = {128, static_cast<uint64_t>(hkv * d * 2), block_bytes,
                                 block_bytes * static_cast<uint64_t>(num_blocks)};
    const uint32_t box[5] = {64, static_cast<uint32_t>(d / 64 * hs), BS, 1, 2};
    return encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, kv, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  const uint64_t dims[4] = {static_cast<uint64_t>(d), static_cast<uint64_t>(BS), static_cast<uint64_t>(hkv),
                            static_cast<uint64_t>(2 * num_layers * num_blocks)};
  const uint64_t strides[3] = {static_cast<uint64_t>(hkv * d * 2), static_cast<uint64_t>(d * 2), block_bytes};
  const uint32_t box[4] = {64, BS, static_cast<uint32_t>(hs), 1};
  return encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, kv, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace
}  // namespace mvb

using namespace mvb;

extern "C" int64_t mvb_paged_attention_workspace_bytes(int64_t batch, int64_t num_q_heads, int64_t head_dim,
                                                       int device) {
  int sms = mvb_num_sms(device);
  if (sms <= 0) sms = 148;
  // counters: one per (sequence, head group); head groups <= KV heads <= query heads; partials
  // for two slots per CTA, up to two CTAs per SM
  const int64_t grid = 2LL * sms;
  return attn_counters_bytes(batch * num_q_heads) + 2LL * grid * num_q_heads * 8 +
         2LL * grid * num_q_heads * head_dim * 4 + 256;
}

extern "C" int mvb_paged_attention_decode_ex(void* out, int64_t out_stride, const void* q, int64_t q_stride,
                                             const void* kv_cache, const int32_t* block_tables, int64_t max_blocks,
                                             const int32_t* ctx_lens, int64_t batch, int64_t num_q_heads,
                                             int64_t num_kv_heads, int64_t head_dim, int64_t num_layers,
                                             int64_t layer, int64_t num_blocks, int64_t block_size, float scale,
                                             float softcap, int64_t window, void* workspace,
                                             int64_t workspace_bytes, mvb_stream_t stream) {
  MVB_REQUIRE(out && q && kv_cache && block_tables && ctx_lens && workspace,
              "mvb_paged_attention_decode: null pointer");
  MVB_REQUIRE(head_dim == 128 || head_dim == 256, "mvb_paged_attention_decode: head_dim %lld (128 or 256)",
              (long long)head_dim);
  MVB_REQUIRE(block_size == BS, "mvb_paged_attention_decode: block_size %lld (this build: 16)",
              (long long)block_size);
  MVB_REQUIRE(num_kv_heads > 0 && num_q_heads % num_kv_heads == 0, "mvb_paged_attention_decode: head counts");
  MVB_REQUIRE(softcap >= 0.0f && window >= 0 && window <= (1LL << 30),
              "mvb_paged_attention_decode: softcap and window must be >= 0");
  const int64_t hs = attn_heads_per_group(num_kv_heads, head_dim);
  const int64_t nhg = num_kv_heads / hs;
  const int max_pairs = head_dim == 128 ? attn_max_pairs<128, 1>() : attn_max_pairs<256, 1>();
  MVB_REQUIRE(batch >= 0 && batch * nhg <= max_pairs,
              "mvb_paged_attention_decode: batch %lld x %lld head groups > %d", (long long)batch, (long long)nhg,
              max_pairs);
  MVB_REQUIRE(layer >= 0 && layer < num_layers && num_blocks > 0 && max_blocks > 0,
              "mvb_paged_attention_decode: cache geometry");
  MVB_REQUIRE(q_stride % 2 == 0 && aligned(q, 4) && out_stride % 2 == 0 && aligned(out, 4),
              "mvb_paged_attention_decode: q/out must be 4-byte aligned with even strides");
  MVB_REQUIRE(aligned(kv_cache, 16) && aligned(workspace, 256), "mvb_paged_attention_decode: alignment");
  if (batch == 0) return MVB_OK;
  const int64_t group = num_q_heads / num_kv_heads;
  const int sms = current_sm_count();
  MVB_REQUIRE(sms > 0, "mvb_paged_attention_decode: no device");
  // Partials at the head, per-(sequence, head group) counters at the tail (nested suffixes
  // across calls of different batch sizes sharing one buffer; the kernel leaves them zero).
  const int64_t ws_end = workspace_bytes / 256 * 256;
  const int64_t cbytes = attn_counters_bytes(batch * nhg);
  const bool dual = attn_dual_for(static_cast<int>(hs), static_cast<int>(head_dim)) && batch * nhg <= kDualMaxPairs;
  const int grid = sms * (dual ? 2 : 1);
  const int64_t need = cbytes + 2LL * grid * num_q_heads * 8 + 2LL * grid * num_q_heads * head_dim * 4;
  MVB_REQUIRE(ws_end >= need, "mvb_paged_attention_decode: workspace %lld < %lld", (long long)workspace_bytes,
              (long long)need);

  CUtensorMap tm;
  MVB_TRY(encode_kv_map(&tm, kv_cache, num_kv_heads, head_dim, hs, num_blocks, num_layers,
                        attn_one_copy_for(static_cast<int>(hs), static_cast<int>(head_dim))));

  AttnArgs a;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_stride = out_stride;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_stride = q_stride;
  a.block_tables = block_tables;
  a.max_blocks = max_blocks;
  a.ctx_lens = ctx_lens;
  a.batch = static_cast<int>(batch);
  a.nhg = static_cast<int>(nhg);
  a.window = static_cast<int>(window);
  a.layer = layer;
  a.num_blocks = num_blocks;
  a.scale_log2 = scale * kLog2e;
  a.cap_scale = softcap > 0.0f ? scale / softcap : 0.0f;
  a.cap_log2 = softcap > 0.0f ? softcap * kLog2e : 0.0f;
  char* ws = static_cast<char*>(workspace);
  a.partial_ml = reinterpret_cast<float2*>(ws);
  a.partial_o = reinterpret_cast<float*>(ws + 2LL * grid * num_q_heads * 8);
  a.counters = reinterpret_cast<int*>(ws + ws_end - cbytes);
  a.err = device_status_ptr();
  // Grid: persistent CTAs, one per SM (192 KB of stages each) or two (the dual form); never
  // more CTAs than blocks.  The block total is only known on the device, so the grid is fixed
  // and CTAs with an empty range exit after the prologue.
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int g = static_cast<int>(group);
  if (head_dim == 256) {
    if (hs == 2) return dispatch_group<2, 256>(g, tm, a, grid, dual, st);
    return dispatch_group<1, 256>(g, tm, a, grid, dual, st);
  }
  switch (num_kv_heads) {
    case 1: return dispatch_group<1, 128>(g, tm, a, grid, dual, st);
    case 2: return dispatch_group<2, 128>(g, tm, a, grid, dual, st);
    case 4: return dispatch_group<4, 128>(g, tm, a, grid, dual, st);
    case 8: return dispatch_group<8, 128>(g, tm, a, grid, dual, st);
    default: return fail(MVB_ERR_UNSUPPORTED, "mvb_paged_attention_decode: %lld KV heads", (long long)num_kv_heads);
  }
}

extern "C" int mvb_paged_attention_decode(void* out, int64_t out_stride, const void* q, int64_t q_stride,
                                          const void* kv_cache, const int32_t* block_tables, int64_t max_blocks,
                                          const int32_t* ctx_lens, int64_t batch, int64_t num_q_heads,
                                          int64_t num_kv_heads, int64_t head_dim, int64_t num_layers, int64_t layer,
                                          int64_t num_blocks, int64_t block_size, float scale, void* workspace,
                                          int64_t workspace_bytes, mvb_stream_t stream) {
  return mvb_paged_attention_decode_ex(out, out_stride, q, q_stride, kv_cache, block_tables, max_blocks, ctx_lens,
                                       batch, num_q_heads, num_kv_heads, head_dim, num_layers, layer, num_blocks,
                                       block_size, scale, 0.0f, 0, workspace, workspace_bytes, stream);
}

// ---------------------------------------------------------------------------------
// Allocation-free variant.  Some callers cannot allocate device memory: a host runtime
// that reaches this library only through its C ABI and owns no device allocator, or a
// server that has already handed all of HBM to the KV pool and cannot afford cudaMalloc's
// implicit device-wide synchronisation on the decode path.  For them the split-KV scratch
// lives in a fixed area compiled into the library instead of a caller-provided workspace.
namespace {

// 6 MiB: partials for up to 32 query heads of 128 dims on a 148-SM B200 (~4.9 MB) plus the
// per-sequence counters of up to 4096 sequences.  Every GPU that loads the library holds
// this area until the process exits.
constexpr int64_t kNoAllocScratchBytes = 6LL << 20;
static __device__ __align__(256) unsigned char g_attn_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[64] = {};  // device address of g_attn_scratch, per device

}  // namespace

extern "C" int mvb_paged_attention_decode_noalloc(void* out, int64_t out_stride, const void* q, int64_t q_stride,
                                                  const void* kv_cache, const int32_t* block_tables,
                                                  int64_t max_blocks, const int32_t* ctx_lens, int64_t batch,
                                                  int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                                                  int64_t num_layers, int64_t layer, int64_t num_blocks,
                                                  int64_t block_size, float scale, mvb_stream_t stream) {
  int dev = 0;
  MVB_TRY(cuda_status(cudaGetDevice(&dev), "mvb_paged_attention_decode_noalloc: cudaGetDevice"));
  MVB_REQUIRE(dev >= 0 && dev < 64, "mvb_paged_attention_decode_noalloc: device %d out of range", dev);
  void* scratch = nullptr;
  {
    // Set-up on the first call on each device (the current one): host code cannot use the
    // array's name as a device address, so look the address up and keep it.  The address is
    // kept for the life of the process: a device reset (cudaDeviceReset) after the first call
    // reloads the module, and the kept address would then be stale, so resetting a device that
    // this entry point has used is not supported.
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (g_scratch_ptr[dev] == nullptr) {
      void* p = nullptr;
      MVB_TRY(cuda_status(cudaGetSymbolAddress(&p, g_attn_scratch),
                          "mvb_paged_attention_decode_noalloc: cudaGetSymbolAddress"));
      g_scratch_ptr[dev] = p;
    }
    scratch = g_scratch_ptr[dev];
  }
  const int sms = current_sm_count();
  MVB_REQUIRE(sms > 0, "mvb_paged_attention_decode_noalloc: no device");
  MVB_REQUIRE(num_q_heads > 0 && num_kv_heads > 0 && head_dim > 0 && batch >= 0 && batch <= 4096,
              "mvb_paged_attention_decode_noalloc: bad shape");
  const int64_t hs = attn_heads_per_group(num_kv_heads, head_dim);
  const int64_t cbytes = attn_counters_bytes(batch * (num_kv_heads / hs));
  const bool dual = attn_dual_for(static_cast<int>(hs), static_cast<int>(head_dim)) && batch * (num_kv_heads / hs) <=
                    kDualMaxPairs;
  const int64_t grid = static_cast<int64_t>(sms) * (dual ? 2 : 1);
  const int64_t need = cbytes + 2LL * grid * num_q_heads * 8 + 2LL * grid * num_q_heads * head_dim * 4;
  if (need > kNoAllocScratchBytes)
    return fail(MVB_ERR_UNSUPPORTED,
                "mvb_paged_attention_decode_noalloc: %lld query heads x %lld dims on %d SMs need %lld bytes of "
                "scratch; the built-in area holds %lld (use mvb_paged_attention_decode with a workspace)",
                (long long)num_q_heads, (long long)head_dim, sms, (long long)need, (long long)kNoAllocScratchBytes);
  if (batch == 0) return MVB_OK;
  // The area keeps whatever the previous call left.  A call that completes leaves its counters
  // at zero, but one whose kernel gave up on a bounded wait may not; the per-sequence counters
  // must start at zero, so clear them (they sit at the tail) in stream order before the kernel.
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MVB_TRY(cuda_status(cudaMemsetAsync(static_cast<char*>(scratch) + kNoAllocScratchBytes - cbytes, 0, cbytes, st),
                      "mvb_paged_attention_decode_noalloc: clear counters"));
  return mvb_paged_attention_decode(out, out_stride, q, q_stride, kv_cache, block_tables, max_blocks, ctx_lens, batch,
                                    num_q_heads, num_kv_heads, head_dim, num_layers, layer, num_blocks, block_size,
                                    scale, scratch, kNoAllocScratchBytes, stream);
}
