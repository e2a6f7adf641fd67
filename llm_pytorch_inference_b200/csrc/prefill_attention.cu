// Causal attention of a batched prefill, K/V read from the paged pool.
//
// Replaces, for the prompt of each new sequence, the causal SDPA of the reference's prefill
// (models/model.py:206-221 with is_causal=True, over the K/V that Attention._write_kv_cache has
// just stored, :226-243):
//   out[t, h] = softmax_{k <= t}(q[t, h] . K[k]^T * scale) V[k]      for every prompt token t.
//
// Work item = (sequence, 16-token query tile, KV head): one CTA.  The tile's 16 query tokens share
// every K/V block of the prefix (blocks 0 .. qt), so each block is read once per 16 queries rather
// than once per query.  Items are independent: no split-KV, no merge.
//
// CTA = 8 consumer warps + 1 producer warp.  The producer streams the KV head's K and V of each
// block through TMA (one copy per (K|V, 64-dim part), 8 KB per stage at head dim 128) into a
// 128-byte-swizzled [kv][part][token][64] image.  Consumer warp w owns query tokens 2w and 2w+1 of
// the tile: its 2 x GROUP query columns (token-major) are the n = 8 side of the transposed tiles
// used by the decode kernel -- S^T = K Q^T, then O^T = V^T P^T with P^T passed to the B operand by
// an 8x8 transpose -- and every warp consumes every stage.  The causal mask is per column: key k
// is visible to the column's query at position p when k <= p.  Online softmax in the exp2 domain.
#include "common.cuh"
#include "host.h"
#include "mma_sync.cuh"

namespace mvb {
namespace {

constexpr int PBS = 16;                      // tokens per KV block and per query tile
constexpr int kPfWarps = 8;                  // consumer warps; 2 query tokens each
constexpr int kPfStages = 12;
constexpr int kPfPart = PBS * 64 * 2;        // 2 KB: 16 tokens x 64 dims of one head

struct PrefillArgs {
  __nv_bfloat16* out;
  int64_t out_stride;
  const __nv_bfloat16* q;
  int64_t q_stride;
  const int32_t* block_tables;  // [num_seqs, max_blocks]
  int64_t max_blocks;
  const int32_t* seq_start;     // first token row of each sequence
  const int32_t* seq_len;
  const int32_t* tile_seq;      // [ntiles] sequence of the tile
  const int32_t* tile_idx;      // [ntiles] query tile index within it
  int num_q_heads;
  int64_t layer;
  int64_t num_blocks;
  float scale_log2;
  unsigned* err;
};

template <int GROUP, int D>
__global__ void __launch_bounds__((kPfWarps + 1) * 32, 2)
    prefill_attention_kernel(const __grid_constant__ CUtensorMap tm, const PrefillArgs a) {
  constexpr int NP = D / 64;
  constexpr int STAGE_BYTES = 2 * NP * kPfPart;
  constexpr int TPW = 2;  // query tokens per warp
  static_assert(TPW * GROUP <= 8, "a warp's columns must fit the n = 8 side of the tile");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPfStages * STAGE_BYTES);
  uint64_t* empty = full + kPfStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kPfStages);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s = a.tile_seq[blockIdx.x];
  const int qt = a.tile_idx[blockIdx.x];
  const int h = blockIdx.y;  // KV head
  const int len = a.seq_len[s];
  const int q0 = qt * PBS;
  // Key blocks 0 .. qt (the tile's last token sits in block qt), never past the table's width: a
  // tile index the block table cannot hold sets the status word, as the decode kernel does.
  int nb = qt + 1;
  if (qt < 0 || nb > a.max_blocks) {
    if (threadIdx.x == 0) report(a.err, kDevBadPosition);
    nb = qt < 0 ? 0 : static_cast<int>(a.max_blocks);
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < kPfStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kPfWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  int issued = 0;
  if (warp == kPfWarps) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tm);
      pdl_wait();  // the K/V of this layer were written by the previous kernel
      const uint64_t pol = l2_policy_evict_last();  // the prefix is read again by the later tiles
      const int32_t* bt = a.block_tables + static_cast<int64_t>(s) * a.max_blocks;
      for (int j = 0; j < nb; ++j) {
        const int st = j % kPfStages;
        if (!mbar_wait(&empty[st], ((j / kPfStages) & 1) ^ 1, abort_flag, a.err)) break;
        int blk = bt[j];
        if (blk < 0 || blk >= a.num_blocks) {
          report(a.err, kDevBadBlock);
          blk = 0;  // stay in bounds; the output is not trusted (status word set)
        }
        mbar_arrive_expect_tx(&full[st], STAGE_BYTES);
        uint8_t* dst = smem + st * STAGE_BYTES;
        for (int kv = 0; kv < 2; ++kv) {
          const int row = static_cast<int>((a.layer * 2 + kv) * a.num_blocks + blk);
          for (int part = 0; part < NP; ++part)
            tma_load_4d(dst + (kv * NP + part) * kPfPart, &tm, &full[st], part * 64, 0, h, row, pol);
        }
        issued = j + 1;
      }
    }
  } else {
    // ------------------------------------------------------------------ consumers
    pdl_wait();
    const int g = lane >> 2, t = lane & 3;
    // This lane's B-operand column g: query token q0 + 2*warp + g / GROUP, head h*GROUP + g % GROUP.
    const int tok_g = q0 + TPW * warp + g / GROUP;
    const bool col_ok = g < TPW * GROUP && tok_g < len;
    uint32_t qa[D / 16][2];
    {
      const __nv_bfloat16* qp = a.q + static_cast<int64_t>(a.seq_start[s] + (col_ok ? tok_g : 0)) * a.q_stride +
                                static_cast<int64_t>(h * GROUP + g % GROUP) * D;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        if (col_ok) {
          qa[kk][0] = *reinterpret_cast<const uint32_t*>(qp + kk * 16 + 2 * t);
          qa[kk][1] = *reinterpret_cast<const uint32_t*>(qp + kk * 16 + 8 + 2 * t);
        } else {
          qa[kk][0] = qa[kk][1] = 0u;
        }
      }
    }
    // This thread's S^T / O^T columns 2t and 2t+1: their query positions (-1 = no query).
    const int ca = 2 * t, cb = 2 * t + 1;
    const int pa = (ca < TPW * GROUP && q0 + TPW * warp + ca / GROUP < len) ? q0 + TPW * warp + ca / GROUP : -1;
    const int pb = (cb < TPW * GROUP && q0 + TPW * warp + cb / GROUP < len) ? q0 + TPW * warp + cb / GROUP : -1;
    float o[D / 16][4];
#pragma unroll
    for (int n = 0; n < D / 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.0f, l_b = 0.0f;
    const uint32_t sbase = smem_u32(smem);
    for (int j = 0; j < nb; ++j) {
      const int st = j % kPfStages;
      mbar_wait(&full[st], (j / kPfStages) & 1, abort_flag, a.err);
      const uint32_t stage_base = sbase + st * STAGE_BYTES;
      float sacc[4][4];
#pragma unroll
      for (int c = 0; c < 4; ++c) sacc[c][0] = sacc[c][1] = sacc[c][2] = sacc[c][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int part = kk >> 2;
        const int mi = lane >> 3;
        const int tok = (mi & 1) * 8 + (lane & 7);
        const int chunk = (kk & 3) * 2 + (mi >> 1);
        const int line = (0 * NP + part) * PBS + tok;
        const uint32_t addr = stage_base + line * 128 + ((chunk ^ (line & 7)) << 4);
        uint32_t k0, k1, k2, k3;
        ldsm_x4(addr, k0, k1, k2, k3);
        mma_bf16_16816(sacc[kk & 3], k0, k1, k2, k3, qa[kk][0], qa[kk][1]);
      }
      // x = S^T[key g | g+8][column 2t | 2t+1], causal-masked per column.
      const int ka = j * PBS + g, kb = ka + 8;
      float x[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float raw = sacc[0][c] + sacc[1][c] + sacc[2][c] + sacc[3][c];
        const int key = c < 2 ? ka : kb;
        const int pos = (c & 1) ? pb : pa;
        x[c] = key <= pos ? raw * a.scale_log2 : -INFINITY;
      }
      float mxa = fmaxf(x[0], x[2]), mxb = fmaxf(x[1], x[3]);
#pragma unroll
      for (int o_ = 4; o_ < 32; o_ <<= 1) {
        mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, o_));
        mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, o_));
      }
      // A column with no visible key yet (no query, or none so far) keeps max -inf: use 0 as
      // the reference so that every exponent is exp2(-inf) = 0 and no NaN appears.
      float mna = fmaxf(m_a, mxa), mnb = fmaxf(m_b, mxb);
      const float ra = mna == -INFINITY ? 0.0f : mna, rb = mnb == -INFINITY ? 0.0f : mnb;
      const float alpha_a = exp2f(m_a - ra), alpha_b = exp2f(m_b - rb);
      float p[4];
      p[0] = exp2f(x[0] - ra);
      p[1] = exp2f(x[1] - rb);
      p[2] = exp2f(x[2] - ra);
      p[3] = exp2f(x[3] - rb);
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
      uint32_t pb0, pb1;
      movmatrix_trans(pack_bf16(p[0], p[1]), pb0);
      movmatrix_trans(pack_bf16(p[2], p[3]), pb1);
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) {
        const int part = mt >> 2;
        const int mi = lane >> 3;
        const int tok = (mi >> 1) * 8 + (lane & 7);
        const int chunk = (mt & 3) * 2 + (mi & 1);
        const int line = (1 * NP + part) * PBS + tok;
        const uint32_t addr = stage_base + line * 128 + ((chunk ^ (line & 7)) << 4);
        uint32_t v0, v1, v2, v3;
        ldsm_x4_t(addr, v0, v1, v2, v3);
        mma_bf16_16816(o[mt], v0, v1, v2, v3, pb0, pb1);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
#pragma unroll
    for (int o_ = 4; o_ < 32; o_ <<= 1) {
      l_a += __shfl_xor_sync(0xffffffffu, l_a, o_);
      l_b += __shfl_xor_sync(0xffffffffu, l_b, o_);
    }
    // Columns 2t / 2t+1: token q0 + 2*warp + c / GROUP, head h*GROUP + c % GROUP.
    const int64_t s0 = a.seq_start[s];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int c = half ? cb : ca;
      const int pos = half ? pb : pa;
      const float l = half ? l_b : l_a;
      if (pos < 0 || l <= 0.0f) continue;
      const float inv = 1.0f / l;
      __nv_bfloat16* op = a.out + (s0 + pos) * a.out_stride + static_cast<int64_t>(h * GROUP + c % GROUP) * D;
#pragma unroll
      for (int n = 0; n < D / 16; ++n) {
        op[16 * n + g] = __float2bfloat16_rn((half ? o[n][1] : o[n][0]) * inv);
        op[16 * n + g + 8] = __float2bfloat16_rn((half ? o[n][3] : o[n][2]) * inv);
      }
    }
  }

  __syncthreads();
  if (warp == kPfWarps && lane == 0) {
    const int first = issued > kPfStages ? issued - kPfStages : 0;
    for (int it = first; it < issued; ++it) mbar_wait(&full[it % kPfStages], (it / kPfStages) & 1, nullptr, a.err);
  }
}

template <int GROUP, int D>
size_t prefill_smem() {
  return static_cast<size_t>(kPfStages) * 2 * (D / 64) * kPfPart + 2 * 8 * kPfStages + 16 + 1024;
}

template <int GROUP, int D>
int launch_prefill(const CUtensorMap& tm, const PrefillArgs& a, dim3 grid, cudaStream_t st) {
  static unsigned long long done_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(done_mask & (1ull << dev))) {
    MVB_TRY(set_smem(prefill_attention_kernel<GROUP, D>, prefill_smem<GROUP, D>(), "prefill_attention: smem"));
    if (dev < 64) done_mask |= 1ull << dev;
  }
  return launch("prefill_attention", prefill_attention_kernel<GROUP, D>, grid, dim3((kPfWarps + 1) * 32),
                prefill_smem<GROUP, D>(), st, tm, a);
}

}  // namespace
}  // namespace mvb

using namespace mvb;

extern "C" int mvb_prefill_attention(void* out, int64_t out_stride, const void* q, int64_t q_stride,
                                     const void* kv_cache, const int32_t* block_tables, int64_t max_blocks,
                                     const int32_t* seq_start, const int32_t* seq_len, const int32_t* tile_seq,
                                     const int32_t* tile_idx, int64_t num_tiles, int64_t num_q_heads,
                                     int64_t num_kv_heads, int64_t head_dim, int64_t num_layers, int64_t layer,
                                     int64_t num_blocks, int64_t block_size, float scale, mvb_stream_t stream) {
  MVB_REQUIRE(out && q && kv_cache && block_tables && seq_start && seq_len && tile_seq && tile_idx,
              "mvb_prefill_attention: null pointer");
  MVB_REQUIRE(head_dim == 128, "mvb_prefill_attention: head_dim %lld (this build: 128)", (long long)head_dim);
  MVB_REQUIRE(block_size == PBS, "mvb_prefill_attention: block_size %lld (this build: 16)", (long long)block_size);
  MVB_REQUIRE(num_kv_heads > 0 && num_kv_heads <= 65535 && num_q_heads % num_kv_heads == 0,
              "mvb_prefill_attention: head counts");
  MVB_REQUIRE(num_tiles >= 0 && num_tiles < (1LL << 31), "mvb_prefill_attention: tiles");
  MVB_REQUIRE(layer >= 0 && layer < num_layers && num_blocks > 0 && max_blocks > 0,
              "mvb_prefill_attention: cache geometry");
  MVB_REQUIRE(q_stride % 2 == 0 && aligned(q, 4) && aligned(kv_cache, 16),
              "mvb_prefill_attention: q must be 4-byte aligned with an even stride");
  if (num_tiles == 0) return MVB_OK;
  const int64_t group = num_q_heads / num_kv_heads;
  CUtensorMap tm;
  {
    // dims: 128 dims, 16 tokens, Hkv heads, rows = (layer*2 + kv)*P + block; box: one 64-dim part
    // of one head of one block
    const uint64_t block_bytes = static_cast<uint64_t>(PBS * num_kv_heads * head_dim * 2);
    const uint64_t dims[4] = {static_cast<uint64_t>(head_dim), PBS, static_cast<uint64_t>(num_kv_heads),
                              static_cast<uint64_t>(2 * num_layers * num_blocks)};
    const uint64_t strides[3] = {static_cast<uint64_t>(num_kv_heads * head_dim * 2),
                                 static_cast<uint64_t>(head_dim * 2), block_bytes};
    const uint32_t box[4] = {64, PBS, 1, 1};
    MVB_TRY(encode_tiled(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, kv_cache, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B));
  }
  PrefillArgs a;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_stride = out_stride;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_stride = q_stride;
  a.block_tables = block_tables;
  a.max_blocks = max_blocks;
  a.seq_start = seq_start;
  a.seq_len = seq_len;
  a.tile_seq = tile_seq;
  a.tile_idx = tile_idx;
  a.num_q_heads = static_cast<int>(num_q_heads);
  a.layer = layer;
  a.num_blocks = num_blocks;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.err = device_status_ptr();
  const dim3 grid(static_cast<unsigned>(num_tiles), static_cast<unsigned>(num_kv_heads));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (group) {
    case 1: return launch_prefill<1, 128>(tm, a, grid, st);
    case 2: return launch_prefill<2, 128>(tm, a, grid, st);
    case 4: return launch_prefill<4, 128>(tm, a, grid, st);
    default:
      return fail(MVB_ERR_UNSUPPORTED, "mvb_prefill_attention: %lld query heads per KV head (1, 2 or 4)",
                  (long long)group);
  }
}
