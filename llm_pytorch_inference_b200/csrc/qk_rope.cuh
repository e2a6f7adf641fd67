// Per-head QK RMSNorm + NeoX RoPE + paged KV-cache write of one new token, for one warp.
//
// Shared by the standalone kernel (qk_rope_cache.cu) and the fused decoder-layer kernel
// (layer.cu).  It replaces, for a single new token per sequence, the chain
//   q_norm / k_norm            models/model.py:174-178   (RMSNorm.forward, model.py:19-25)
//   apply_rotary_pos_emb       models/model.py:184       (q*cos + rotate_half(q)*sin, bf16 ops)
//   Attention._write_kv_cache  models/model.py:226-243   (kv[l, 0|1, bt[pos//bs], pos%bs] = k|v)
// Lane l owns head_dim/32 consecutive elements; its rotate_half partner sits 16 lanes away.
// The slot of a token is (block_tables[b][pos / bs], pos % bs) exactly as the reference computes
// it; an out-of-range table index or block id is reported in the device status word and nothing
// is written for that token.
#pragma once

#include "common.cuh"
#include "splitk.cuh"

namespace mvb {


// One warp: the projection's values of head h of sequence b's new token, x[E] for the lane's E
// consecutive features (bf16-rounded): from `qkv` (bf16 rows) or, with `partials`, from the
// split-K partial slots of the GEMM that produced it (summed in contributor order).
template <int D>
__device__ __forceinline__ void qk_load_x(int b, int h, int lane, float (&x)[D / 32],
                                          const __nv_bfloat16* __restrict__ qkv, int64_t qkv_stride,
                                          const float* __restrict__ partials, const SplitKPlan& plan) {
  constexpr int E = D / 32;
  const int d0 = lane * E;
  if (partials == nullptr) {
    const __nv_bfloat16* src = qkv + static_cast<int64_t>(b) * qkv_stride + static_cast<int64_t>(h) * D + d0;
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = __bfloat162float(src[e]);
    return;
  }
  // The lane's E consecutive features sit in one 128-feature tile, read as float4 per contributor.
  const int n0 = h * D + d0;
  const int t = n0 / kSplitBM, r = n0 - t * kSplitBM;
  float acc[E];
  if constexpr (E % 4 == 0) {
#pragma unroll
    for (int e4 = 0; e4 < E; e4 += 4) {
      const float4 q = sk_sum4(partials, plan, t, b, r + e4);
      acc[e4] = q.x;
      acc[e4 + 1] = q.y;
      acc[e4 + 2] = q.z;
      acc[e4 + 3] = q.w;
    }
  } else {
    const int nc = sk_count(plan, t);
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] = 0.0f;
    for (int j = 0; j < nc; ++j) {
      const float* src_p = partials + sk_offset(plan, t, j, b, r);
#pragma unroll
      for (int e = 0; e < E; ++e) acc[e] += __ldcg(src_p + e);
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = bf16_round(acc[e]);
}

// What one warp's head needs besides the projection: the token's slot in the paged pool, the
// norm weights and the cos/sin row of its position.  All of it is step metadata or constant
// tables, so the standalone kernel loads it before waiting on the GEMM that feeds it.
template <int D>
struct QkMeta {
  static_assert(D % 64 == 0, "a lane holds an even number of features");
  // norm weights (norm), cos / sin of the position (rope): the lane's E values as bf16 pairs
  __nv_bfloat162 w[D / 64], c[D / 64], s[D / 64];
  int64_t dst_off;                          // K/V heads: element offset of the token's slot
  bool write;                               // false: bad position or block id (reported), no write
  bool norm;                                // the head has norm weights
  bool rope;                                // the position has a cos/sin row (else q/k are zeroed)
};

template <int D>
__device__ __forceinline__ void qk_meta_load(QkMeta<D>& m, int b, int h, int lane,
                                             const __nv_bfloat16* __restrict__ qnw,
                                             const __nv_bfloat16* __restrict__ knw,
                                             const __nv_bfloat16* __restrict__ cos_t,
                                             const __nv_bfloat16* __restrict__ sin_t, int64_t table_len,
                                             const int32_t* __restrict__ positions,
                                             const int32_t* __restrict__ block_tables, int64_t max_blocks, int nq,
                                             int nkv, int64_t layer, int64_t num_blocks, int bs, unsigned* err) {
  constexpr int E = D / 32;
  const int d0 = lane * E;
  const int pos = positions[b];
  const bool is_q = h < nq, is_k = !is_q && h < nq + nkv;
  m.write = true;
  m.norm = false;
  m.rope = false;
  m.dst_off = -1;
  // Slot of this token in the paged pool (only K/V heads need it).
  if (!is_q) {
    const int64_t bidx = pos / bs;
    if (pos < 0 || bidx >= max_blocks) {
      if (lane == 0) report(err, kDevBadPosition);
      m.write = false;
      return;
    }
    const int64_t blk = block_tables[static_cast<int64_t>(b) * max_blocks + bidx];
    if (blk < 0 || blk >= num_blocks) {
      if (lane == 0) report(err, kDevBadBlock);
      m.write = false;
      return;
    }
    const int kvh = is_k ? h - nq : h - nq - nkv;
    const int64_t which = is_k ? 0 : 1;
    m.dst_off = ((((layer * 2 + which) * num_blocks + blk) * bs + (pos % bs)) * nkv + kvh) * D + d0;
  }
  if (!is_q && !is_k) return;  // V: a plain copy
  const __nv_bfloat16* nw = is_q ? qnw : knw;
  if (nw != nullptr) {
    m.norm = true;
#pragma unroll
    for (int e = 0; e < E / 2; ++e) m.w[e] = reinterpret_cast<const __nv_bfloat162*>(nw + d0)[e];
  }
  if (pos < 0 || pos >= table_len) {
    if (lane == 0) report(err, kDevBadPosition);
  } else {
    m.rope = true;
    const __nv_bfloat16* c = cos_t + static_cast<int64_t>(pos) * D + d0;
    const __nv_bfloat16* sn = sin_t + static_cast<int64_t>(pos) * D + d0;
#pragma unroll
    for (int e = 0; e < E / 2; ++e) {
      m.c[e] = reinterpret_cast<const __nv_bfloat162*>(c)[e];
      m.s[e] = reinterpret_cast<const __nv_bfloat162*>(sn)[e];
    }
  }
}

// Norm, RoPE and store of one head from the projection's values x[E] of the lane's E features
// (already bf16-rounded) and the head's metadata.
template <int D>
__device__ __forceinline__ void qk_apply(const QkMeta<D>& m, int b, int h, int lane, float (&x)[D / 32],
                                         __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ kv,
                                         int nq, int nkv, float eps, int plus_one) {
  constexpr int E = D / 32;
  const int d0 = lane * E;
  if (!m.write) return;
  const bool is_q = h < nq, is_k = !is_q && h < nq + nkv;
  if (!is_q && !is_k) {  // V: plain copy into the cache
#pragma unroll
    for (int e = 0; e < E; ++e) kv[m.dst_off + e] = __float2bfloat16_rn(x[e]);
    return;
  }

  // Per-head RMSNorm (model semantics: T(w * (x * r)); Gemma's plus-one form T((x * r) * (1 + w)),
  // models/gemma3_model.py:21-25).
  if (m.norm) {
    float ss = 0.0f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss += x[e] * x[e];
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float wv = (e & 1) ? __high2float(m.w[e / 2]) : __low2float(m.w[e / 2]);
      x[e] = plus_one ? bf16_round((x[e] * r) * (1.0f + wv)) : bf16_round(wv * (x[e] * r));
    }
  }

  // RoPE with the model's bf16 cos/sin rows: T(T(x*cos) + T(rot(x)*sin)).
  float out[E];
  if (!m.rope) {
#pragma unroll
    for (int e = 0; e < E; ++e) out[e] = 0.0f;
  } else {
    const bool low = lane < 16;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
      const float rot = low ? -partner : partner;
      const float cv = (e & 1) ? __high2float(m.c[e / 2]) : __low2float(m.c[e / 2]);
      const float sv = (e & 1) ? __high2float(m.s[e / 2]) : __low2float(m.s[e / 2]);
      const float a = bf16_round(x[e] * cv);
      const float bb = bf16_round(rot * sv);
      out[e] = a + bb;
    }
  }

  if (is_q) {
    __nv_bfloat16* q = q_out + (static_cast<int64_t>(b) * nq + h) * D + d0;
#pragma unroll
    for (int e = 0; e < E; ++e) q[e] = __float2bfloat16_rn(out[e]);
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) kv[m.dst_off + e] = __float2bfloat16_rn(out[e]);
  }
}

// The same from the projection's values x[E] of the lane's E features (already bf16-rounded).
template <int D>
__device__ __forceinline__ void qk_norm_rope_kv_x(
    int b, int h, int lane, float (&x)[D / 32], __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ kv,
    const __nv_bfloat16* __restrict__ qnw, const __nv_bfloat16* __restrict__ knw,
    const __nv_bfloat16* __restrict__ cos_t, const __nv_bfloat16* __restrict__ sin_t, int64_t table_len,
    const int32_t* __restrict__ positions, const int32_t* __restrict__ block_tables, int64_t max_blocks, int nq,
    int nkv, int64_t layer, int64_t num_blocks, int bs, float eps, int plus_one, unsigned* err) {
  QkMeta<D> m;
  qk_meta_load<D>(m, b, h, lane, qnw, knw, cos_t, sin_t, table_len, positions, block_tables, max_blocks, nq, nkv,
                  layer, num_blocks, bs, err);
  qk_apply<D>(m, b, h, lane, x, q_out, kv, nq, nkv, eps, plus_one);
}

}  // namespace mvb
