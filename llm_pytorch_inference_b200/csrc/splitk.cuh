// Stream-K work split of the decode GEMMs, shared by the GEMM and by the kernels that
// consume its fp32 partials directly (MVB_EPI_PARTIALS).
//
// The linearised (output tile, k-block) space of T = tiles * kblocks k-blocks is cut into
// `grid` contiguous ranges, CTA c owning [c*T/grid, (c+1)*T/grid).  The CTAs whose range meets
// tile t are its contributors c_first(t)..c_last(t); contributor j = c - c_first(t) stores
// its fp32 partial of the tile in slot t*maxc + j, laid out [bn batch columns][128 rows].
// A consumer reads element (b, n) as the sum over j in contributor order (deterministic).
#pragma once

#include <stdint.h>

namespace mvb {

constexpr int kSplitBM = 128;  // output features per tile
constexpr int kSplitBK = 64;   // k per k-block

struct SplitKPlan {
  int grid;     // CTAs
  int tiles;    // output tiles of 128 features
  int kblocks;  // k / 64
  int bn;       // batch columns per tile (64, 128 or 256)
  int maxc;     // most contributors of any tile
};

__host__ __device__ __forceinline__ int64_t sk_range_start(int c, int64_t total, int grid) {
  return static_cast<int64_t>(c) * total / grid;
}

// CTA whose range holds linear k-block x.
__host__ __device__ __forceinline__ int sk_cta_of(int64_t x, int64_t total, int grid) {
  return static_cast<int>(((x + 1) * grid + total - 1) / total - 1);
}

__host__ __device__ __forceinline__ int sk_first(const SplitKPlan& p, int t) {
  return sk_cta_of(static_cast<int64_t>(t) * p.kblocks, static_cast<int64_t>(p.tiles) * p.kblocks, p.grid);
}

__host__ __device__ __forceinline__ int sk_count(const SplitKPlan& p, int t) {
  const int64_t total = static_cast<int64_t>(p.tiles) * p.kblocks;
  return sk_cta_of(static_cast<int64_t>(t + 1) * p.kblocks - 1, total, p.grid) -
         sk_cta_of(static_cast<int64_t>(t) * p.kblocks, total, p.grid) + 1;
}

// Offset (floats) of element (column b, row r) of contributor j of tile t.
__host__ __device__ __forceinline__ int64_t sk_offset(const SplitKPlan& p, int t, int j, int b, int r) {
  return ((static_cast<int64_t>(t) * p.maxc + j) * p.bn + b) * kSplitBM + r;
}

// Sum, in contributor order, of the float4 at (column b, rows r..r+3) over the contributors of
// tile t.  The loads of up to 8 contributors are issued together: one L2 round trip per 8
// contributors instead of one per contributor (the order of the additions is unchanged).
__device__ __forceinline__ float4 sk_sum4(const float* partials, const SplitKPlan& p, int t, int b, int r) {
  const int nc = sk_count(p, t);
  const float* base = partials + sk_offset(p, t, 0, b, r);
  const int64_t stride = static_cast<int64_t>(p.bn) * kSplitBM;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j0 = 0; j0 < nc; j0 += 8) {
    float4 q[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j0 + j < nc) q[j] = __ldcg(reinterpret_cast<const float4*>(base + (j0 + j) * stride));
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j0 + j < nc) {
        acc.x += q[j].x;
        acc.y += q[j].y;
        acc.z += q[j].z;
        acc.w += q[j].w;
      }
  }
  return acc;
}

// sk_sum4 of two elements at once, 4 contributors of each in flight together; `second` false
// skips the second one.
__device__ __forceinline__ void sk_sum4_x2(const float* partials, const SplitKPlan& p, int t1, int b1, int r1,
                                           int t2, int b2, int r2, bool second, float4& o1, float4& o2) {
  const int n1 = sk_count(p, t1), n2 = second ? sk_count(p, t2) : 0;
  const float* base1 = partials + sk_offset(p, t1, 0, b1, r1);
  const float* base2 = partials + sk_offset(p, t2, 0, b2, r2);
  const int64_t stride = static_cast<int64_t>(p.bn) * kSplitBM;
  o1 = make_float4(0.f, 0.f, 0.f, 0.f);
  o2 = o1;
  for (int j0 = 0; j0 < n1 || j0 < n2; j0 += 4) {
    float4 q1[4], q2[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j0 + j < n1) q1[j] = __ldcg(reinterpret_cast<const float4*>(base1 + (j0 + j) * stride));
      if (j0 + j < n2) q2[j] = __ldcg(reinterpret_cast<const float4*>(base2 + (j0 + j) * stride));
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j0 + j < n1) {
        o1.x += q1[j].x;
        o1.y += q1[j].y;
        o1.z += q1[j].z;
        o1.w += q1[j].w;
      }
      if (j0 + j < n2) {
        o2.x += q2[j].x;
        o2.y += q2[j].y;
        o2.z += q2[j].z;
        o2.w += q2[j].w;
      }
    }
  }
}

// sk_sum4 of N elements at once (element i valid when i < nvalid), 4 contributors of each in
// flight together.
template <int N>
__device__ __forceinline__ void sk_sum4_n(const float* partials, const SplitKPlan& p, const int (&t)[N],
                                          const int (&b)[N], const int (&r)[N], int nvalid, float4 (&o)[N]) {
  const int64_t stride = static_cast<int64_t>(p.bn) * kSplitBM;
  int n[N];
  int nmax = 0;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    n[i] = i < nvalid ? sk_count(p, t[i]) : 0;
    nmax = n[i] > nmax ? n[i] : nmax;
    o[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int j0 = 0; j0 < nmax; j0 += 4) {
    float4 q[N][4];
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (j0 + j < n[i])
          q[i][j] = __ldcg(reinterpret_cast<const float4*>(partials + sk_offset(p, t[i], j0 + j, b[i], r[i])));
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (j0 + j < n[i]) {
          o[i].x += q[i][j].x;
          o[i].y += q[i][j].y;
          o[i].z += q[i][j].z;
          o[i].w += q[i][j].w;
        }
  }
}

inline int sk_bn_for(int64_t m) { return m <= 64 ? 64 : (m <= 128 ? 128 : 256); }

// CTAs a decode GEMM of m batch rows may use on `sms` SMs.  At BN = 64 a CTA holds 4 x 24 KB
// stages and 128 TMEM columns, so two fit on an SM; two CTAs per SM double the bytes in flight
// per SM (4 stages x 16 KB of weights at ~1.8 us load latency sustain only ~5.4 TB/s).
inline int64_t splitk_ctas(int64_t m, int sms) { return sk_bn_for(m) == 64 ? 2LL * sms : sms; }

// The plan for `tiles` output tiles of a k-deep product over `m` batch rows on at most `ctas` CTAs.
inline SplitKPlan splitk_plan_ctas(int64_t m, int tiles, int64_t k, int64_t ctas) {
  SplitKPlan p;
  p.tiles = tiles;
  p.kblocks = static_cast<int>(k / kSplitBK);
  const int64_t total = static_cast<int64_t>(p.tiles) * p.kblocks;
  p.grid = static_cast<int>(total < ctas ? total : ctas);
  p.bn = sk_bn_for(m);
  p.maxc = 1;
  for (int t = 0; t < p.tiles; ++t) {
    const int c = sk_count(p, t);
    if (c > p.maxc) p.maxc = c;
  }
  return p;
}

// The plan for `tiles` output tiles of a k-deep product over `m` batch rows on `sms` SMs.
inline SplitKPlan splitk_plan_tiles(int64_t m, int tiles, int64_t k, int sms) {
  return splitk_plan_ctas(m, tiles, k, splitk_ctas(m, sms));
}

// The plan the GEMM uses for a plain (non-SwiGLU) m x n x k product on `sms` SMs.
inline SplitKPlan splitk_plan(int64_t m, int64_t n, int64_t k, int sms) {
  return splitk_plan_tiles(m, static_cast<int>((n + kSplitBM - 1) / kSplitBM), k, sms);
}

// The plan of a SwiGLU-paired product (W = [gate; up], 2 * inter rows): tile t holds gate
// features 64t..64t+63 in rows 0-63 and the matching up features in rows 64-127.
inline SplitKPlan splitk_plan_swiglu(int64_t m, int64_t inter, int64_t k, int sms) {
  return splitk_plan_tiles(m, static_cast<int>((inter + 63) / 64), k, sms);
}

// CTAs of a row-parallel GEMM in a tensor-parallel group of `nranks` > 1.  Such a GEMM pushes
// every contributor's fp32 partial tile over NVLink to the rows' owners, so a tile is split over
// at most one CTA per 16 k-blocks: at 8 ranks (k = 512 for o_proj) the stream-K split would put
// ~9 contributors on every tile and push ~9x the bytes of the tile itself.
inline int64_t splitk_push_ctas(int64_t m, int64_t n, int64_t k, int sms, int nranks) {
  const int64_t full = splitk_ctas(m, sms);
  if (nranks <= 1) return full;
  const int64_t c = (n + kSplitBM - 1) / kSplitBM * ((k / kSplitBK + 15) / 16);
  return c < full ? c : full;
}

inline SplitKPlan splitk_plan_push(int64_t m, int64_t n, int64_t k, int sms, int nranks) {
  return splitk_plan_ctas(m, static_cast<int>((n + kSplitBM - 1) / kSplitBM), k,
                          splitk_push_ctas(m, n, k, sms, nranks));
}

inline int64_t splitk_partials_bytes(const SplitKPlan& p) {
  return static_cast<int64_t>(p.tiles) * p.maxc * p.bn * kSplitBM * 4;
}

}  // namespace mvb
