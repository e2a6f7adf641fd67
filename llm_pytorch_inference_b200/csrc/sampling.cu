// Sampling kernels: greedy argmax, top-k / top-p filtering, temperature softmax and
// one draw per row.
//
// Semantics follow the reference's sampling on a CUDA tensor (engine/sampler.py:40-48
// -> ops/sampling.py fallbacks):
//   greedy      argmax, lowest index among equal maxima        (ops/sampling.py:19-21)
//   top-k       drop x < (k-th largest value); ties at it kept  (ops/sampling.py:39-40)
//   top-p       on the untempered logits: sort descending, p = softmax, drop where
//               cumsum(p) - p >= top_p                          (ops/sampling.py:42-48)
//   temperature x / T, softmax                                  (ops/sampling.py:69-71)
// The reference's torch.sort leaves the order of equal logits unspecified; here ties
// are ordered by ascending index.  The draw is an inverse CDF over the surviving
// tokens in vocabulary order with one Philox4x32-10 uniform per row (counter
// (row, offset_lo, offset_hi, 'SAMP'), key = seed), 24-bit resolution.
//
// One 1024-thread CTA per row.  The k-th largest key is found by radix selection over
// the order-preserving integer image of the logits (2 passes for 16-bit types, 4 for
// fp32); the <= 2048 candidates are then sorted in shared memory.
#include "common.cuh"
#include "host.h"

namespace mvb {
namespace {

constexpr int kThreads = 1024;
constexpr int kCandMax = 2048;  // top_k <= 1024 plus ties at the k-th value

// Order-preserving unsigned image of a float / half / bf16 bit pattern.
template <typename T>
struct KeyOf;
template <>
struct KeyOf<float> {
  using U = uint32_t;
  static constexpr int kBits = 32;
  __device__ static U key(float v) {
    uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  }
};
template <>
struct KeyOf<__nv_bfloat16> {
  using U = uint32_t;
  static constexpr int kBits = 16;
  __device__ static U key(__nv_bfloat16 v) {
    uint32_t u = __bfloat16_as_ushort(v);
    return (u & 0x8000u) ? (~u & 0xFFFFu) : (u | 0x8000u);
  }
};
template <>
struct KeyOf<__half> {
  using U = uint32_t;
  static constexpr int kBits = 16;
  __device__ static U key(__half v) {
    uint32_t u = __half_as_ushort(v);
    return (u & 0x8000u) ? (~u & 0xFFFFu) : (u | 0x8000u);
  }
};

// Element t of a 16-byte vector of T.
template <typename T>
__device__ __forceinline__ T vec_elem(const uint4& w, int t);
template <>
__device__ __forceinline__ float vec_elem<float>(const uint4& w, int t) {
  return __uint_as_float(t == 0 ? w.x : t == 1 ? w.y : t == 2 ? w.z : w.w);
}
template <>
__device__ __forceinline__ __nv_bfloat16 vec_elem<__nv_bfloat16>(const uint4& w, int t) {
  const uint32_t u = (t >> 1) == 0 ? w.x : (t >> 1) == 1 ? w.y : (t >> 1) == 2 ? w.z : w.w;
  return __ushort_as_bfloat16(static_cast<unsigned short>((t & 1) ? (u >> 16) : (u & 0xFFFFu)));
}
template <>
__device__ __forceinline__ __half vec_elem<__half>(const uint4& w, int t) {
  const uint32_t u = (t >> 1) == 0 ? w.x : (t >> 1) == 1 ? w.y : (t >> 1) == 2 ? w.z : w.w;
  return __ushort_as_half(static_cast<unsigned short>((t & 1) ? (u >> 16) : (u & 0xFFFFu)));
}

// Visits a row of n elements: as 16-byte vectors (thread t takes vectors t, t + blockDim, ...;
// four loads in flight per thread) when the row is 16-byte aligned, then the ragged tail element
// by element.  Each thread sees its elements in ascending index order.  Every lane of a warp
// calls f(value, index, valid) the same number of times (the trip counts are uniform over the
// block), so f may use warp collectives; `valid` is false on lanes past the end.
template <typename T, typename F>
__device__ __forceinline__ void for_each_elem(const T* x, int64_t n, F&& f) {
  constexpr int V = 16 / static_cast<int>(sizeof(T));
  constexpr int U = 4;
  int64_t nv = 0;
  if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    nv = n / V;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    const int64_t trips = (nv + blockDim.x - 1) / blockDim.x;
    for (int64_t r = 0; r < trips; r += U) {
      uint4 w[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t j = (r + u) * blockDim.x + threadIdx.x;
        w[u] = j < nv ? __ldg(xv + j) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t j = (r + u) * blockDim.x + threadIdx.x;
#pragma unroll
        for (int t = 0; t < V; ++t) f(vec_elem<T>(w[u], t), j * V + t, j < nv);
      }
    }
  }
  const int64_t rest = n - nv * V;
  const int64_t trips = (rest + blockDim.x - 1) / blockDim.x;
  for (int64_t r = 0; r < trips; ++r) {
    const int64_t i = nv * V + r * blockDim.x + threadIdx.x;
    const bool ok = i < n;
    f(ok ? x[i] : x[0], i, ok);
  }
}

// ------------------------------------------------------------------ Philox4x32-10
__device__ __forceinline__ uint32_t philox_u32(uint64_t seed, uint32_t row, uint64_t offset) {
  uint32_t c0 = row, c1 = static_cast<uint32_t>(offset), c2 = static_cast<uint32_t>(offset >> 32),
           c3 = 0x53414D50u;  // 'SAMP'
  uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
  }
  return c0;
}

__device__ __forceinline__ float uniform24(uint64_t seed, uint32_t row, uint64_t offset) {
  return static_cast<float>(philox_u32(seed, row, offset) >> 8) * (1.0f / 16777216.0f);
}

// ------------------------------------------------------------------ block reductions
struct Shared {
  unsigned hist[256];
  float redf[32];
  int redi[32];
  unsigned long long cand[kCandMax];  // (key << 32) | (0xFFFFFFFF - index): larger = earlier
  float scan[kCandMax];
  int ncand;
  unsigned prefix;
  int remaining;
  int token;
};

__device__ float block_max(float v, Shared& s) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) s.redf[w] = v;
  __syncthreads();
  v = warp_max(l < (blockDim.x >> 5) ? s.redf[l] : -INFINITY);
  __syncthreads();
  return v;
}

__device__ float block_sum_f(float v, Shared& s) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) s.redf[w] = v;
  __syncthreads();
  v = warp_sum(l < (blockDim.x >> 5) ? s.redf[l] : 0.0f);
  __syncthreads();
  return v;
}

// Argmax with the lowest index among equal maxima.  Each thread sees its elements in
// ascending index order, so a strict '>' keeps its earliest maximum.
template <typename T>
__device__ int block_argmax(const T* x, int64_t n, Shared& s) {
  float best = -INFINITY;
  int bi = static_cast<int>(n);  // sentinel
  for_each_elem(x, n, [&](T e, int64_t i, bool ok) {
    const float v = to_f<T>(e);
    if (ok && (bi == n || v > best)) {
      best = v;
      bi = static_cast<int>(i);
    }
  });
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) {
      best = ob;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    s.redf[w] = best;
    s.redi[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    best = l < (blockDim.x >> 5) ? s.redf[l] : -INFINITY;
    bi = l < (blockDim.x >> 5) ? s.redi[l] : static_cast<int>(n);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    if (l == 0) s.token = bi;
  }
  __syncthreads();
  const int r = s.token;
  __syncthreads();
  return r >= n ? 0 : r;
}

// Key of the k-th largest element (1-based k) by MSB-first radix selection.
template <typename T>
__device__ uint32_t radix_kth_key(const T* x, int64_t n, int k, Shared& s) {
  constexpr int kBits = KeyOf<T>::kBits;
  if (threadIdx.x == 0) {
    s.prefix = 0;
    s.remaining = k;
  }
  __syncthreads();
  for (int shift = kBits - 8; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) s.hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s.prefix;
    const uint32_t mask_hi = shift + 8 >= 32 ? 0u : (0xFFFFFFFFu << (shift + 8));
    for_each_elem(x, n, [&](T e, int64_t, bool ok) {
      const uint32_t key = KeyOf<T>::key(e);
      if (ok && (key & mask_hi) == (prefix & mask_hi)) atomicAdd(&s.hist[(key >> shift) & 0xFFu], 1u);
    });
    __syncthreads();
    if (threadIdx.x == 0) {
      int rem = s.remaining;
      int d = 255;
      for (; d > 0; --d) {
        const int c = static_cast<int>(s.hist[d]);
        if (c >= rem) break;
        rem -= c;
      }
      s.prefix = prefix | (static_cast<uint32_t>(d) << shift);
      s.remaining = rem;
    }
    __syncthreads();
  }
  return s.prefix;
}

// Bitonic sort of s.cand[0, n2) descending (n2 a power of two <= kCandMax).
__device__ void bitonic_desc(unsigned long long* a, int n2) {
  for (int size = 2; size <= n2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < n2 / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool desc = ((lo & size) == 0);
        const unsigned long long x = a[lo], y = a[hi];
        if ((x < y) == desc) {
          a[lo] = y;
          a[hi] = x;
        }
      }
      __syncthreads();
    }
  }
}

// Inclusive block scan of s.scan[0, n) (n <= kCandMax), in place.
__device__ void block_scan_inclusive(float* v, int n, Shared& s) {
  // Each thread owns two consecutive elements.
  const int i0 = 2 * threadIdx.x, i1 = i0 + 1;
  float a0 = i0 < n ? v[i0] : 0.0f;
  float a1 = i1 < n ? v[i1] : 0.0f;
  a1 += a0;
  float t = a1;
  const int l = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float u = __shfl_up_sync(0xffffffffu, t, o);
    if (l >= o) t += u;
  }
  if (l == 31) s.redf[w] = t;
  __syncthreads();
  if (w == 0) {
    float x = s.redf[l];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float u = __shfl_up_sync(0xffffffffu, x, o);
      if (l >= o) x += u;
    }
    s.redf[l] = x;
  }
  __syncthreads();
  const float base = (w > 0 ? s.redf[w - 1] : 0.0f) + (t - a1);
  if (i0 < n) v[i0] = base + a0;
  if (i1 < n) v[i1] = base + a1;
  __syncthreads();
}

__device__ __forceinline__ float key_to_value_f32(uint32_t key) {
  const uint32_t u = (key & 0x80000000u) ? (key & 0x7FFFFFFFu) : ~key;
  return __uint_as_float(u);
}
template <typename T>
__device__ __forceinline__ float key_value(uint32_t key);
template <>
__device__ __forceinline__ float key_value<float>(uint32_t key) { return key_to_value_f32(key); }
template <>
__device__ __forceinline__ float key_value<__nv_bfloat16>(uint32_t key) {
  const uint32_t u = (key & 0x8000u) ? (key & 0x7FFFu) : (~key & 0xFFFFu);
  return __bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(u)));
}
template <>
__device__ __forceinline__ float key_value<__half>(uint32_t key) {
  const uint32_t u = (key & 0x8000u) ? (key & 0x7FFFu) : (~key & 0xFFFFu);
  return __half2float(__ushort_as_half(static_cast<unsigned short>(u)));
}

// Gathers {i : key(x_i) >= kth} into s.cand and sorts them (value desc, index asc).
// Returns the candidate count (clipped to kCandMax; excess reported).
template <typename T>
__device__ int gather_sorted_candidates(const T* x, int64_t n, uint32_t kth, Shared& s, unsigned* err) {
  if (threadIdx.x == 0) s.ncand = 0;
  __syncthreads();
  for_each_elem(x, n, [&](T e, int64_t i, bool ok) {
    const uint32_t key = KeyOf<T>::key(e);
    if (ok && key >= kth) {
      const int slot = atomicAdd(&s.ncand, 1);
      if (slot < kCandMax)
        s.cand[slot] = (static_cast<unsigned long long>(key) << 32) | (0xFFFFFFFFull - static_cast<uint32_t>(i));
    }
  });
  __syncthreads();
  int nc = s.ncand;
  if (nc > kCandMax) {
    if (threadIdx.x == 0) report(err, kDevSamplerTies);
    nc = kCandMax;
  }
  int n2 = 1;
  while (n2 < nc) n2 <<= 1;
  for (int i = nc + threadIdx.x; i < n2; i += blockDim.x) s.cand[i] = 0ull;
  __syncthreads();
  bitonic_desc(s.cand, n2);
  return nc;
}

__device__ __forceinline__ int cand_index(unsigned long long c) {
  return static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(c & 0xFFFFFFFFull));
}

// Number of sorted candidates that survive top-p (computed on the untempered values).
template <typename T>
__device__ int top_p_keep(int nc, float top_p, Shared& s) {
  if (!(top_p < 1.0f)) return nc;
  const float xmax = key_value<T>(static_cast<uint32_t>(s.cand[0] >> 32));
  float e_local = 0.0f;
  for (int i = threadIdx.x; i < nc; i += blockDim.x) {
    const float e = expf(key_value<T>(static_cast<uint32_t>(s.cand[i] >> 32)) - xmax);
    s.scan[i] = e;
    e_local += e;
  }
  __syncthreads();
  const float z = block_sum_f(e_local, s);
  for (int i = threadIdx.x; i < nc; i += blockDim.x) s.scan[i] = s.scan[i] / z;
  __syncthreads();
  // keep i while cumsum(p)_i - p_i < top_p; removal is monotone in i.
  float p_own[2];
  for (int j = 0; j < 2; ++j) {
    const int i = 2 * threadIdx.x + j;
    p_own[j] = i < nc ? s.scan[i] : 0.0f;
  }
  __syncthreads();
  block_scan_inclusive(s.scan, nc, s);
  int keep_local = 0;
  for (int j = 0; j < 2; ++j) {
    const int i = 2 * threadIdx.x + j;
    if (i < nc && !((s.scan[i] - p_own[j]) >= top_p)) keep_local = i + 1;
  }
  // max over threads of the last kept position
  int v = keep_local;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) s.redi[w] = v;
  __syncthreads();
  if (w == 0) {
    v = l < (blockDim.x >> 5) ? s.redi[l] : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (l == 0) s.token = v < 1 ? 1 : v;
  }
  __syncthreads();
  const int keep = s.token;
  __syncthreads();
  return keep;
}


// Full-vocabulary nucleus (top-p without top-k).  Survivors are the tokens whose
// probability mass strictly before them in (value desc, index asc) order is below
// top_p.  Found exactly by radix selection on mass: the cutoff key `tau`, the mass of
// all keys above it, and how many of the tokens tied at `tau` (in index order) survive.
struct Nucleus {
  uint32_t tau;
  int kept_ties;
  float xmax;
};

template <typename T>
__device__ Nucleus nucleus_threshold(const T* x, int64_t n, float top_p, Shared& s) {
  // Masses accumulate in fp64: at 152k tokens a boundary token carries ~1e-5 of the mass,
  // below what fp32 sums of the whole row resolve.
  constexpr int kBits = KeyOf<T>::kBits;
  float m = -INFINITY;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, to_f<T>(x[i]));
  m = block_max(m, s);
  double zl = 0.0;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) zl += static_cast<double>(expf(to_f<T>(x[i]) - m));
  double* red = reinterpret_cast<double*>(s.scan);       // [0, 32): reduction, [32, 288): bins
  double* hmass = red + 32;
  {
    zl += __shfl_xor_sync(0xffffffffu, zl, 16);
    zl += __shfl_xor_sync(0xffffffffu, zl, 8);
    zl += __shfl_xor_sync(0xffffffffu, zl, 4);
    zl += __shfl_xor_sync(0xffffffffu, zl, 2);
    zl += __shfl_xor_sync(0xffffffffu, zl, 1);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = zl;
    __syncthreads();
    if (threadIdx.x == 0) {
      double z = 0.0;
      for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) z += red[w];
      red[0] = z;
    }
    __syncthreads();
  }
  const double target = static_cast<double>(top_p) * red[0];
  __syncthreads();
  if (threadIdx.x == 0) {
    s.prefix = 0;
    red[1] = 0.0;  // mass above the current prefix range
  }
  __syncthreads();
  double mass_above = 0.0;
  unsigned ties = 0;
  for (int shift = kBits - 8; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
      s.hist[i] = 0;
      hmass[i] = 0.0;
    }
    __syncthreads();
    const uint32_t prefix = s.prefix;
    const uint32_t mask_hi = shift + 8 >= 32 ? 0u : (0xFFFFFFFFu << (shift + 8));
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
      const T v = x[i];
      const uint32_t key = KeyOf<T>::key(v);
      if ((key & mask_hi) == (prefix & mask_hi)) {
        const int d = (key >> shift) & 0xFF;
        atomicAdd(&s.hist[d], 1u);
        atomicAdd(&hmass[d], static_cast<double>(expf(to_f<T>(v) - m)));
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      double above = red[1];
      int d = 255, last_nonempty = -1;
      for (; d >= 0; --d) {
        if (s.hist[d] == 0) continue;
        last_nonempty = d;
        if (above + hmass[d] >= target) break;
        above += hmass[d];
      }
      if (d < 0) {  // mass never reached top_p (rounding): keep everything down to the smallest key
        d = last_nonempty;
        above -= hmass[d];
      }
      s.prefix = prefix | (static_cast<uint32_t>(d) << shift);
      red[1] = above;
      s.ncand = static_cast<int>(s.hist[d]);
    }
    __syncthreads();
    mass_above = red[1];
    ties = static_cast<unsigned>(s.ncand);
    __syncthreads();
  }
  Nucleus r;
  r.tau = s.prefix;
  r.xmax = m;
  const double e_tau = static_cast<double>(expf(key_value<T>(r.tau) - m));
  int kept = 0;
  if (target > mass_above && e_tau > 0.0) {
    const double q = ceil((target - mass_above) / e_tau);
    kept = q >= static_cast<double>(ties) ? static_cast<int>(ties) : static_cast<int>(q);
  }
  if (kept < 1 && mass_above == 0.0) kept = 1;  // the top token always survives
  r.kept_ties = kept;
  return r;
}

// Exclusive prefix (over threads, in thread order) of a per-thread count.
__device__ int block_excl_count(int c, Shared& s) {
  s.scan[threadIdx.x] = static_cast<float>(c);
  __syncthreads();
  block_scan_inclusive(s.scan, blockDim.x, s);
  const int r = static_cast<int>(s.scan[threadIdx.x]) - c;
  __syncthreads();
  return r;
}

// ---------------------------------------------------------------------- kernels
template <typename T>
__global__ void __launch_bounds__(kThreads) greedy_kernel(int64_t* out, const T* logits, int64_t vocab,
                                                          int64_t row_stride) {
  __shared__ Shared s;
  pdl_launch_dependents();
  pdl_wait();
  const T* x = logits + blockIdx.x * row_stride;
  const int r = block_argmax(x, vocab, s);
  if (threadIdx.x == 0) out[blockIdx.x] = r;
}

// In-place top-k / top-p filter (ops API): non-survivors become -inf.
template <typename T>
__global__ void __launch_bounds__(kThreads) filter_kernel(T* logits, int64_t vocab, int top_k, float top_p,
                                                          unsigned* err) {
  __shared__ Shared s;
  pdl_launch_dependents();
  pdl_wait();
  T* x = logits + blockIdx.x * vocab;
  const int k = (top_k > 0 && top_k < vocab) ? top_k : static_cast<int>(vocab < kCandMax ? vocab : 0);
  if (k == 0) {
    // Full-vocabulary nucleus: survivors are keys above tau plus the first kept_ties
    // tokens (index order) at tau.  Threads own contiguous chunks for the tie ranks.
    const Nucleus nu = nucleus_threshold(x, vocab, top_p, s);
    const int64_t chunk = (vocab + blockDim.x - 1) / blockDim.x;
    const int64_t lo = threadIdx.x * chunk, hi = min(vocab, lo + chunk);
    int ties = 0;
    for (int64_t i = lo; i < hi; ++i) ties += KeyOf<T>::key(x[i]) == nu.tau;
    int rank = block_excl_count(ties, s);
    for (int64_t i = lo; i < hi; ++i) {
      const uint32_t key = KeyOf<T>::key(x[i]);
      bool keep = key > nu.tau;
      if (key == nu.tau) keep = rank++ < nu.kept_ties;
      if (!keep) x[i] = from_f<T>(-INFINITY);
    }
    return;
  }
  const uint32_t kth = radix_kth_key(x, vocab, k, s);
  const int nc = gather_sorted_candidates(x, vocab, kth, s, err);
  const int keep = top_p_keep<T>(nc, top_p, s);
  // Survivors: the first `keep` sorted candidates.  Mark them in the hist-sized bitmap
  // would not scale to the vocabulary, so compare against the boundary candidate
  // (value, index) order instead: element i survives iff (key, -i) >= boundary.
  const unsigned long long boundary = s.cand[keep - 1];
  __syncthreads();
  for (int64_t i = threadIdx.x; i < vocab; i += blockDim.x) {
    const unsigned long long c =
        (static_cast<unsigned long long>(KeyOf<T>::key(x[i])) << 32) | (0xFFFFFFFFull - static_cast<uint32_t>(i));
    if (c < boundary) x[i] = from_f<T>(-INFINITY);
  }
}

struct SampleParams {
  const float* temperature;
  const int32_t* top_k;
  const float* top_p;
  float t_default;
  int k_default;
  float p_default;
  uint64_t seed;
  uint64_t offset;
  const int64_t* offset_dev;
};

// Full sampler: greedy when T == 0, else filter -> tempered softmax -> Philox draw.
template <typename T>
__global__ void __launch_bounds__(kThreads) sample_kernel(int64_t* out, float* probs_out, const T* logits,
                                                          int64_t vocab, int64_t row_stride, SampleParams p,
                                                          unsigned* err) {
  __shared__ Shared s;
  pdl_launch_dependents();
  pdl_wait();
  const int row = blockIdx.x;
  const T* x = logits + row * row_stride;
  const float temp = p.temperature ? p.temperature[row] : p.t_default;
  const int top_k = p.top_k ? p.top_k[row] : p.k_default;
  const float top_p = p.top_p ? p.top_p[row] : p.p_default;
  float* po = probs_out ? probs_out + row * vocab : nullptr;

  if (!(temp > 0.0f)) {  // greedy (sampler.py:33-38)
    const int r = block_argmax(x, vocab, s);
    if (threadIdx.x == 0) out[row] = r;
    if (po) {
      for (int64_t i = threadIdx.x; i < vocab; i += blockDim.x) po[i] = (i == r) ? 1.0f : 0.0f;
    }
    return;
  }
  const uint64_t offset = p.offset + (p.offset_dev ? static_cast<uint64_t>(*p.offset_dev) : 0ull);
  const float u = uniform24(p.seed, static_cast<uint32_t>(row), offset);
  const bool use_k = top_k > 0 && top_k < vocab;
  if (!use_k && !(top_p < 1.0f)) {
    // No filter: tempered softmax over the whole vocabulary, inverse CDF in index order.
    float m = -INFINITY;
    for (int64_t i = threadIdx.x; i < vocab; i += blockDim.x) m = fmaxf(m, to_f<T>(x[i]) / temp);
    m = block_max(m, s);
    const int64_t chunk = (vocab + blockDim.x - 1) / blockDim.x;
    const int64_t lo = threadIdx.x * chunk, hi = min(vocab, lo + chunk);
    float part = 0.0f;
    for (int64_t i = lo; i < hi; ++i) part += expf(to_f<T>(x[i]) / temp - m);
    // exclusive scan of per-thread partial sums
    s.scan[threadIdx.x] = part;
    __syncthreads();
    block_scan_inclusive(s.scan, blockDim.x, s);
    const float total = s.scan[blockDim.x - 1];
    const float excl = s.scan[threadIdx.x] - part;
    const float target = u * total;
    // The chunk holding the target: the last non-empty chunk starting at or below it.
    if (threadIdx.x == 0) s.remaining = -1;
    __syncthreads();
    if (part > 0.0f && excl <= target) atomicMax(&s.remaining, static_cast<int>(threadIdx.x));
    __syncthreads();
    if (static_cast<int>(threadIdx.x) == s.remaining) {
      float run = excl;
      int64_t pick = -1;
      for (int64_t i = lo; i < hi; ++i) {
        const float e = expf(to_f<T>(x[i]) / temp - m);
        run += e;
        if (e > 0.0f) pick = i;
        if (run > target) break;
      }
      out[row] = pick;
    }
    if (po) {
      const float inv = 1.0f / total;
      for (int64_t i = threadIdx.x; i < vocab; i += blockDim.x) po[i] = expf(to_f<T>(x[i]) / temp - m) * inv;
    }
    return;
  }
  const int k = use_k ? top_k : (vocab < kCandMax ? static_cast<int>(vocab) : 0);
  if (k == 0) {
    // Full-vocabulary nucleus, then a tempered inverse-CDF draw over the survivors in
    // index order (threads own contiguous chunks).
    const Nucleus nu = nucleus_threshold(x, vocab, top_p, s);
    const int64_t chunk = (vocab + blockDim.x - 1) / blockDim.x;
    const int64_t lo = threadIdx.x * chunk, hi = min(vocab, lo + chunk);
    int ties = 0;
    for (int64_t i = lo; i < hi; ++i) ties += KeyOf<T>::key(x[i]) == nu.tau;
    const int rank0 = block_excl_count(ties, s);
    const float ymax = nu.xmax / temp;
    float part = 0.0f;
    {
      int rank = rank0;
      for (int64_t i = lo; i < hi; ++i) {
        const uint32_t key = KeyOf<T>::key(x[i]);
        bool keep = key > nu.tau;
        if (key == nu.tau) keep = rank++ < nu.kept_ties;
        if (keep) part += expf(to_f<T>(x[i]) / temp - ymax);
      }
    }
    s.scan[threadIdx.x] = part;
    __syncthreads();
    block_scan_inclusive(s.scan, blockDim.x, s);
    const float total = s.scan[blockDim.x - 1];
    const float excl = s.scan[threadIdx.x] - part;
    const float target = u * total;
    if (threadIdx.x == 0) s.remaining = -1;
    __syncthreads();
    if (part > 0.0f && excl <= target) atomicMax(&s.remaining, static_cast<int>(threadIdx.x));
    __syncthreads();
    const bool owner = static_cast<int>(threadIdx.x) == s.remaining;
    int rank = rank0;
    float run = excl;
    int64_t pick = -1;
    bool done = false;
    const float inv = 1.0f / total;
    for (int64_t i = lo; i < hi; ++i) {
      const uint32_t key = KeyOf<T>::key(x[i]);
      bool keep = key > nu.tau;
      if (key == nu.tau) keep = rank++ < nu.kept_ties;
      const float e = keep ? expf(to_f<T>(x[i]) / temp - ymax) : 0.0f;
      if (po) po[i] = e * inv;
      if (owner && !done && keep) {
        run += e;
        pick = i;
        if (run > target) done = true;
      }
    }
    if (owner) out[row] = pick;
    return;
  }
  const uint32_t kth = radix_kth_key(x, vocab, k, s);
  const int nc = gather_sorted_candidates(x, vocab, kth, s, err);
  const int keep = top_p_keep<T>(nc, top_p, s);
  // Re-sort the survivors by index ascending for the vocabulary-order draw.
  int n2 = 1;
  while (n2 < keep) n2 <<= 1;
  for (int i = threadIdx.x; i < n2; i += blockDim.x) {
    if (i < keep) {
      const unsigned long long c = s.cand[i];
      const uint32_t key = static_cast<uint32_t>(c >> 32);
      // sort key: larger = smaller index; payload keeps the value key
      s.cand[i] = (static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(cand_index(c))) << 32) | key;
    } else {
      s.cand[i] = 0ull;
    }
  }
  __syncthreads();
  bitonic_desc(s.cand, n2);
  // Tempered weights: y = x / T, e = exp(y - max y) (max y is the largest survivor).
  float ymax = -INFINITY;
  for (int i = threadIdx.x; i < keep; i += blockDim.x)
    ymax = fmaxf(ymax, key_value<T>(static_cast<uint32_t>(s.cand[i] & 0xFFFFFFFFull)) / temp);
  ymax = block_max(ymax, s);
  for (int i = threadIdx.x; i < keep; i += blockDim.x)
    s.scan[i] = expf(key_value<T>(static_cast<uint32_t>(s.cand[i] & 0xFFFFFFFFull)) / temp - ymax);
  __syncthreads();
  float w_own[2];
  for (int j = 0; j < 2; ++j) {
    const int i = 2 * threadIdx.x + j;
    w_own[j] = i < keep ? s.scan[i] : 0.0f;
  }
  __syncthreads();
  block_scan_inclusive(s.scan, keep, s);
  const float total = s.scan[keep - 1];
  const float target = u * total;
  if (threadIdx.x == 0) s.token = keep - 1;
  __syncthreads();
  for (int j = 0; j < 2; ++j) {
    const int i = 2 * threadIdx.x + j;
    if (i < keep && s.scan[i] > target) atomicMin(&s.token, i);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned long long c = s.cand[s.token];
    out[row] = static_cast<int64_t>(0xFFFFFFFFu - static_cast<uint32_t>(c >> 32));
  }
  if (po) {
    for (int64_t i = threadIdx.x; i < vocab; i += blockDim.x) po[i] = 0.0f;
    __syncthreads();
    const float inv = 1.0f / total;
    for (int j = 0; j < 2; ++j) {
      const int i = 2 * threadIdx.x + j;
      if (i < keep) {
        const int idx = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(s.cand[i] >> 32));
        po[idx] = w_own[j] * inv;
      }
    }
  }
}

}  // namespace
}  // namespace mvb

using namespace mvb;

#define MVB_DISPATCH_SAMPLING(dtype, NAME, ...)                                         \
  switch (dtype) {                                                                      \
    case MVB_F32: { using T = float; __VA_ARGS__; }                                     \
    case MVB_F16: { using T = __half; __VA_ARGS__; }                                    \
    case MVB_BF16: { using T = __nv_bfloat16; __VA_ARGS__; }                            \
    default: return fail(MVB_ERR_INVALID_ARG, NAME ": unsupported dtype %d", dtype);  \
  }

extern "C" int mvb_greedy_sample(int64_t* out, const void* logits, int64_t rows, int64_t vocab, int64_t row_stride,
                                 int dtype, mvb_stream_t stream) {
  MVB_REQUIRE(out && logits && rows >= 0 && vocab > 0 && vocab < (1LL << 31) && row_stride >= vocab,
              "mvb_greedy_sample: bad arguments");
  if (rows == 0) return MVB_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MVB_DISPATCH_SAMPLING(dtype, "mvb_greedy_sample",
                        return launch("greedy_sample", greedy_kernel<T>, dim3(static_cast<unsigned>(rows)),
                                      dim3(kThreads), 0, st, out, (const T*)logits, vocab, row_stride));
}

extern "C" int mvb_top_k_top_p_filter(void* logits, int64_t rows, int64_t vocab, int top_k, float top_p, int dtype,
                                      mvb_stream_t stream) {
  MVB_REQUIRE(logits && rows >= 0 && vocab > 0 && vocab < (1LL << 31), "mvb_top_k_top_p_filter: bad arguments");
  MVB_REQUIRE(top_k <= 1024, "mvb_top_k_top_p_filter: top_k %d > 1024 is not supported", top_k);
  const bool use_k = top_k > 0 && top_k < vocab;
  if (!use_k && !(top_p < 1.0f)) return MVB_OK;  // nothing to filter
  if (rows == 0) return MVB_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned* err = device_status_ptr();
  MVB_DISPATCH_SAMPLING(dtype, "mvb_top_k_top_p_filter",
                        return launch("top_k_top_p_filter", filter_kernel<T>, dim3(static_cast<unsigned>(rows)),
                                      dim3(kThreads), 0, st, (T*)logits, vocab, top_k, top_p, err));
}

extern "C" int mvb_sample(int64_t* out, float* probs_out, const void* logits, int64_t rows, int64_t vocab,
                          int64_t row_stride, const float* temperature, const int32_t* top_k, const float* top_p,
                          uint64_t seed, uint64_t offset, const int64_t* offset_dev, int dtype,
                          mvb_stream_t stream) {
  MVB_REQUIRE(out && logits && rows >= 0 && vocab > 0 && vocab < (1LL << 31) && row_stride >= vocab,
              "mvb_sample: bad arguments");
  if (rows == 0) return MVB_OK;
  SampleParams p;
  p.temperature = temperature;
  p.top_k = top_k;
  p.top_p = top_p;
  p.t_default = 1.0f;
  p.k_default = -1;
  p.p_default = 1.0f;
  p.seed = seed;
  p.offset = offset;
  p.offset_dev = offset_dev;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned* err = device_status_ptr();
  MVB_DISPATCH_SAMPLING(dtype, "mvb_sample",
                        return launch("sample", sample_kernel<T>, dim3(static_cast<unsigned>(rows)), dim3(kThreads),
                                      0, st, out, probs_out, (const T*)logits, vocab, row_stride, p, err));
}

extern "C" int mvb_softmax_multinomial_sample(int64_t* out, const void* logits, int64_t rows, int64_t vocab,
                                              float temperature, uint64_t seed, uint64_t offset, int dtype,
                                              mvb_stream_t stream) {
  MVB_REQUIRE(out && logits && rows >= 0 && vocab > 0 && vocab < (1LL << 31),
              "mvb_softmax_multinomial_sample: bad arguments");
  if (rows == 0) return MVB_OK;
  SampleParams p;
  p.temperature = nullptr;
  p.top_k = nullptr;
  p.top_p = nullptr;
  // ops/sampling.py:69-70 divides only when T > 0 and T != 1; T <= 0 samples at T = 1.
  p.t_default = temperature > 0.0f ? temperature : 1.0f;
  p.k_default = -1;
  p.p_default = 1.0f;
  p.seed = seed;
  p.offset = offset;
  p.offset_dev = nullptr;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned* err = device_status_ptr();
  MVB_DISPATCH_SAMPLING(dtype, "mvb_softmax_multinomial_sample",
                        return launch("softmax_multinomial_sample", sample_kernel<T>,
                                      dim3(static_cast<unsigned>(rows)), dim3(kThreads), 0, st, out,
                                      (float*)nullptr, (const T*)logits, vocab, vocab, p, err));
}
