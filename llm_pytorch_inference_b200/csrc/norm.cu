// RMSNorm family: rmsnorm, rmsnorm_plus_one, fused residual-add + RMSNorm.
//
// One CTA per row; fp32 sum of squares reduced across the whole CTA and broadcast
// to every warp (the reference's block_reduce_sum leaves the result in warp 0
// only, csrc/include/mini_vllm/utils.cuh:27-30).  The rounding sequence of each
// variant reproduces the PyTorch expression it replaces:
//   ops      (ops/rmsnorm.py:12-20)  y = T( T(w*x) * r )
//   ops +1   (ops/rmsnorm.py:23-31)  y = T( (1+w) * (x*r) )
//   ops +1 fused (ops/rmsnorm.py:51) y = T( ((1+w)*x) * r )
//   model    (models/model.py:19-25) y = T( w * (x*r) )       model +1: T( (x*r) * (1+w) )
// with r = 1/sqrt(mean(x^2) + eps) in fp32 and T() rounding to the storage type.
#include "common.cuh"
#include "host.h"
#include "splitk.cuh"
#include "tp.cuh"

namespace mvb {
namespace {

template <typename T>
__device__ __forceinline__ float norm_out(float x, float w, float r, int plus_one, int semantics, bool fused) {
  if (semantics == MVB_NORM_OPS) {
    if (!plus_one) return rnd<T>(rnd<T>(w * x) * r);
    if (fused) return rnd<T>(((1.0f + w) * x) * r);
    return rnd<T>((1.0f + w) * (x * r));
  }
  if (!plus_one) return rnd<T>(w * (x * r));
  return rnd<T>((x * r) * (1.0f + w));
}

// CTA-wide sum broadcast to all threads.
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = (blockDim.x + 31) >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.0f;
  t = warp_sum(t);
  __syncthreads();
  return t;
}

template <typename T>
__global__ void rmsnorm_kernel(T* __restrict__ out, int64_t out_stride, const T* __restrict__ in, int64_t in_stride,
                               const T* __restrict__ w, int hidden, float eps, int plus_one, int semantics) {
  __shared__ float red[32];
  pdl_launch_dependents();
  pdl_wait();
  const T* x = in + blockIdx.x * in_stride;
  T* y = out + blockIdx.x * out_stride;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    float v = to_f<T>(x[i]);
    ss += v * v;
  }
  ss = block_sum(ss, red);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(hidden) + eps);
  for (int i = threadIdx.x; i < hidden; i += blockDim.x)
    y[i] = from_f<T>(norm_out<T>(to_f<T>(x[i]), to_f<T>(w[i]), r, plus_one, semantics, false));
}

template <typename T>
__global__ void fused_add_rmsnorm_kernel(T* __restrict__ out, T* __restrict__ residual, const T* __restrict__ in,
                                         const T* __restrict__ w, int hidden, float eps, int plus_one,
                                         int semantics) {
  __shared__ float red[32];
  pdl_launch_dependents();
  pdl_wait();
  T* res = residual + static_cast<int64_t>(blockIdx.x) * hidden;
  const T* x = in + static_cast<int64_t>(blockIdx.x) * hidden;
  T* y = out + static_cast<int64_t>(blockIdx.x) * hidden;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    float v = rnd<T>(to_f<T>(res[i]) + to_f<T>(x[i]));
    res[i] = from_f<T>(v);
    ss += v * v;
  }
  ss = block_sum(ss, red);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(hidden) + eps);
  for (int i = threadIdx.x; i < hidden; i += blockDim.x)
    y[i] = from_f<T>(norm_out<T>(to_f<T>(res[i]), to_f<T>(w[i]), r, plus_one, semantics, true));
}

// Many rows (a prefill's tokens, more than 256), bf16: one warp per row, 8 rows per 256-thread CTA.
// The row stays in registers as 16-byte vectors of 8 values (vector j * 32 + lane) between the
// sum-of-squares pass and the output pass, so it is read from HBM once, with 512-byte warp accesses.
// One CTA per row (the kernels above) keeps too few bytes in flight for HBM at this row count.  The
// per-element rounding is the kernels' above; only the order of the fp32 sum of squares differs.
// ADD: residual += in (rounded to bf16, written back), then the norm of the sum.  `out` may be `in`.
template <int MAXV, bool ADD>
__global__ void __launch_bounds__(256) norm_rows_kernel(__nv_bfloat16* out, int64_t out_stride,
                                                        __nv_bfloat16* residual, const __nv_bfloat16* in,
                                                        int64_t in_stride, const __nv_bfloat16* __restrict__ w,
                                                        int64_t rows, int hidden, float eps, int plus_one,
                                                        int semantics) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nv = hidden >> 8;  // vectors per lane
  const uint4* x = reinterpret_cast<const uint4*>(in + row * in_stride);
  uint4* res = ADD ? reinterpret_cast<uint4*>(residual + row * hidden) : nullptr;
  uint4 v[MAXV];
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < MAXV; ++j) {
    if (j < nv) {
      uint4 a = x[j * 32 + lane];
      __nv_bfloat162* pa = reinterpret_cast<__nv_bfloat162*>(&a);
      if (ADD) {
        const uint4 b = res[j * 32 + lane];
        const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 fa = __bfloat1622float2(pa[k]), fb = __bfloat1622float2(pb[k]);
          pa[k] = __floats2bfloat162_rn(fb.x + fa.x, fb.y + fa.y);
        }
        res[j * 32 + lane] = a;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(pa[k]);
        ss += f.x * f.x;
        ss += f.y * f.y;
      }
      v[j] = a;
    }
  }
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(hidden) + eps);
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  uint4* y = reinterpret_cast<uint4*>(out + row * out_stride);
#pragma unroll
  for (int j = 0; j < MAXV; ++j) {
    if (j < nv) {
      const uint4 wq = wv[j * 32 + lane];
      const __nv_bfloat162* pw = reinterpret_cast<const __nv_bfloat162*>(&wq);
      __nv_bfloat162* px = reinterpret_cast<__nv_bfloat162*>(&v[j]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 fx = __bfloat1622float2(px[k]), fw = __bfloat1622float2(pw[k]);
        px[k] = __floats2bfloat162_rn(norm_out<__nv_bfloat16>(fx.x, fw.x, r, plus_one, semantics, ADD),
                                      norm_out<__nv_bfloat16>(fx.y, fw.y, r, plus_one, semantics, ADD));
      }
      y[j * 32 + lane] = v[j];
    }
  }
}

// Residual add + RMSNorm whose input is a GEMM's output still in split-K partial form: the
// linear layer's bf16 output is formed here as bf16(sum of the tile's partial slots, contributor
// order), then residual += it and out = RMSNorm(residual) (model semantics, models/model.py:19-25,
// :319).
//
// Row b (blockIdx.y) is split over a cluster of gridDim.x CTAs: CTA c owns the runs of 4
// consecutive features [c * runs_per_cta, (c + 1) * runs_per_cta), each thread up to
// kFaddMaxRuns of them, kept in registers between the two passes (float4 partial loads,
// 8-byte residual accesses).  Each CTA reduces its share of the sum of squares, publishes it
// in shared memory, and every CTA of the cluster sums the published shares in CTA order
// through distributed shared memory, so all chunks of a row scale by the same 1/rms.
//
// Tensor-parallel form (TP = true): the partials were pushed by every rank's row-parallel GEMM
// into this rank's receive area (layout sk_push_offset) for the rows this rank owns
// (blockIdx.y indexes them); the sum runs over source ranks, then contributors.  The
// normalised row is written into every rank's copy of the activations (all-gather), and each
// CTA then signals every rank.  The residual stream of a row lives on its owner only.
constexpr int kFaddMaxRuns = 4;
constexpr int kFaddMaxCluster = 8;

struct TpFadd {
  int nranks, rank, rows_per_rank;
  const float* recv;                       // this rank's receive area
  __nv_bfloat16* out[kTpMaxRanks];         // every rank's copy of the normalised activations
  uint32_t* signal[kTpMaxRanks];           // every rank's counter [point][this rank]
  uint32_t* arrive;                        // this rank's arrival counter of the signal point
  const uint32_t* wait;                    // this rank's counters of the GEMM's push point
  uint32_t wait_count;
  const int32_t* epoch;
};

// Sum over the cluster's CTAs (in CTA order) of each CTA's share `ss` of a row's sum of squares.
__device__ __forceinline__ float cluster_row_sum(float ss, float* red, float* cta_ss) {
  ss = block_sum(ss, red);
  if (threadIdx.x == 0) *cta_ss = ss;
  cluster_sync();
  float total = 0.0f;
  for (unsigned c = 0; c < gridDim.x; ++c) total += dsmem_ld_f32(cta_ss, c);
  cluster_sync();  // no CTA leaves (or rewrites its share) while another may still read it
  return total;
}

// POST (Gemma's sandwich norms, models/gemma3_model.py:270-283): the linear layer's output is
// itself normalised with the post weight `pw` before the residual add,
//   residual += T((y * r_y) * (1 + pw)),  out = T((residual * r) * (1 + w))   (plus_one form),
// which takes a second cluster-wide sum of squares (over y) first.
template <bool TP, bool POST>
__global__ void fused_add_rmsnorm_gemm_kernel(__nv_bfloat16* __restrict__ out, __nv_bfloat16* __restrict__ residual,
                                              const float* __restrict__ partials, SplitKPlan p,
                                              const __nv_bfloat16* __restrict__ w,
                                              const __nv_bfloat16* __restrict__ pw, int hidden, int runs_per_cta,
                                              float eps, int plus_one, const __grid_constant__ TpFadd tp,
                                              unsigned* err) {
  __shared__ float red[32];
  __shared__ float cta_ss;
  pdl_launch_dependents();
  pdl_wait();
  if (TP) {
    if (threadIdx.x == 0)
      wait_counters(tp.wait, tp.nranks, static_cast<uint32_t>(*tp.epoch) * tp.wait_count, err);
    __syncthreads();
  }
  const int bl = blockIdx.y;
  const int b = TP ? tp.rank * tp.rows_per_rank + bl : bl;
  const int run0 = blockIdx.x * runs_per_cta;
  const int run_end = min(run0 + runs_per_cta, hidden / 4);
  __nv_bfloat16* res = residual + static_cast<int64_t>(b) * hidden;
  float v[kFaddMaxRuns][4];
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < kFaddMaxRuns; ++k) {
    const int run = run0 + threadIdx.x + k * blockDim.x;
    if (run < run_end) {
      const int i = run * 4;
      const int t = i / kSplitBM, r = i - t * kSplitBM;
      const int nc = sk_count(p, t);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      const int nsrc = TP ? tp.nranks : 1;
      for (int src = 0; src < nsrc; ++src) {
        for (int j = 0; j < nc; ++j) {
          const float* q = TP ? tp.recv + sk_push_offset(p, src, t, j, tp.rows_per_rank, bl, r)
                              : partials + sk_offset(p, t, j, b, r);
          const float4 qv = __ldcg(reinterpret_cast<const float4*>(q));
          acc.x += qv.x;
          acc.y += qv.y;
          acc.z += qv.z;
          acc.w += qv.w;
        }
      }
      v[k][0] = bf16_round(acc.x);  // the linear layer's bf16 output
      v[k][1] = bf16_round(acc.y);
      v[k][2] = bf16_round(acc.z);
      v[k][3] = bf16_round(acc.w);
      if constexpr (POST) {
        ss += v[k][0] * v[k][0] + v[k][1] * v[k][1] + v[k][2] * v[k][2] + v[k][3] * v[k][3];
      } else {
        const uint2 rr = *reinterpret_cast<const uint2*>(res + i);
        const __nv_bfloat162 r01 = *reinterpret_cast<const __nv_bfloat162*>(&rr.x);
        const __nv_bfloat162 r23 = *reinterpret_cast<const __nv_bfloat162*>(&rr.y);
        v[k][0] = bf16_round(__low2float(r01) + v[k][0]);
        v[k][1] = bf16_round(__high2float(r01) + v[k][1]);
        v[k][2] = bf16_round(__low2float(r23) + v[k][2]);
        v[k][3] = bf16_round(__high2float(r23) + v[k][3]);
        __nv_bfloat162 o01 = __floats2bfloat162_rn(v[k][0], v[k][1]);
        __nv_bfloat162 o23 = __floats2bfloat162_rn(v[k][2], v[k][3]);
        uint2 ov;
        ov.x = *reinterpret_cast<uint32_t*>(&o01);
        ov.y = *reinterpret_cast<uint32_t*>(&o23);
        *reinterpret_cast<uint2*>(res + i) = ov;
        ss += v[k][0] * v[k][0] + v[k][1] * v[k][1] + v[k][2] * v[k][2] + v[k][3] * v[k][3];
      }
    }
  }
  if constexpr (POST) {
    // y -> post-norm(y) -> residual add; the sum of squares of the new residual follows.
    const float ry = 1.0f / sqrtf(cluster_row_sum(ss, red, &cta_ss) / static_cast<float>(hidden) + eps);
    ss = 0.0f;
#pragma unroll
    for (int k = 0; k < kFaddMaxRuns; ++k) {
      const int run = run0 + threadIdx.x + k * blockDim.x;
      if (run < run_end) {
        const int i = run * 4;
        const uint2 wr = *reinterpret_cast<const uint2*>(pw + i);
        const __nv_bfloat162 w01 = *reinterpret_cast<const __nv_bfloat162*>(&wr.x);
        const __nv_bfloat162 w23 = *reinterpret_cast<const __nv_bfloat162*>(&wr.y);
        const float wf[4] = {__low2float(w01), __high2float(w01), __low2float(w23), __high2float(w23)};
        const uint2 rr = *reinterpret_cast<const uint2*>(res + i);
        const __nv_bfloat162 r01 = *reinterpret_cast<const __nv_bfloat162*>(&rr.x);
        const __nv_bfloat162 r23 = *reinterpret_cast<const __nv_bfloat162*>(&rr.y);
        const float rf[4] = {__low2float(r01), __high2float(r01), __low2float(r23), __high2float(r23)};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float z = norm_out<__nv_bfloat16>(v[k][e], wf[e], ry, plus_one, MVB_NORM_MODEL, true);
          v[k][e] = bf16_round(rf[e] + z);
          ss += v[k][e] * v[k][e];
        }
        __nv_bfloat162 o01 = __floats2bfloat162_rn(v[k][0], v[k][1]);
        __nv_bfloat162 o23 = __floats2bfloat162_rn(v[k][2], v[k][3]);
        uint2 ov;
        ov.x = *reinterpret_cast<uint32_t*>(&o01);
        ov.y = *reinterpret_cast<uint32_t*>(&o23);
        *reinterpret_cast<uint2*>(res + i) = ov;
      }
    }
  }
  const float total = cluster_row_sum(ss, red, &cta_ss);
  const float rr = 1.0f / sqrtf(total / static_cast<float>(hidden) + eps);
#pragma unroll
  for (int k = 0; k < kFaddMaxRuns; ++k) {
    const int run = run0 + threadIdx.x + k * blockDim.x;
    if (run < run_end) {
      const int i = run * 4;
      const uint2 wr = *reinterpret_cast<const uint2*>(w + i);
      const __nv_bfloat162 w01 = *reinterpret_cast<const __nv_bfloat162*>(&wr.x);
      const __nv_bfloat162 w23 = *reinterpret_cast<const __nv_bfloat162*>(&wr.y);
      const float wf[4] = {__low2float(w01), __high2float(w01), __low2float(w23), __high2float(w23)};
      float o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        o[e] = norm_out<__nv_bfloat16>(v[k][e], wf[e], rr, plus_one, MVB_NORM_MODEL, true);
      __nv_bfloat162 o01 = __floats2bfloat162_rn(o[0], o[1]);
      __nv_bfloat162 o23 = __floats2bfloat162_rn(o[2], o[3]);
      uint2 ov;
      ov.x = *reinterpret_cast<uint32_t*>(&o01);
      ov.y = *reinterpret_cast<uint32_t*>(&o23);
      const int64_t off = static_cast<int64_t>(b) * hidden + i;
      if (TP) {
        for (int q = 0; q < tp.nranks; ++q) *reinterpret_cast<uint2*>(tp.out[q] + off) = ov;
      } else {
        *reinterpret_cast<uint2*>(out + off) = ov;
      }
    }
  }
  if (TP) {
    __syncthreads();
    if (threadIdx.x == 0) signal_ranks_once(tp.arrive, gridDim.x * gridDim.y, tp.signal, tp.nranks);
  }
}

// Cluster split of a row of `hidden` features: CTAs per row, runs of 4 per CTA, threads per CTA.
struct FaddSplit {
  int ctas, runs_per_cta, threads;
};
inline FaddSplit fadd_split(int64_t hidden) {
  FaddSplit s;
  const int runs = static_cast<int>(hidden / 4);
  s.ctas = static_cast<int>((hidden + 511) / 512);
  if (s.ctas > kFaddMaxCluster) s.ctas = kFaddMaxCluster;
  s.runs_per_cta = (runs + s.ctas - 1) / s.ctas;
  const int per_thread = (s.runs_per_cta + 255) / 256;
  s.threads = ((s.runs_per_cta + per_thread - 1) / per_thread + 31) / 32 * 32;
  if (s.threads < 64) s.threads = 64;
  return s;
}

int threads_for(int64_t hidden) {
  int t = static_cast<int>(((hidden + 3) / 4 + 31) / 32 * 32);
  return t < 64 ? 64 : (t > 1024 ? 1024 : t);
}

// norm_rows_kernel covers bf16 calls of more than 256 rows with hidden a multiple of 256 up to
// 8192 and 16-byte aligned rows; every other call (decode batches among them) takes the CTA-per-row
// kernels.
bool rows_form(int dtype, int64_t rows, int64_t hidden, const void* out, int64_t out_stride, const void* in,
               int64_t in_stride, const void* w, const void* residual) {
  return dtype == MVB_BF16 && rows > 256 && hidden % 256 == 0 && hidden <= 8192 && aligned(out, 16) &&
         aligned(in, 16) && aligned(w, 16) && (residual == nullptr || aligned(residual, 16)) && out_stride % 8 == 0 &&
         in_stride % 8 == 0;
}

template <bool ADD>
int launch_norm_rows(void* out, int64_t out_stride, void* residual, const void* in, int64_t in_stride,
                     const void* w, int64_t rows, int64_t hidden, float eps, int plus_one, int semantics,
                     cudaStream_t st) {
  const char* name = ADD ? "fused_add_rmsnorm_rows" : "rmsnorm_rows";
  const dim3 grid(static_cast<unsigned>((rows + 7) / 8)), block(256);
  auto* o = static_cast<__nv_bfloat16*>(out);
  auto* r = static_cast<__nv_bfloat16*>(residual);
  auto* x = static_cast<const __nv_bfloat16*>(in);
  auto* wt = static_cast<const __nv_bfloat16*>(w);
  const int h = static_cast<int>(hidden);
  if (hidden <= 2048)
    return launch(name, norm_rows_kernel<8, ADD>, grid, block, 0, st, o, out_stride, r, x, in_stride, wt, rows, h,
                  eps, plus_one, semantics);
  if (hidden <= 4096)
    return launch(name, norm_rows_kernel<16, ADD>, grid, block, 0, st, o, out_stride, r, x, in_stride, wt, rows, h,
                  eps, plus_one, semantics);
  return launch(name, norm_rows_kernel<32, ADD>, grid, block, 0, st, o, out_stride, r, x, in_stride, wt, rows, h,
                eps, plus_one, semantics);
}

}  // namespace
}  // namespace mvb

using namespace mvb;

extern "C" int mvb_rmsnorm(void* out, int64_t out_stride, const void* in, int64_t in_stride, const void* weight,
                           int64_t rows, int64_t hidden, float eps, int plus_one, int semantics, int dtype,
                           mvb_stream_t stream) {
  MVB_REQUIRE(out && in && weight, "mvb_rmsnorm: null pointer");
  MVB_REQUIRE(rows >= 0 && hidden > 0 && hidden <= (1 << 20), "mvb_rmsnorm: bad shape rows=%lld hidden=%lld",
              (long long)rows, (long long)hidden);
  MVB_REQUIRE(out_stride >= hidden && in_stride >= hidden, "mvb_rmsnorm: stride < hidden");
  MVB_REQUIRE(semantics == MVB_NORM_OPS || semantics == MVB_NORM_MODEL, "mvb_rmsnorm: bad semantics %d", semantics);
  if (rows == 0) return MVB_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (rows_form(dtype, rows, hidden, out, out_stride, in, in_stride, weight, nullptr))
    return launch_norm_rows<false>(out, out_stride, nullptr, in, in_stride, weight, rows, hidden, eps, plus_one,
                                   semantics, st);
  dim3 grid(static_cast<unsigned>(rows)), block(threads_for(hidden));
  switch (dtype) {
    case MVB_F32:
      return launch("rmsnorm", rmsnorm_kernel<float>, grid, block, 0, st, (float*)out, out_stride, (const float*)in,
                    in_stride, (const float*)weight, (int)hidden, eps, plus_one, semantics);
    case MVB_F16:
      return launch("rmsnorm", rmsnorm_kernel<__half>, grid, block, 0, st, (__half*)out, out_stride,
                    (const __half*)in, in_stride, (const __half*)weight, (int)hidden, eps, plus_one, semantics);
    case MVB_BF16:
      return launch("rmsnorm", rmsnorm_kernel<__nv_bfloat16>, grid, block, 0, st, (__nv_bfloat16*)out, out_stride,
                    (const __nv_bfloat16*)in, in_stride, (const __nv_bfloat16*)weight, (int)hidden, eps, plus_one,
                    semantics);
    default:
      return fail(MVB_ERR_INVALID_ARG, "mvb_rmsnorm: unsupported dtype %d", dtype);
  }
}

extern "C" int mvb_fused_add_rmsnorm(void* out, void* residual, const void* in, const void* weight, int64_t rows,
                                     int64_t hidden, float eps, int plus_one, int semantics, int dtype,
                                     mvb_stream_t stream) {
  MVB_REQUIRE(out && residual && in && weight, "mvb_fused_add_rmsnorm: null pointer");
  MVB_REQUIRE(rows >= 0 && hidden > 0 && hidden <= (1 << 20), "mvb_fused_add_rmsnorm: bad shape");
  MVB_REQUIRE(semantics == MVB_NORM_OPS || semantics == MVB_NORM_MODEL, "mvb_fused_add_rmsnorm: bad semantics");
  if (rows == 0) return MVB_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (rows_form(dtype, rows, hidden, out, hidden, in, hidden, weight, residual))
    return launch_norm_rows<true>(out, hidden, residual, in, hidden, weight, rows, hidden, eps, plus_one, semantics,
                                  st);
  dim3 grid(static_cast<unsigned>(rows)), block(threads_for(hidden));
  switch (dtype) {
    case MVB_F32:
      return launch("fused_add_rmsnorm", fused_add_rmsnorm_kernel<float>, grid, block, 0, st, (float*)out,
                    (float*)residual, (const float*)in, (const float*)weight, (int)hidden, eps, plus_one, semantics);
    case MVB_F16:
      return launch("fused_add_rmsnorm", fused_add_rmsnorm_kernel<__half>, grid, block, 0, st, (__half*)out,
                    (__half*)residual, (const __half*)in, (const __half*)weight, (int)hidden, eps, plus_one,
                    semantics);
    case MVB_BF16:
      return launch("fused_add_rmsnorm", fused_add_rmsnorm_kernel<__nv_bfloat16>, grid, block, 0, st,
                    (__nv_bfloat16*)out, (__nv_bfloat16*)residual, (const __nv_bfloat16*)in,
                    (const __nv_bfloat16*)weight, (int)hidden, eps, plus_one, semantics);
    default:
      return fail(MVB_ERR_INVALID_ARG, "mvb_fused_add_rmsnorm: unsupported dtype %d", dtype);
  }
}

extern "C" int mvb_fused_add_rmsnorm_gemm(void* out, void* residual, const void* gemm_workspace, int64_t rows,
                                          int64_t hidden, int64_t gemm_k, const void* weight, float eps,
                                          int plus_one, mvb_stream_t stream) {
  MVB_REQUIRE(out && residual && gemm_workspace && weight, "mvb_fused_add_rmsnorm_gemm: null pointer");
  MVB_REQUIRE(rows > 0 && rows <= 256 && hidden > 0 && gemm_k > 0 && gemm_k % kSplitBK == 0,
              "mvb_fused_add_rmsnorm_gemm: bad shape");
  const int sms = current_sm_count();
  MVB_REQUIRE(sms > 0, "mvb_fused_add_rmsnorm_gemm: no device");
  MVB_REQUIRE(hidden % 4 == 0 && hidden <= 16384,
              "mvb_fused_add_rmsnorm_gemm: hidden %lld must be a multiple of 4 and <= 16384", (long long)hidden);
  MVB_REQUIRE(aligned(residual, 8) && aligned(out, 8) && aligned(weight, 8),
              "mvb_fused_add_rmsnorm_gemm: 8-byte alignment");
  const SplitKPlan p = splitk_plan(rows, hidden, gemm_k, sms);
  const FaddSplit sp = fadd_split(hidden);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const TpFadd none{};
  return launch_cluster("fused_add_rmsnorm_gemm", fused_add_rmsnorm_gemm_kernel<false, false>,
                        dim3(static_cast<unsigned>(sp.ctas), static_cast<unsigned>(rows)), dim3(sp.threads),
                        static_cast<unsigned>(sp.ctas), 0, st, (__nv_bfloat16*)out, (__nv_bfloat16*)residual,
                        (const float*)gemm_workspace, p, (const __nv_bfloat16*)weight, (const __nv_bfloat16*)nullptr,
                        (int)hidden, sp.runs_per_cta, eps, plus_one, none, device_status_ptr());
}

extern "C" int mvb_fused_norm_add_rmsnorm_gemm(void* out, void* residual, const void* gemm_workspace, int64_t rows,
                                               int64_t hidden, int64_t gemm_k, const void* post_weight,
                                               const void* weight, float eps, int plus_one, mvb_stream_t stream) {
  MVB_REQUIRE(out && residual && gemm_workspace && post_weight && weight,
              "mvb_fused_norm_add_rmsnorm_gemm: null pointer");
  MVB_REQUIRE(rows > 0 && rows <= 256 && hidden > 0 && gemm_k > 0 && gemm_k % kSplitBK == 0,
              "mvb_fused_norm_add_rmsnorm_gemm: bad shape");
  const int sms = current_sm_count();
  MVB_REQUIRE(sms > 0, "mvb_fused_norm_add_rmsnorm_gemm: no device");
  MVB_REQUIRE(hidden % 4 == 0 && hidden <= 16384,
              "mvb_fused_norm_add_rmsnorm_gemm: hidden %lld must be a multiple of 4 and <= 16384", (long long)hidden);
  MVB_REQUIRE(aligned(residual, 8) && aligned(out, 8) && aligned(weight, 8) && aligned(post_weight, 8),
              "mvb_fused_norm_add_rmsnorm_gemm: 8-byte alignment");
  const SplitKPlan p = splitk_plan(rows, hidden, gemm_k, sms);
  const FaddSplit sp = fadd_split(hidden);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const TpFadd none{};
  return launch_cluster("fused_norm_add_rmsnorm_gemm", fused_add_rmsnorm_gemm_kernel<false, true>,
                        dim3(static_cast<unsigned>(sp.ctas), static_cast<unsigned>(rows)), dim3(sp.threads),
                        static_cast<unsigned>(sp.ctas), 0, st, (__nv_bfloat16*)out, (__nv_bfloat16*)residual,
                        (const float*)gemm_workspace, p, (const __nv_bfloat16*)weight,
                        (const __nv_bfloat16*)post_weight, (int)hidden, sp.runs_per_cta, eps, plus_one, none,
                        device_status_ptr());
}

static int tp_fused_add_rmsnorm_gemm_impl(mvb_tp_comm* comm, void* residual, int64_t rows, int64_t hidden,
                                          int64_t gemm_k, const void* post_weight, const void* weight, float eps,
                                          int plus_one, int64_t recv_offset, int wait_point, int64_t out_offset,
                                          int signal_point, mvb_stream_t stream) {
  MVB_REQUIRE(comm && residual && weight, "mvb_tp_fused_add_rmsnorm_gemm: null pointer");
  const int nr = comm->nranks;
  MVB_REQUIRE(rows > 0 && rows <= 256 && rows % nr == 0 && gemm_k > 0 && gemm_k % kSplitBK == 0,
              "mvb_tp_fused_add_rmsnorm_gemm: rows %lld must be in [1, 256] and a multiple of %d ranks",
              (long long)rows, nr);
  MVB_REQUIRE(hidden % 4 == 0 && hidden > 0 && hidden <= 16384,
              "mvb_tp_fused_add_rmsnorm_gemm: hidden %lld must be a multiple of 4 and <= 16384", (long long)hidden);
  MVB_REQUIRE(wait_point >= 0 && wait_point < kTpMaxPoints && signal_point >= 0 && signal_point < kTpMaxPoints &&
                  wait_point != signal_point,
              "mvb_tp_fused_add_rmsnorm_gemm: bad signal points");
  MVB_REQUIRE(comm->point_count[wait_point] > 0, "mvb_tp_fused_add_rmsnorm_gemm: nothing signals point %d",
              wait_point);
  MVB_REQUIRE(aligned(residual, 8) && aligned(weight, 8), "mvb_tp_fused_add_rmsnorm_gemm: 8-byte alignment");
  const int sms = current_sm_count();
  MVB_REQUIRE(sms > 0, "mvb_tp_fused_add_rmsnorm_gemm: no device");
  const int rpr = static_cast<int>(rows / nr);
  const SplitKPlan p = splitk_plan_push(rows, hidden, gemm_k, sms, nr);
  MVB_REQUIRE(recv_offset >= kTpSignalBytes && recv_offset % 16 == 0 &&
                  recv_offset + splitk_push_bytes(p, nr, rpr) <= comm->heap_bytes,
              "mvb_tp_fused_add_rmsnorm_gemm: receive area outside the heap");
  MVB_REQUIRE(out_offset >= kTpSignalBytes && out_offset % 16 == 0 &&
                  out_offset + rows * hidden * 2 <= comm->heap_bytes,
              "mvb_tp_fused_add_rmsnorm_gemm: output outside the heap");
  TpFadd tp{};
  tp.nranks = nr;
  tp.rank = comm->rank;
  tp.rows_per_rank = rpr;
  tp.recv = reinterpret_cast<const float*>(comm->base[comm->rank] + recv_offset);
  for (int q = 0; q < nr; ++q) {
    tp.out[q] = reinterpret_cast<__nv_bfloat16*>(comm->base[q] + out_offset);
    tp.signal[q] = comm->signal_slot(q, signal_point);
  }
  tp.arrive = comm->arrive_slot(signal_point);
  tp.wait = comm->wait_row(wait_point);
  tp.wait_count = comm->point_count[wait_point];
  tp.epoch = comm->epoch;
  const FaddSplit sp = fadd_split(hidden);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MVB_REQUIRE(post_weight == nullptr || aligned(post_weight, 8), "mvb_tp_fused_add_rmsnorm_gemm: 8-byte alignment");
  if (post_weight != nullptr) {
    MVB_TRY(launch_cluster("tp_fused_norm_add_rmsnorm_gemm", fused_add_rmsnorm_gemm_kernel<true, true>,
                           dim3(static_cast<unsigned>(sp.ctas), static_cast<unsigned>(rpr)), dim3(sp.threads),
                           static_cast<unsigned>(sp.ctas), 0, st, (__nv_bfloat16*)nullptr, (__nv_bfloat16*)residual,
                           (const float*)nullptr, p, (const __nv_bfloat16*)weight,
                           (const __nv_bfloat16*)post_weight, (int)hidden, sp.runs_per_cta, eps, plus_one, tp,
                           device_status_ptr()));
  } else {
    MVB_TRY(launch_cluster("tp_fused_add_rmsnorm_gemm", fused_add_rmsnorm_gemm_kernel<true, false>,
                           dim3(static_cast<unsigned>(sp.ctas), static_cast<unsigned>(rpr)), dim3(sp.threads),
                           static_cast<unsigned>(sp.ctas), 0, st, (__nv_bfloat16*)nullptr, (__nv_bfloat16*)residual,
                           (const float*)nullptr, p, (const __nv_bfloat16*)weight, (const __nv_bfloat16*)nullptr,
                           (int)hidden, sp.runs_per_cta, eps, plus_one, tp, device_status_ptr()));
  }
  comm->point_count[signal_point] = 1;
  return MVB_OK;
}

extern "C" int mvb_tp_fused_add_rmsnorm_gemm(mvb_tp_comm* comm, void* residual, int64_t rows, int64_t hidden,
                                             int64_t gemm_k, const void* weight, float eps, int plus_one,
                                             int64_t recv_offset, int wait_point, int64_t out_offset,
                                             int signal_point, mvb_stream_t stream) {
  return tp_fused_add_rmsnorm_gemm_impl(comm, residual, rows, hidden, gemm_k, nullptr, weight, eps, plus_one,
                                        recv_offset, wait_point, out_offset, signal_point, stream);
}

extern "C" int mvb_tp_fused_norm_add_rmsnorm_gemm(mvb_tp_comm* comm, void* residual, int64_t rows, int64_t hidden,
                                                  int64_t gemm_k, const void* post_weight, const void* weight,
                                                  float eps, int plus_one, int64_t recv_offset, int wait_point,
                                                  int64_t out_offset, int signal_point, mvb_stream_t stream) {
  MVB_REQUIRE(post_weight != nullptr, "mvb_tp_fused_norm_add_rmsnorm_gemm: null post weight");
  return tp_fused_add_rmsnorm_gemm_impl(comm, residual, rows, hidden, gemm_k, post_weight, weight, eps, plus_one,
                                        recv_offset, wait_point, out_offset, signal_point, stream);
}
