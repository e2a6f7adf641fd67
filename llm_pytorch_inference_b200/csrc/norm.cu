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

// Residual add + RMSNorm whose input is a GEMM's output still in split-K partial form: the
// linear layer's bf16 output is formed here as bf16(sum of the tile's partial slots, contributor
// order), then residual += it and out = RMSNorm(residual) (model semantics, models/model.py:19-25,
// :319).  Each thread owns runs of 4 consecutive features (float4 partial loads, 8-byte residual
// loads) and keeps its values in registers between the two passes; per-tile contributor counts
// are computed once per CTA.  Supports hidden % 4 == 0 and hidden <= 16 * blockDim.
constexpr int kFaddMaxRuns = 4;
constexpr int kFaddMaxTiles = 256;

__global__ void fused_add_rmsnorm_gemm_kernel(__nv_bfloat16* __restrict__ out, __nv_bfloat16* __restrict__ residual,
                                              const float* __restrict__ partials, SplitKPlan p,
                                              const __nv_bfloat16* __restrict__ w, int hidden, float eps,
                                              int plus_one) {
  __shared__ float red[32];
  __shared__ unsigned char s_nc[kFaddMaxTiles];
  pdl_launch_dependents();
  const int tiles = (hidden + kSplitBM - 1) / kSplitBM;
  for (int t = threadIdx.x; t < tiles; t += blockDim.x) s_nc[t] = static_cast<unsigned char>(sk_count(p, t));
  pdl_wait();
  __syncthreads();
  const int b = blockIdx.x;
  __nv_bfloat16* res = residual + static_cast<int64_t>(b) * hidden;
  __nv_bfloat16* y = out + static_cast<int64_t>(b) * hidden;
  float v[kFaddMaxRuns][4];
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < kFaddMaxRuns; ++k) {
    const int i = (threadIdx.x + k * blockDim.x) * 4;
    if (i < hidden) {
      const int t = i / kSplitBM, r = i - t * kSplitBM;
      const int nc = s_nc[t];
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int j = 0; j < nc; ++j) {
        const float4 q = __ldcg(reinterpret_cast<const float4*>(partials + sk_offset(p, t, j, b, r)));
        acc.x += q.x;
        acc.y += q.y;
        acc.z += q.z;
        acc.w += q.w;
      }
      const uint2 rr = *reinterpret_cast<const uint2*>(res + i);
      const __nv_bfloat162 r01 = *reinterpret_cast<const __nv_bfloat162*>(&rr.x);
      const __nv_bfloat162 r23 = *reinterpret_cast<const __nv_bfloat162*>(&rr.y);
      v[k][0] = bf16_round(__low2float(r01) + bf16_round(acc.x));
      v[k][1] = bf16_round(__high2float(r01) + bf16_round(acc.y));
      v[k][2] = bf16_round(__low2float(r23) + bf16_round(acc.z));
      v[k][3] = bf16_round(__high2float(r23) + bf16_round(acc.w));
      __nv_bfloat162 o01 = __floats2bfloat162_rn(v[k][0], v[k][1]);
      __nv_bfloat162 o23 = __floats2bfloat162_rn(v[k][2], v[k][3]);
      uint2 ov;
      ov.x = *reinterpret_cast<uint32_t*>(&o01);
      ov.y = *reinterpret_cast<uint32_t*>(&o23);
      *reinterpret_cast<uint2*>(res + i) = ov;
      ss += v[k][0] * v[k][0] + v[k][1] * v[k][1] + v[k][2] * v[k][2] + v[k][3] * v[k][3];
    }
  }
  ss = block_sum(ss, red);
  const float rr = 1.0f / sqrtf(ss / static_cast<float>(hidden) + eps);
#pragma unroll
  for (int k = 0; k < kFaddMaxRuns; ++k) {
    const int i = (threadIdx.x + k * blockDim.x) * 4;
    if (i < hidden) {
      float o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        o[e] = norm_out<__nv_bfloat16>(v[k][e], __bfloat162float(w[i + e]), rr, plus_one, MVB_NORM_MODEL, true);
      __nv_bfloat162 o01 = __floats2bfloat162_rn(o[0], o[1]);
      __nv_bfloat162 o23 = __floats2bfloat162_rn(o[2], o[3]);
      uint2 ov;
      ov.x = *reinterpret_cast<uint32_t*>(&o01);
      ov.y = *reinterpret_cast<uint32_t*>(&o23);
      *reinterpret_cast<uint2*>(y + i) = ov;
    }
  }
}

int threads_for(int64_t hidden) {
  int t = static_cast<int>(((hidden + 3) / 4 + 31) / 32 * 32);
  return t < 64 ? 64 : (t > 1024 ? 1024 : t);
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
  MVB_REQUIRE(hidden % 4 == 0 && hidden <= 4 * 1024 * kFaddMaxRuns && (hidden + 127) / 128 <= kFaddMaxTiles,
              "mvb_fused_add_rmsnorm_gemm: hidden %lld must be a multiple of 4 and <= 16384", (long long)hidden);
  MVB_REQUIRE(aligned(residual, 8) && aligned(out, 8), "mvb_fused_add_rmsnorm_gemm: 8-byte alignment");
  const SplitKPlan p = splitk_plan(rows, hidden, gemm_k, sms);
  MVB_REQUIRE(p.maxc <= 255, "mvb_fused_add_rmsnorm_gemm: too many split-K contributors");
  int threads = static_cast<int>((hidden / 4 + kFaddMaxRuns - 1) / kFaddMaxRuns);
  threads = (threads + 31) / 32 * 32;
  if (threads < 128) threads = 128;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return launch("fused_add_rmsnorm_gemm", fused_add_rmsnorm_gemm_kernel, dim3(static_cast<unsigned>(rows)),
                dim3(threads), 0, st, (__nv_bfloat16*)out, (__nv_bfloat16*)residual,
                (const float*)gemm_workspace, p, (const __nv_bfloat16*)weight, (int)hidden, eps, plus_one);
}
