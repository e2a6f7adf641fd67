// Elementwise / row ops of the mini_vllm ops API: activations, gated activations,
// fused MLP activation, embedding gather, row softmax, standalone RoPE.
//
// Each reproduces the rounding sequence of the PyTorch expression it replaces:
//   silu / gelu(tanh)            ops/activation.py:10-30       y = T(act(x))
//   swiglu / geglu               ops/activation.py:33-66       y = T(T(act(g)) * u)
//   fused_mlp (FusedMLP fallback) ops/mlp.py:73-82             y = T(T(act(g)) * u)
//   swiglu of split-K partials   models/model.py:116-117       y = T(T(silu(T(g))) * T(u))
//   embedding                    ops/embedding.py:11-35        y = W[id] (* scale, rounded)
//   softmax                      ops/softmax.py:5-25           fp32 exp/sum, one rounding
//   rotary                       ops/rope.py:74-76             y = T(T(x*cos) + T(rot(x)*sin))
#include "common.cuh"
#include "host.h"
#include "splitk.cuh"

namespace mvb {
namespace {

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float kBeta = 0.7978845608028654f;  // sqrt(2/pi)
  const float kKappa = 0.044715f;
  return 0.5f * x * (1.0f + tanhf(kBeta * (x + kKappa * x * x * x)));
}

__device__ __forceinline__ float act_f(float x, int act) { return act == MVB_ACT_SILU ? silu_f(x) : gelu_tanh_f(x); }

template <typename T>
__global__ void activation_kernel(T* __restrict__ out, const T* __restrict__ in, int64_t n, int act) {
  pdl_launch_dependents();
  pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = from_f<T>(act_f(to_f<T>(in[i]), act));
}

template <typename T>
__global__ void gated_kernel(T* __restrict__ out, const T* __restrict__ gate, const T* __restrict__ up, int64_t n,
                             int act) {
  pdl_launch_dependents();
  pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = from_f<T>(rnd<T>(act_f(to_f<T>(gate[i]), act)) * to_f<T>(up[i]));
}

template <typename T>
__global__ void fused_mlp_kernel(T* __restrict__ out, const T* __restrict__ gate_up, int64_t rows, int64_t inter,
                                 int act) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t n = rows * inter;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / inter, j = i - r * inter;
    const T* row = gate_up + r * 2 * inter;
    out[i] = from_f<T>(rnd<T>(act_f(to_f<T>(row[j]), act)) * to_f<T>(row[inter + j]));
  }
}

// act(gate) * up of a SwiGLU-paired GEMM still in split-K partial form
// (MVB_EPI_SWIGLU_PARTIALS): tile t = j / 64 holds gate feature j in row j % 64 and up feature
// j in row 64 + j % 64 of each contributor slot.  Both sums run in contributor order; the
// rounding sequence is that of the GEMM's SWIGLU epilogue.  act: SiLU (SwiGLU) or tanh-GELU
// (GeGLU, models/gemma3_model.py:104-105).  Thread = 4 consecutive features of one batch row
// (blockIdx.y).
__global__ void swiglu_gemm_kernel(__nv_bfloat16* __restrict__ out, int64_t out_stride,
                                   const float* __restrict__ partials, SplitKPlan p, int inter, int act) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.y;
  const int j = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (j >= inter) return;
  const int t = j >> 6, r = j & 63;
  const int nc = sk_count(p, t);
  float4 g = make_float4(0.f, 0.f, 0.f, 0.f), u = g;
  for (int c = 0; c < nc; ++c) {
    const float* base = partials + sk_offset(p, t, c, b, r);
    const float4 pg = __ldcg(reinterpret_cast<const float4*>(base));
    const float4 pu = __ldcg(reinterpret_cast<const float4*>(base + 64));
    g.x += pg.x;
    g.y += pg.y;
    g.z += pg.z;
    g.w += pg.w;
    u.x += pu.x;
    u.y += pu.y;
    u.z += pu.z;
    u.w += pu.w;
  }
  auto h = [act](float gv, float uv) { return bf16_round(act_f(bf16_round(gv), act)) * bf16_round(uv); };
  __nv_bfloat162 o01 = __floats2bfloat162_rn(h(g.x, u.x), h(g.y, u.y));
  __nv_bfloat162 o23 = __floats2bfloat162_rn(h(g.z, u.z), h(g.w, u.w));
  uint2 ov;
  ov.x = *reinterpret_cast<uint32_t*>(&o01);
  ov.y = *reinterpret_cast<uint32_t*>(&o23);
  *reinterpret_cast<uint2*>(out + static_cast<int64_t>(b) * out_stride + j) = ov;
}

// Gemma-2 final-logit soft-capping, x = T(T(tanh(T(x / cap))) * cap) (the three PyTorch ops
// `x / cap`, `tanh`, `* cap` in the logits' dtype).
template <typename T>
__global__ void softcap_kernel(T* __restrict__ x, int64_t n, float cap) {
  pdl_launch_dependents();
  pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float t = rnd<T>(tanhf(rnd<T>(to_f<T>(x[i]) / cap)));
    x[i] = from_f<T>(t * cap);
  }
}

// Input ids of a step from the previous step's sampled tokens when *feed is nonzero (the engine
// launched the step before reading those tokens back); otherwise the ids stay as uploaded.
__global__ void feed_ids_kernel(int32_t* __restrict__ ids, const int64_t* __restrict__ tokens,
                                const int32_t* __restrict__ feed, int64_t n) {
  pdl_launch_dependents();
  pdl_wait();
  if (*feed == 0) return;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    ids[i] = static_cast<int32_t>(tokens[i]);
}

template <typename T, typename I>
__global__ void embedding_kernel(T* __restrict__ out, const I* __restrict__ ids, const T* __restrict__ w,
                                 int64_t hidden, int64_t vocab, float scale, unsigned* err) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t t = blockIdx.x;
  const int64_t id = static_cast<int64_t>(ids[t]);
  T* y = out + t * hidden;
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) report(err, kDevBadToken);
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) y[i] = from_f<T>(0.0f);
    return;
  }
  const T* src = w + id * hidden;
  if (scale == 1.0f) {
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) y[i] = src[i];
  } else {
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) y[i] = from_f<T>(to_f<T>(src[i]) * scale);
  }
}

template <typename T>
__global__ void softmax_kernel(T* __restrict__ out, const T* __restrict__ in, int64_t n) {
  __shared__ float red[32];
  pdl_launch_dependents();
  pdl_wait();
  const T* x = in + blockIdx.x * n;
  T* y = out + blockIdx.x * n;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  float m = -INFINITY;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, to_f<T>(x[i]));
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = warp_max(lane < nw ? red[lane] : -INFINITY);
  __syncthreads();
  float s = 0.0f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += expf(to_f<T>(x[i]) - m);
  s = warp_sum(s);
  if (lane == 0) red[warp] = s;
  __syncthreads();
  s = warp_sum(lane < nw ? red[lane] : 0.0f);
  const float inv = 1.0f / s;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) y[i] = from_f<T>(expf(to_f<T>(x[i]) - m) * inv);
}

template <typename T>
__global__ void rope_kernel(T* __restrict__ out, const T* __restrict__ in, const T* __restrict__ cos,
                            const T* __restrict__ sin, int64_t rows, int hd) {
  pdl_launch_dependents();
  pdl_wait();
  const int half = hd / 2;
  const int64_t n = rows * hd;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / hd;
    const int d = static_cast<int>(i - r * hd);
    const T* x = in + r * hd;
    const float xv = to_f<T>(x[d]);
    const float rot = d < half ? -to_f<T>(x[d + half]) : to_f<T>(x[d - half]);
    const float a = rnd<T>(xv * to_f<T>(cos[i]));
    const float b = rnd<T>(rot * to_f<T>(sin[i]));
    out[i] = from_f<T>(a + b);
  }
}

dim3 grid_for(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  if (b > 148 * 32) b = 148 * 32;
  if (b < 1) b = 1;
  return dim3(static_cast<unsigned>(b));
}

}  // namespace
}  // namespace mvb

using namespace mvb;

#define MVB_DISPATCH_FLOAT(dtype, NAME, ...)                                            \
  switch (dtype) {                                                                      \
    case MVB_F32: { using T = float; __VA_ARGS__; }                                     \
    case MVB_F16: { using T = __half; __VA_ARGS__; }                                    \
    case MVB_BF16: { using T = __nv_bfloat16; __VA_ARGS__; }                            \
    default: return fail(MVB_ERR_INVALID_ARG, NAME ": unsupported dtype %d", dtype);  \
  }

extern "C" int mvb_activation(void* out, const void* in, int64_t n, int act, int dtype, mvb_stream_t stream) {
  MVB_REQUIRE(out && in && n >= 0, "mvb_activation: bad arguments");
  MVB_REQUIRE(act == MVB_ACT_SILU || act == MVB_ACT_GELU_TANH, "mvb_activation: bad act %d", act);
  if (n == 0) return MVB_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MVB_DISPATCH_FLOAT(dtype, "mvb_activation",
                     return launch("activation", activation_kernel<T>, grid_for(n, 256), dim3(256), 0, st, (T*)out,
                                   (const T*)in, n, act));
}

extern "C" int mvb_gated_activation(void* out, const void* gate, const void* up, int64_t n, int act, int dtype,
                                    mvb_stream_t stream) {
  MVB_REQUIRE(out && gate && up && n >= 0, "mvb_gated_activation: bad arguments");
  MVB_REQUIRE(act == MVB_ACT_SILU || act == MVB_ACT_GELU_TANH, "mvb_gated_activation: bad act %d", act);
  if (n == 0) return MVB_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MVB_DISPATCH_FLOAT(dtype, "mvb_gated_activation",
                     return launch("gated_activation", gated_kernel<T>, grid_for(n, 256), dim3(256), 0, st, (T*)out,
                                   (const T*)gate, (const T*)up, n, act));
}

extern "C" int mvb_fused_mlp(void* out, const void* gate_up, int64_t rows, int64_t inter, int act, int dtype,
                             mvb_stream_t stream) {
  MVB_REQUIRE(out && gate_up && rows >= 0 && inter > 0, "mvb_fused_mlp: bad arguments");
  MVB_REQUIRE(act == MVB_ACT_SILU || act == MVB_ACT_GELU_TANH, "mvb_fused_mlp: bad act %d", act);
  if (rows == 0) return MVB_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MVB_DISPATCH_FLOAT(dtype, "mvb_fused_mlp",
                     return launch("fused_mlp", fused_mlp_kernel<T>, grid_for(rows * inter, 256), dim3(256), 0, st,
                                   (T*)out, (const T*)gate_up, rows, inter, act));
}

extern "C" int mvb_embedding(void* out, const void* ids, int ids_dtype, const void* weight, int64_t tokens,
                             int64_t hidden, int64_t vocab, float scale, int dtype, mvb_stream_t stream) {
  MVB_REQUIRE(out && ids && weight && tokens >= 0 && hidden > 0 && vocab > 0, "mvb_embedding: bad arguments");
  MVB_REQUIRE(ids_dtype == MVB_I32 || ids_dtype == MVB_I64, "mvb_embedding: ids must be int32 or int64");
  if (tokens == 0) return MVB_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned* err = device_status_ptr();
  const int threads = hidden >= 1024 ? 256 : 128;
  dim3 grid(static_cast<unsigned>(tokens));
  if (ids_dtype == MVB_I64) {
    MVB_DISPATCH_FLOAT(dtype, "mvb_embedding",
                       return launch("embedding", embedding_kernel<T, int64_t>, grid, dim3(threads), 0, st, (T*)out,
                                     (const int64_t*)ids, (const T*)weight, hidden, vocab, scale, err));
  }
  MVB_DISPATCH_FLOAT(dtype, "mvb_embedding",
                     return launch("embedding", embedding_kernel<T, int32_t>, grid, dim3(threads), 0, st, (T*)out,
                                   (const int32_t*)ids, (const T*)weight, hidden, vocab, scale, err));
}

extern "C" int mvb_softmax(void* out, const void* in, int64_t rows, int64_t n, int dtype, mvb_stream_t stream) {
  MVB_REQUIRE(out && in && rows >= 0 && n > 0, "mvb_softmax: bad arguments");
  if (rows == 0) return MVB_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int threads = n >= 4096 ? 1024 : (n >= 512 ? 256 : 64);
  MVB_DISPATCH_FLOAT(dtype, "mvb_softmax",
                     return launch("softmax", softmax_kernel<T>, dim3(static_cast<unsigned>(rows)), dim3(threads), 0,
                                   st, (T*)out, (const T*)in, n));
}

extern "C" int mvb_rotary_pos_emb(void* out, const void* in, const void* cos, const void* sin, int64_t rows,
                                  int64_t head_dim, int dtype, mvb_stream_t stream) {
  MVB_REQUIRE(out && in && cos && sin && rows >= 0, "mvb_rotary_pos_emb: bad arguments");
  MVB_REQUIRE(head_dim > 0 && head_dim % 2 == 0 && head_dim <= 1024, "mvb_rotary_pos_emb: bad head_dim %lld",
              (long long)head_dim);
  if (rows == 0) return MVB_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MVB_DISPATCH_FLOAT(dtype, "mvb_rotary_pos_emb",
                     return launch("rotary_pos_emb", rope_kernel<T>, grid_for(rows * head_dim, 256), dim3(256), 0,
                                   st, (T*)out, (const T*)in, (const T*)cos, (const T*)sin, rows, (int)head_dim));
}

extern "C" int mvb_softcap(void* x, int64_t n, float cap, int dtype, mvb_stream_t stream) {
  MVB_REQUIRE(x && n >= 0 && cap > 0.0f, "mvb_softcap: bad arguments");
  if (n == 0) return MVB_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int sms = current_sm_count();
  MVB_REQUIRE(sms > 0, "mvb_softcap: no device");
  int64_t blocks = (n + 255) / 256;
  if (blocks > 8LL * sms) blocks = 8LL * sms;
  switch (dtype) {
    case MVB_BF16:
      return launch("softcap", softcap_kernel<__nv_bfloat16>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, st,
                    (__nv_bfloat16*)x, n, cap);
    case MVB_F32:
      return launch("softcap", softcap_kernel<float>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, st,
                    (float*)x, n, cap);
    default:
      return fail(MVB_ERR_INVALID_ARG, "mvb_softcap: unsupported dtype %d", dtype);
  }
}

extern "C" int mvb_feed_ids(int32_t* ids, const int64_t* tokens, const int32_t* feed, int64_t n, mvb_stream_t stream) {
  MVB_REQUIRE(ids && tokens && feed && n >= 0 && n <= (1LL << 20), "mvb_feed_ids: bad arguments");
  if (n == 0) return MVB_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return launch("feed_ids", feed_ids_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, st, ids,
                tokens, feed, n);
}

extern "C" int mvb_gated_gemm(void* out, int64_t out_stride, const void* gemm_workspace, int64_t rows, int64_t inter,
                              int64_t gemm_k, int act, mvb_stream_t stream) {
  MVB_REQUIRE(act == MVB_ACT_SILU || act == MVB_ACT_GELU_TANH, "mvb_gated_gemm: activation %d", act);
  MVB_REQUIRE(out && gemm_workspace, "mvb_swiglu_gemm: null pointer");
  MVB_REQUIRE(rows > 0 && rows <= 256 && inter > 0 && inter % 4 == 0 && inter < (1LL << 30) && gemm_k > 0 &&
                  gemm_k % kSplitBK == 0,
              "mvb_swiglu_gemm: bad shape rows=%lld inter=%lld k=%lld", (long long)rows, (long long)inter,
              (long long)gemm_k);
  MVB_REQUIRE(out_stride >= inter && out_stride % 4 == 0 && aligned(out, 8),
              "mvb_swiglu_gemm: out_stride must be >= inter and a multiple of 4, out 8-byte aligned");
  const int sms = current_sm_count();
  MVB_REQUIRE(sms > 0, "mvb_swiglu_gemm: no device");
  const SplitKPlan p = splitk_plan_swiglu(rows, inter, gemm_k, sms);
  const unsigned bx = static_cast<unsigned>((inter / 4 + 255) / 256);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return launch("swiglu_gemm", swiglu_gemm_kernel, dim3(bx, static_cast<unsigned>(rows)), dim3(256), 0, st,
                (__nv_bfloat16*)out, out_stride, (const float*)gemm_workspace, p, (int)inter, act);
}

extern "C" int mvb_swiglu_gemm(void* out, int64_t out_stride, const void* gemm_workspace, int64_t rows, int64_t inter,
                               int64_t gemm_k, mvb_stream_t stream) {
  return mvb_gated_gemm(out, out_stride, gemm_workspace, rows, inter, gemm_k, MVB_ACT_SILU, stream);
}
