// Fused per-head QK RMSNorm + NeoX RoPE + paged KV-cache write for one decode step.
//
// Replaces, for a single new token per sequence, the chain
//   q_norm / k_norm            models/model.py:174-178   (RMSNorm.forward, model.py:19-25)
//   apply_rotary_pos_emb       models/model.py:184       (q*cos + rotate_half(q)*sin, bf16 ops)
//   Attention._write_kv_cache  models/model.py:226-243   (kv[l, 0|1, bt[pos//bs], pos%bs] = k|v)
// One warp per (sequence, head) of the fused q|k|v projection row.  Lane l owns
// head_dim/32 consecutive elements; its rotate_half partner sits 16 lanes away.
// The slot of a token is (block_tables[b][pos / bs], pos % bs) exactly as the
// reference computes it; an out-of-range table index or block id is reported in
// the device status word and nothing is written for that token.
#include "common.cuh"
#include "host.h"
#include "qk_rope.cuh"
#include "splitk.cuh"

namespace mvb {
namespace {

template <int D>
__global__ void __launch_bounds__(256) qk_norm_rope_kv_kernel(
    __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ kv, const __nv_bfloat16* __restrict__ qkv,
    int64_t qkv_stride, const __nv_bfloat16* __restrict__ qnw, const __nv_bfloat16* __restrict__ knw,
    const __nv_bfloat16* __restrict__ cos_t, const __nv_bfloat16* __restrict__ sin_t, int64_t table_len,
    const int32_t* __restrict__ positions, const int32_t* __restrict__ block_tables, int64_t max_blocks, int batch,
    int nq, int nkv, int64_t layer, int64_t num_blocks, int bs, float eps, int plus_one, unsigned* err,
    const float* __restrict__ partials, SplitKPlan plan) {
  pdl_launch_dependents();
  const int warp_global = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int heads = nq + 2 * nkv;
  if (warp_global >= batch * heads) return;
  const int b = warp_global / heads;
  const int h = warp_global - b * heads;
  // Programmatic dependent launch: the position, block table, norm weights and cos/sin are step
  // metadata or constant tables, loaded while the GEMM before this kernel still runs; only the
  // projection itself waits for it.
  QkMeta<D> m;
  qk_meta_load<D>(m, b, h, lane, qnw, knw, cos_t, sin_t, table_len, positions, block_tables, max_blocks, nq, nkv,
                  layer, num_blocks, bs, err);
  pdl_wait();
  float x[D / 32];
  qk_load_x<D>(b, h, lane, x, qkv, qkv_stride, partials, plan);
  qk_apply<D>(m, b, h, lane, x, q_out, kv, nq, nkv, eps, plus_one);
}

}  // namespace
}  // namespace mvb

using namespace mvb;

static int qk_norm_rope_kv_write_impl(void* q_out, void* kv_cache, const void* qkv, int64_t qkv_stride,
                                      const void* q_norm_w, const void* k_norm_w, const void* cos, const void* sin,
                                      int64_t table_len, const int32_t* positions, const int32_t* block_tables,
                                      int64_t max_blocks, int64_t batch, int64_t num_q_heads, int64_t num_kv_heads,
                                      int64_t head_dim, int64_t num_layers, int64_t layer, int64_t num_blocks,
                                      int64_t block_size, float eps, int plus_one, const float* partials,
                                      SplitKPlan plan, mvb_stream_t stream) {
  MVB_REQUIRE(q_out && kv_cache && (qkv || partials) && cos && sin && positions && block_tables,
              "mvb_qk_norm_rope_kv_write: null pointer");
  MVB_REQUIRE((q_norm_w == nullptr) == (k_norm_w == nullptr),
              "mvb_qk_norm_rope_kv_write: pass both norm weights or neither");
  MVB_REQUIRE(batch >= 0 && num_q_heads > 0 && num_kv_heads > 0 && num_q_heads % num_kv_heads == 0,
              "mvb_qk_norm_rope_kv_write: bad head counts");
  MVB_REQUIRE(layer >= 0 && layer < num_layers && num_blocks > 0 && block_size > 0 && max_blocks > 0,
              "mvb_qk_norm_rope_kv_write: bad cache geometry");
  MVB_REQUIRE(partials || qkv_stride >= (num_q_heads + 2 * num_kv_heads) * head_dim,
              "mvb_qk_norm_rope_kv_write: qkv_stride");
  if (batch == 0) return MVB_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned* err = device_status_ptr();
  const int64_t warps = batch * (num_q_heads + 2 * num_kv_heads);
  dim3 grid(static_cast<unsigned>((warps + 7) / 8)), block(256);
#define MVB_QKR_LAUNCH(D)                                                                                        \
  return launch("qk_norm_rope_kv_write", qk_norm_rope_kv_kernel<D>, grid, block, 0, st, (__nv_bfloat16*)q_out,  \
                (__nv_bfloat16*)kv_cache, (const __nv_bfloat16*)qkv, qkv_stride, (const __nv_bfloat16*)q_norm_w, \
                (const __nv_bfloat16*)k_norm_w, (const __nv_bfloat16*)cos, (const __nv_bfloat16*)sin, table_len,  \
                positions, block_tables, max_blocks, (int)batch, (int)num_q_heads, (int)num_kv_heads, layer,     \
                num_blocks, (int)block_size, eps, plus_one, err, partials, plan)
  switch (head_dim) {
    case 64: MVB_QKR_LAUNCH(64);
    case 128: MVB_QKR_LAUNCH(128);
    case 256: MVB_QKR_LAUNCH(256);
    default: return fail(MVB_ERR_UNSUPPORTED, "mvb_qk_norm_rope_kv_write: head_dim %lld", (long long)head_dim);
  }
#undef MVB_QKR_LAUNCH
}

extern "C" int mvb_qk_norm_rope_kv_write(void* q_out, void* kv_cache, const void* qkv, int64_t qkv_stride,
                                         const void* q_norm_w, const void* k_norm_w, const void* cos,
                                         const void* sin, int64_t table_len, const int32_t* positions,
                                         const int32_t* block_tables, int64_t max_blocks, int64_t batch,
                                         int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                                         int64_t num_layers, int64_t layer, int64_t num_blocks, int64_t block_size,
                                         float eps, int plus_one, mvb_stream_t stream) {
  return qk_norm_rope_kv_write_impl(q_out, kv_cache, qkv, qkv_stride, q_norm_w, k_norm_w, cos, sin, table_len,
                                    positions, block_tables, max_blocks, batch, num_q_heads, num_kv_heads, head_dim,
                                    num_layers, layer, num_blocks, block_size, eps, plus_one, nullptr, SplitKPlan{},
                                    stream);
}

extern "C" int mvb_qk_norm_rope_kv_write_gemm(void* q_out, void* kv_cache, const void* gemm_workspace,
                                              int64_t gemm_k, const void* q_norm_w, const void* k_norm_w,
                                              const void* cos, const void* sin, int64_t table_len,
                                              const int32_t* positions, const int32_t* block_tables,
                                              int64_t max_blocks, int64_t batch, int64_t num_q_heads,
                                              int64_t num_kv_heads, int64_t head_dim, int64_t num_layers,
                                              int64_t layer, int64_t num_blocks, int64_t block_size, float eps,
                                              int plus_one, mvb_stream_t stream) {
  MVB_REQUIRE(gemm_workspace && batch > 0 && batch <= 256 && gemm_k > 0 && gemm_k % kSplitBK == 0,
              "mvb_qk_norm_rope_kv_write_gemm: bad arguments");
  const int sms = current_sm_count();
  MVB_REQUIRE(sms > 0, "mvb_qk_norm_rope_kv_write_gemm: no device");
  const SplitKPlan plan = splitk_plan(batch, (num_q_heads + 2 * num_kv_heads) * head_dim, gemm_k, sms);
  return qk_norm_rope_kv_write_impl(q_out, kv_cache, nullptr, 0, q_norm_w, k_norm_w, cos, sin, table_len,
                                    positions, block_tables, max_blocks, batch, num_q_heads, num_kv_heads, head_dim,
                                    num_layers, layer, num_blocks, block_size, eps, plus_one,
                                    static_cast<const float*>(gemm_workspace), plan, stream);
}
