/*
 * mvb200.h -- C ABI of the B200 (sm_100a) mini_vllm decode-path kernels.
 *
 * Every entry point takes caller-owned device pointers, plain sizes and a
 * cudaStream_t, launches on that stream, never allocates, never synchronises,
 * and returns an int status (MVB_OK or an MVB_ERR_* code; the message is in
 * mvb_last_error()).  Device-side conditions that a kernel detects instead of
 * faulting (a bounded wait that gave up, a block id or position out of range)
 * are ORed into a device status word read back with mvb_device_status().
 *
 * Reference interface replaced by each entry point: the torch dispatcher schema
 * in csrc/bindings/ops_binding.cpp:10-26 (TORCH_LIBRARY(mini_vllm_ops)) and the
 * host wrappers in csrc/kernels/<op>/<op>_kernel.cu, plus the model/engine code
 * for the entry points that the reference implements in Python/cuBLAS.
 *
 * Layouts are row-major.  dtype codes: MVB_F32, MVB_F16, MVB_BF16.
 */
#ifndef MVB200_H_
#define MVB200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* mvb_stream_t; /* == cudaStream_t */

/* ---- status codes -------------------------------------------------------- */
#define MVB_OK 0
#define MVB_ERR_INVALID_ARG 1 /* a size, pointer, alignment or dtype the kernel does not take */
#define MVB_ERR_UNSUPPORTED 2 /* a shape outside what this build was compiled for */
#define MVB_ERR_CUDA 3        /* launch / runtime error (message names it) */
#define MVB_ERR_DRIVER 4      /* driver entry point (tensor-map encoder) unavailable */

/* ---- device status bits (mvb_device_status) ------------------------------ */
#define MVB_DEV_WAIT_TIMEOUT 0x1u /* a bounded wait expired; the kernel unwound */
#define MVB_DEV_BAD_BLOCK 0x2u    /* a block-table entry was outside [0, num_blocks) */
#define MVB_DEV_BAD_POSITION 0x4u /* a position was outside its block table / table */
#define MVB_DEV_BAD_TOKEN 0x8u    /* a token id was outside [0, vocab) */
#define MVB_DEV_SAMPLER_TIES 0x10u /* > 2048 logits tied at the top-k cutoff; ties past 2048 were dropped */

/* ---- dtype codes ---------------------------------------------------------- */
#define MVB_F32 0
#define MVB_F16 1
#define MVB_BF16 2
#define MVB_I32 3
#define MVB_I64 4

/* ---- activation codes (mlp_kernel.cu:12-13: 0 = silu, 1 = gelu) ---------- */
#define MVB_ACT_SILU 0
#define MVB_ACT_GELU_TANH 1

/* ---- library / status ------------------------------------------------------ */
const char* mvb_last_error(void);   /* message of the last failing call on this thread */
int mvb_version(void);               /* ABI version */
int mvb_num_sms(int device);         /* SM count of `device` (148 on B200) */
/* Read (and with clear != 0, reset) the device status word of the current device.
 * Synchronises `stream`.  *status receives the OR of MVB_DEV_* bits. */
int mvb_device_status(unsigned int* status, int clear, mvb_stream_t stream);

/* ---- RMSNorm family -------------------------------------------------------
 * Replaces rmsnorm_forward / rmsnorm_plus_one_forward (ops_binding.cpp:11-12,
 * rmsnorm_kernel.cu:153-185).  out/in: [rows, hidden], weight: [hidden].
 * semantics: MVB_NORM_OPS reproduces the ops-API formula of ops/rmsnorm.py:12-31
 * (w*x rounded to the dtype before the 1/rms scale); MVB_NORM_MODEL reproduces
 * RMSNorm.forward of models/model.py:19-25 (x*(1/rms) in fp32, then w*, one rounding).
 * in_stride / out_stride: elements between rows (>= hidden); out may be in.  bf16 calls of more
 * than 256 rows (hidden % 256 == 0, <= 8192, 16-byte aligned rows) run one warp per row: the same
 * per-element rounding, the fp32 sum of squares in another order. */
#define MVB_NORM_OPS 0
#define MVB_NORM_MODEL 1
int mvb_rmsnorm(void* out, int64_t out_stride, const void* in, int64_t in_stride, const void* weight, int64_t rows,
                int64_t hidden, float eps, int plus_one, int semantics, int dtype, mvb_stream_t stream);

/* Replaces fused_add_rmsnorm_forward / ..._plus_one_forward (ops_binding.cpp:13-14,
 * rmsnorm_kernel.cu:187-223): residual += in (in place, rounded to the dtype);
 * out = norm(residual).  Same `semantics` switch as mvb_rmsnorm
 * (ops/rmsnorm.py:34-53 vs. the model's add-then-RMSNorm, model.py:319-322). */
int mvb_fused_add_rmsnorm(void* out, void* residual, const void* in, const void* weight, int64_t rows,
                          int64_t hidden, float eps, int plus_one, int semantics, int dtype, mvb_stream_t stream);

/* Residual add + RMSNorm (model semantics) of a linear layer's output still in split-K partial
 * form (models/model.py:319-322, :328 + the next RMSNorm): `gemm_workspace` is the workspace of
 * the preceding mvb_gemm_bf16(MVB_EPI_PARTIALS) call of shape [rows, hidden, gemm_k];
 * residual += bf16(sum of partials) (in place, bf16), out = RMSNorm(residual).  bf16 only. */
int mvb_fused_add_rmsnorm_gemm(void* out, void* residual, const void* gemm_workspace, int64_t rows, int64_t hidden,
                               int64_t gemm_k, const void* weight, float eps, int plus_one, mvb_stream_t stream);

/* ---- RoPE ------------------------------------------------------------------
 * Replaces rotary_pos_emb_forward (ops_binding.cpp:15, rope_kernel.cu:44-61):
 * NeoX rotate-half RoPE, out = x*cos + rotate_half(x)*sin, each product and the
 * sum rounded to the dtype as the PyTorch path does (ops/rope.py:74-76).
 * in/out/cos/sin: [rows, head_dim]. */
int mvb_rotary_pos_emb(void* out, const void* in, const void* cos, const void* sin, int64_t rows,
                       int64_t head_dim, int dtype, mvb_stream_t stream);

/* ---- activations -------------------------------------------------------------
 * silu_forward / gelu_forward (ops_binding.cpp:16-17, activation_kernel.cu:82-114),
 * swiglu_forward / geglu_forward (:18-19, :116-146), fused_mlp_forward
 * (:25, mlp_kernel.cu:61-93: out[r, j] = act(gate_up[r, j]) * gate_up[r, I + j]).
 * gelu is the tanh approximation (ops/activation.py:28). */
int mvb_activation(void* out, const void* in, int64_t n, int act, int dtype, mvb_stream_t stream);
int mvb_gated_activation(void* out, const void* gate, const void* up, int64_t n, int act, int dtype,
                         mvb_stream_t stream);
int mvb_fused_mlp(void* out, const void* gate_up, int64_t rows, int64_t intermediate, int act, int dtype,
                  mvb_stream_t stream);

/* ---- embedding / softmax -------------------------------------------------------
 * embedding_forward (ops_binding.cpp:23, embedding_kernel.cu:41-65): out[t] = W[ids[t]] * scale.
 * ids: int32 or int64 (ids_dtype); an id outside [0, vocab) yields a zero row and MVB_DEV_BAD_TOKEN.
 * softmax_forward (:24, softmax_kernel.cu:83-100): last-dim softmax, fp32 math. */
int mvb_embedding(void* out, const void* ids, int ids_dtype, const void* weight, int64_t tokens, int64_t hidden,
                  int64_t vocab, float scale, int dtype, mvb_stream_t stream);
int mvb_softmax(void* out, const void* in, int64_t rows, int64_t n, int dtype, mvb_stream_t stream);

/* ---- sampling ------------------------------------------------------------------
 * greedy_sample (ops_binding.cpp:20, sampling_kernel.cu:195-215): row argmax,
 * lowest index among equal maxima (torch.argmax semantics).  out: int64 [rows].
 * top_k_top_p_filter (:21, :218-231): in place; logits outside the top-k
 * (ties at the k-th value kept) and outside the top-p nucleus of the untempered
 * distribution become -inf (ops/sampling.py:26-50).  top_k <= 0 / top_p >= 1 disable.
 * softmax_multinomial_sample (:22, :236-254): temperature-scaled softmax and one
 * draw per row.  The draw is an inverse CDF in vocabulary order with one
 * Philox4x32-10 uniform per row, counter (row, offset, 'SAMP'), key = seed. */
int mvb_greedy_sample(int64_t* out, const void* logits, int64_t rows, int64_t vocab, int64_t row_stride,
                      int dtype, mvb_stream_t stream);
int mvb_top_k_top_p_filter(void* logits, int64_t rows, int64_t vocab, int top_k, float top_p, int dtype,
                           mvb_stream_t stream);
int mvb_softmax_multinomial_sample(int64_t* out, const void* logits, int64_t rows, int64_t vocab,
                                   float temperature, uint64_t seed, uint64_t offset, int dtype,
                                   mvb_stream_t stream);

/* Fused decode sampler (replaces Sampler.sample's per-sequence loop, engine.py:352-356 +
 * sampler.py:21-48): per row, temperature == 0 -> greedy; otherwise top-k, top-p on the
 * untempered logits, /T, softmax, Philox inverse-CDF draw.  Per-row parameters (arrays of
 * `rows`; any may be NULL for "use scalar default": T=1, top_k=-1, top_p=1).
 * probs_out (nullable, fp32 [rows, vocab]): the filtered tempered distribution, for callers
 * that draw with their own generator.  offset_dev (nullable): a device int64 added to
 * `offset` at run time, so a captured CUDA graph draws fresh uniforms on every replay.
 * top_k is limited to 1024; rows with top_k <= 0 and top_p < 1 take the full-vocabulary
 * nucleus path. */
int mvb_sample(int64_t* out, float* probs_out, const void* logits, int64_t rows, int64_t vocab,
               int64_t row_stride, const float* temperature, const int32_t* top_k, const float* top_p,
               uint64_t seed, uint64_t offset, const int64_t* offset_dev, int dtype, mvb_stream_t stream);

/* ---- fused QK-norm + RoPE + paged KV write ---------------------------------
 * Replaces, for one decode step of one layer, the q_norm/k_norm RMSNorm
 * (model.py:174-178), apply_rotary_pos_emb (:184) and Attention._write_kv_cache
 * (:226-243; model_cuda.py:182-207).  qkv: [B, (Hq + 2*Hkv) * D] bf16 (row stride
 * qkv_stride) -- the fused q|k|v projection.  q_norm_w / k_norm_w: [D] bf16 or NULL
 * (no QK-norm); plus_one != 0 scales by (1 + w) in fp32 as Gemma's RMSNorm does
 * (models/gemma3_model.py:14-25).  cos/sin: the model's bf16 tables [table_len, D].  positions: int32 [B]
 * (token position = slot index = cached tokens, engine.py:316/326).  block_tables:
 * int32 [B, max_blocks].  kv_cache: the KVCacheManager tensor
 * [L, 2, num_blocks, block_size, Hkv, D] bf16 (kv_cache.py:24-29).
 * q_out: [B, Hq, D] bf16.  Writes K (normed, roped) and V of each token to
 * (layer, block_tables[b][pos / block_size], pos % block_size). */
int mvb_qk_norm_rope_kv_write(void* q_out, void* kv_cache, const void* qkv, int64_t qkv_stride,
                              const void* q_norm_w, const void* k_norm_w, const void* cos, const void* sin,
                              int64_t table_len, const int32_t* positions, const int32_t* block_tables,
                              int64_t max_blocks, int64_t batch, int64_t num_q_heads, int64_t num_kv_heads,
                              int64_t head_dim, int64_t num_layers, int64_t layer, int64_t num_blocks,
                              int64_t block_size, float eps, int plus_one, mvb_stream_t stream);

/* The same, with the fused q|k|v projection still in split-K partial form: `gemm_workspace`
 * is the workspace of the preceding mvb_gemm_bf16(MVB_EPI_PARTIALS) call of shape
 * [batch, (Hq + 2*Hkv) * head_dim, gemm_k]; each element is taken as bf16(sum of its tile's
 * partials), i.e. exactly the projection's bf16 output (model.py:170-172). */
int mvb_qk_norm_rope_kv_write_gemm(void* q_out, void* kv_cache, const void* gemm_workspace, int64_t gemm_k,
                                   const void* q_norm_w, const void* k_norm_w, const void* cos, const void* sin,
                                   int64_t table_len, const int32_t* positions, const int32_t* block_tables,
                                   int64_t max_blocks, int64_t batch, int64_t num_q_heads, int64_t num_kv_heads,
                                   int64_t head_dim, int64_t num_layers, int64_t layer, int64_t num_blocks,
                                   int64_t block_size, float eps, int plus_one, mvb_stream_t stream);

/* ---- paged attention decode --------------------------------------------------
 * Replaces Attention._read_kv_cache_batch + GQA expand + SDPA for one query token per
 * sequence (model.py:191-221, model_cuda.py:145-177): out[b, h] =
 * softmax(q[b,h] . K[b, :ctx_lens[b]]^T * scale) V, reading K/V straight out of the
 * paged pool through block_tables.  q/out: [B, Hq, D] bf16 (row stride in elements
 * q_stride / out_stride between sequences).  Split-KV across the whole GPU with a
 * deterministic merge.  workspace: >= mvb_paged_attention_workspace_bytes(), zero before
 * the first call (partials at its head, per-sequence counters at its tail, left zero). */
int64_t mvb_paged_attention_workspace_bytes(int64_t batch, int64_t num_q_heads, int64_t head_dim, int device);
int mvb_paged_attention_decode(void* out, int64_t out_stride, const void* q, int64_t q_stride,
                               const void* kv_cache, const int32_t* block_tables, int64_t max_blocks,
                               const int32_t* ctx_lens, int64_t batch, int64_t num_q_heads, int64_t num_kv_heads,
                               int64_t head_dim, int64_t num_layers, int64_t layer, int64_t num_blocks,
                               int64_t block_size, float scale, void* workspace, int64_t workspace_bytes,
                               mvb_stream_t stream);

/* mvb_paged_attention_decode with the Gemma attention variants (Gemma-2/3 decode,
 * models/gemma3_model.py:169-195 for head_dim 256 and the query_pre_attn_scalar scale).
 * softcap > 0: every scaled score s becomes softcap * tanh(s / softcap) before the softmax
 * (Gemma-2's attention logit soft-capping; 0 = off).  window > 0: sequence b attends to its
 * newest `window` keys only, positions [ctx_b - window, ctx_b) (a sliding-window layer;
 * 0 = all keys).  head_dim 128 or 256.  mvb_paged_attention_decode is this call with
 * softcap = 0 and window = 0. */
int mvb_paged_attention_decode_ex(void* out, int64_t out_stride, const void* q, int64_t q_stride,
                                  const void* kv_cache, const int32_t* block_tables, int64_t max_blocks,
                                  const int32_t* ctx_lens, int64_t batch, int64_t num_q_heads, int64_t num_kv_heads,
                                  int64_t head_dim, int64_t num_layers, int64_t layer, int64_t num_blocks,
                                  int64_t block_size, float scale, float softcap, int64_t window, void* workspace,
                                  int64_t workspace_bytes, mvb_stream_t stream);

/* Causal attention of a batched prefill over the paged pool (the prefill's SDPA with
 * is_causal=True, models/model.py:206-221, after Attention._write_kv_cache, :226-243): for every
 * prompt token t of every sequence, out[t, h] = softmax_{k <= t}(q[t, h] . K[k]^T * scale) V[k].
 * q/out: [tokens, Hq, D] bf16 rows (row stride q_stride / out_stride), sequence s occupying rows
 * seq_start[s] .. seq_start[s] + seq_len[s] - 1.  block_tables: int32 [num_seqs, max_blocks].
 * The work is num_tiles (sequence, 16-token query tile) pairs: tile i is query tokens
 * 16 tile_idx[i] .. of sequence tile_seq[i] (tile_idx < ceil(seq_len / 16)); order them longest
 * first.  The tile's K/V prefix is read once for its 16 queries.  head_dim 128, 1, 2 or 4 query
 * heads per KV head, block_size 16. */
int mvb_prefill_attention(void* out, int64_t out_stride, const void* q, int64_t q_stride, const void* kv_cache,
                          const int32_t* block_tables, int64_t max_blocks, const int32_t* seq_start,
                          const int32_t* seq_len, const int32_t* tile_seq, const int32_t* tile_idx,
                          int64_t num_tiles, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                          int64_t num_layers, int64_t layer, int64_t num_blocks, int64_t block_size, float scale,
                          mvb_stream_t stream);

/* Allocation-free paged attention (no counterpart in the reference).  Same arguments and
 * result as mvb_paged_attention_decode, minus the workspace: the split-KV scratch is a
 * 6 MiB area built into the library, for callers that cannot allocate device memory (a host
 * runtime binding this C ABI without a device allocator of its own, or a server whose HBM is
 * all committed to the KV pool and that cannot take cudaMalloc's device-wide sync).
 * Limit: the scratch covers up to 32 query heads of 128 dims on a 148-SM GPU and up to 4096
 * sequences; larger shapes return MVB_ERR_UNSUPPORTED.  The first call on a device looks up
 * the area's device address (cudaGetSymbolAddress), so make that first call before any
 * stream capture.  All calls on a device share the area: each call clears its counters
 * itself, and calls that overlap on the GPU (e.g. on two streams) race.  The looked-up address
 * is kept until the process exits: do not reset a device (cudaDeviceReset) after using this
 * entry point on it. */
int mvb_paged_attention_decode_noalloc(void* out, int64_t out_stride, const void* q, int64_t q_stride,
                                       const void* kv_cache, const int32_t* block_tables, int64_t max_blocks,
                                       const int32_t* ctx_lens, int64_t batch, int64_t num_q_heads,
                                       int64_t num_kv_heads, int64_t head_dim, int64_t num_layers, int64_t layer,
                                       int64_t num_blocks, int64_t block_size, float scale, mvb_stream_t stream);

/* ---- dense GEMM on tcgen05 --------------------------------------------------------
 * Replaces the nn.Linear (cuBLAS) projections of the decode step (model_cuda.py:124-126,
 * :180, ops/mlp.py:66/84, model_cuda.py:413): Y[m, n] = sum_k X[m, k] * W[n, k] (bf16 in,
 * fp32 accumulate in TMEM).  Stream-K over all SMs (two CTAs per SM at m <= 64); partial tiles
 * merged in a fixed order.
 * epilogue: MVB_EPI_STORE  Y = bf16(acc)
 *           MVB_EPI_SWIGLU W is the reference's cat([gate, up]) of 2*inter rows; Y[m, j] =
 *                          bf16(bf16(silu(bf16(gate))) * bf16(up)), j < inter (model.py:116-117)
 *           MVB_EPI_RESADD Y = bf16(aux[m, n] + bf16(acc)) (residual add, model.py:319/328)
 *           MVB_EPI_PARTIALS  no Y (y may be NULL): every stream-K segment leaves its fp32 partial in
 *                          the workspace for a consuming kernel to sum (mvb_fused_add_rmsnorm_gemm,
 *                          mvb_qk_norm_rope_kv_write_gemm); the GEMM then ends without a merge
 *           MVB_EPI_SWIGLU_PARTIALS  the SWIGLU pairing of W's rows with MVB_EPI_PARTIALS' output:
 *                          fp32 partials of gate and up features, finished by mvb_swiglu_gemm
 * Requires k % 64 == 0, ldx/ldw/ldy multiples of 8, 16-byte aligned pointers, m < 2^24.  More
 * than 256 rows (a prefill's tokens) take STORE, SWIGLU or RESADD on one GPU: 256-row tiles, and
 * whole 256 x 256 output tiles (two 128-row weight tiles per activation tile) when the 128-row
 * weight tiles (64-row gate/up pairs for SWIGLU) are even in number.
 * workspace: >= mvb_gemm_workspace_bytes(m, n, k, device); zero before the first call.  fp32
 * partials use its head, per-tile counters its tail; the kernel leaves the counters zero, so
 * one buffer serves any number of calls on one stream.  Calls of different shapes may share
 * a buffer sized for the largest partial area plus the largest counter area among them. */
#define MVB_EPI_STORE 0
#define MVB_EPI_SWIGLU 1
#define MVB_EPI_RESADD 2
#define MVB_EPI_PARTIALS 3
#define MVB_EPI_SWIGLU_PARTIALS 4
int64_t mvb_gemm_workspace_bytes(int64_t m, int64_t n, int64_t k, int device);
int mvb_gemm_bf16(void* y, int64_t ldy, const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t m,
                  int64_t n, int64_t k, int epilogue, const void* aux, int64_t ld_aux, void* workspace,
                  int64_t workspace_bytes, mvb_stream_t stream);

/* The activation of FusedMLP (ops/mlp.py:65-84; mlp_kernel.cu:17-36 with SiLU) applied to a
 * gate_up product still in split-K partial form: `gemm_workspace` is the workspace of the
 * preceding mvb_gemm_bf16(MVB_EPI_SWIGLU_PARTIALS) call of shape [rows, 2 * inter, gemm_k];
 * out[r, j] = bf16(bf16(silu(bf16(gate))) * bf16(up)) for j < inter, the same values
 * MVB_EPI_SWIGLU writes.  Requires inter % 4 == 0, out_stride % 4 == 0, 8-byte aligned out. */
int mvb_swiglu_gemm(void* out, int64_t out_stride, const void* gemm_workspace, int64_t rows, int64_t inter,
                    int64_t gemm_k, mvb_stream_t stream);

/* mvb_swiglu_gemm with the activation chosen: MVB_ACT_SILU (SwiGLU) or MVB_ACT_GELU_TANH
 * (GeGLU: Gemma's down(gelu_tanh(gate(x)) * up(x)), models/gemma3_model.py:104-105;
 * mlp_kernel.cu:17-36 with GELU): out = bf16(bf16(act(bf16(gate))) * bf16(up)). */
int mvb_gated_gemm(void* out, int64_t out_stride, const void* gemm_workspace, int64_t rows, int64_t inter,
                   int64_t gemm_k, int act, mvb_stream_t stream);

/* Post-norm, residual add and RMSNorm of a linear layer's output still in split-K partial
 * form (Gemma's sandwich norms, models/gemma3_model.py:270-283): y = bf16(sum of partials),
 * residual = bf16(residual + RMSNorm(y; post_weight)), out = RMSNorm(residual; weight), both
 * norms in the model's form (plus_one: T((x * r) * (1 + w)), models/gemma3_model.py:21-25).
 * Same arguments and requirements as mvb_fused_add_rmsnorm_gemm plus post_weight [hidden]. */
int mvb_fused_norm_add_rmsnorm_gemm(void* out, void* residual, const void* gemm_workspace, int64_t rows,
                                    int64_t hidden, int64_t gemm_k, const void* post_weight, const void* weight,
                                    float eps, int plus_one, mvb_stream_t stream);

/* ---- fused decoder layer --------------------------------------------------------------
 * Everything of one dense decode layer after its attention, and the next layer's projection,
 * in one persistent launch (DecoderLayer.forward after self_attn, models/model.py:315-328,
 * model_cuda.py:306-321; then Attention.forward's q/k/v projections, QK-norm, RoPE and
 * _write_kv_cache of the next layer, model.py:154-243):
 *   residual += o_proj(attn);  xn = RMSNorm(residual; ln2)
 *   h = silu(gate(xn)) * up(xn)             (wgu = cat([gate, up]), ops/mlp.py:87-121)
 *   residual += down(h);       xn = RMSNorm(residual; ln_next)   (next input norm | final norm)
 *   if wqkv_next: q|k|v = xn W^T, QK-norm (q_norm_next / k_norm_next, or none), RoPE at
 *                 positions, K/V written to (next_layer, block_tables[b][pos/bs], pos%bs), q -> q_out
 * The GEMMs run on tcgen05 with a stream-K split over two CTAs per SM (fp32 partials summed in a
 * fixed order: deterministic); results agree with the unfused kernels to bf16 rounding.  All CTAs
 * are resident and meet at grid barriers; every wait is bounded (MVB_DEV_WAIT_TIMEOUT).
 * Shapes: batch m <= 64, head_dim 128, hidden a multiple of 64 and <= 4096, intermediate a
 * multiple of 64; weights contiguous [n, k] bf16; attn [m, Hq*D] (row stride attn_stride),
 * residual / xn [m, hidden], h [m, inter], q_out [m, Hq, D].
 * workspace: >= mvb_decoder_layer_workspace_bytes(), 256-byte aligned (fp32 partials and
 * per-tile flags).  barrier: 256 bytes, 128-byte aligned.  Zero both before the first call; the
 * calls leave them ready for the next one; calls that share them must be stream-ordered.  After a
 * call that reported MVB_DEV_WAIT_TIMEOUT, zero both again. */
int64_t mvb_decoder_layer_workspace_bytes(int64_t m, int64_t hidden, int64_t q_dim, int64_t inter, int64_t qkv_dim,
                                          int device);
int mvb_decoder_layer_tail(const void* attn, int64_t attn_stride, const void* wo, const void* ln2, const void* wgu,
                           const void* wdown, const void* ln_next, const void* wqkv_next, const void* q_norm_next,
                           const void* k_norm_next, void* residual, void* xn, void* h, void* q_out, void* kv_cache,
                           const void* cos, const void* sin, int64_t table_len, const int32_t* positions,
                           const int32_t* block_tables, int64_t max_blocks, int64_t m, int64_t hidden,
                           int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim, int64_t inter,
                           int64_t num_layers, int64_t next_layer, int64_t num_blocks, int64_t block_size, float eps,
                           void* workspace, int64_t workspace_bytes, void* barrier, mvb_stream_t stream);

/* Logit soft-capping in place (Gemma-2's final_logit_softcapping): x = T(T(tanh(T(x / cap))) * cap),
 * the rounding sequence of `logits / cap; tanh; * cap` in the logits' dtype.  n elements of
 * dtype MVB_BF16 or MVB_F32; cap > 0. */
int mvb_softcap(void* x, int64_t n, float cap, int dtype, mvb_stream_t stream);

/* Input ids of a decode step from the previous step's sampled tokens: ids[i] = tokens[i] for
 * i < n when *feed != 0, nothing otherwise.  ids: int32 [n] (the step metadata's id words),
 * tokens: int64 [n] (the sampler's output), feed: one int32 of the same metadata, read on the
 * device, so a captured step can take either its uploaded ids or the tokens the previous step
 * sampled.  Replaces the host round trip of engine.py:315-317 (the next step's input_ids built
 * from the tokens the last step appended) when the caller runs a step ahead of reading them. */
int mvb_feed_ids(int32_t* ids, const int64_t* tokens, const int32_t* feed, int64_t n, mvb_stream_t stream);

/* ---- sparse mixture of experts (Qwen3-MoE) ---------------------------------------------
 * Replace Qwen3MoeSparseMoe.forward (models/qwen3_moe_model.py:39-65) for one decode step.
 *
 * mvb_moe_route: router logits [rows, E] (bf16, the gate GEMM's output) -> fp32 softmax (the
 * reference's GPU decode runs under CUDA autocast, where softmax computes in fp32), top_k experts
 * per row (ties to the lower expert index), weights renormalised over the top_k when norm_topk.
 * Outputs: topk_ids / topk_w [rows, top_k] (slots in descending probability); the dispatch order
 * of the (row, slot) pairs -- by expert, rows ascending within an expert: pair_row [rows, top_k]
 * (position of each pair), row_token [rows * top_k] (row of each position), expert_off [E + 1]
 * (first position of each expert), active [1 + E] (count of experts with rows, then their ids
 * ascending).  rows <= 256, E <= 256, top_k <= 16.  One CTA. */
int mvb_moe_route(const void* logits, int64_t rows, int64_t num_experts, int64_t top_k, int norm_topk,
                  int32_t* topk_ids, float* topk_w, int32_t* pair_row, int32_t* row_token, int32_t* expert_off,
                  int32_t* active, mvb_stream_t stream);
/* out[r] = x[row_token[r]] for r < nrows (bf16 rows of `hidden`, hidden % 8 == 0). */
int mvb_moe_gather(void* out, const void* x, int64_t hidden, const int32_t* row_token, int64_t nrows,
                   mvb_stream_t stream);
/* Grouped GEMM over the active experts (tcgen05): w = [num_experts, n_per_expert, k] bf16; rows
 * expert_off[e] .. expert_off[e+1]-1 of x (dispatch order, at most max_rows_per_expert <= 256 per
 * expert) are multiplied by expert e's matrix:
 *   MVB_EPI_STORE   y[r, j] = bf16(sum_k x[r, k] w[e, j, k]), j < n_per_expert   (down_proj)
 *   MVB_EPI_SWIGLU  w[e] = cat(gate, up) of 2*inter rows (inter % 64 == 0):
 *                   y[r, j] = bf16(bf16(silu(bf16(gate))) * bf16(up)), j < inter  (gate/up_proj) */
int mvb_moe_gemm_bf16(void* y, int64_t ldy, const void* x, int64_t ldx, const void* w, int64_t n_per_expert,
                      int64_t k, int64_t num_experts, int64_t nrows, int64_t max_rows_per_expert, int epilogue,
                      const int32_t* expert_off, const int32_t* active, mvb_stream_t stream);
/* Expert-parallel form: w holds only experts first_expert .. first_expert + local_experts - 1
 * ([local_experts, n_per_expert, k]); the routing (expert_off, active) still covers all
 * num_experts, and only the dispatched rows of the local experts are computed and stored. */
int mvb_moe_gemm_bf16_experts(void* y, int64_t ldy, const void* x, int64_t ldx, const void* w, int64_t n_per_expert,
                              int64_t k, int64_t num_experts, int64_t first_expert, int64_t local_experts,
                              int64_t nrows, int64_t max_rows_per_expert, int epilogue, const int32_t* expert_off,
                              const int32_t* active, mvb_stream_t stream);
/* out[row] = the reference's accumulation of the row's expert outputs y[pair_row] (bf16 rows of
 * `hidden`): experts in ascending index, acc = bf16(acc + w * y) from acc = 0. */
int mvb_moe_combine(void* out, const void* y, const float* topk_w, const int32_t* topk_ids, const int32_t* pair_row,
                    int64_t rows, int64_t top_k, int64_t hidden, mvb_stream_t stream);
/* Expert-parallel form: only the slots on experts first_expert .. first_expert + local_experts - 1
 * (the ranks' outputs are then summed across the group). */
int mvb_moe_combine_experts(void* out, const void* y, const float* topk_w, const int32_t* topk_ids,
                            const int32_t* pair_row, int64_t rows, int64_t top_k, int64_t hidden,
                            int64_t first_expert, int64_t local_experts, mvb_stream_t stream);

/* ---- tensor parallelism (one process per GPU, NVLink peer memory) ----------------------
 * No counterpart in the reference beyond its stub (distributed/tensor_parallel.py:14-35,
 * tp_size > 1 raises).  These replace the NCCL all-reduce a Megatron-style split of the decode
 * step would need after each row-parallel GEMM, and the all-gather of vocab-parallel logits.
 *
 * Symmetric heap: every rank calls mvb_tp_heap_alloc with the same size (one cudaMalloc,
 * zeroed; the first mvb_tp_signal_bytes() bytes are signal counters), exchanges the 64-byte
 * IPC handles (e.g. with torch.distributed.all_gather_object), then calls mvb_tp_comm_init with
 * all handles in rank order.  Buffers inside the heap are named by byte offset, the same on
 * every rank.  Each step starts with mvb_tp_begin_step (a one-thread kernel that advances
 * this rank's step counter on the device, so a CUDA graph of a step can be replayed), and
 * every rank issues the same sequence of mvb_tp_* calls per step.  A wait for a peer gives up
 * after 2 s and sets MVB_DEV_WAIT_TIMEOUT (the kernel then completes with whatever data
 * arrived).
 *
 * Signal points are small integers (< 1024) chosen by the caller, one per exchange site in a
 * step; a call that waits on a point must come after the call that signals it. */
#define MVB_TP_IPC_HANDLE_BYTES 64
typedef struct mvb_tp_comm mvb_tp_comm;
int64_t mvb_tp_signal_bytes(void);
int mvb_tp_heap_alloc(int64_t bytes, void** base, void* ipc_handle);
int mvb_tp_heap_free(void* base);
int mvb_tp_comm_init(int rank, int nranks, void* local_base, const void* ipc_handles, int64_t heap_bytes,
                     mvb_tp_comm** comm);
int mvb_tp_comm_destroy(mvb_tp_comm* comm);
int mvb_tp_begin_step(mvb_tp_comm* comm, mvb_stream_t stream);

/* Tensor-parallel form of mvb_decoder_layer_tail, one call per rank of the group: the local
 * shards (num_q_heads, num_kv_heads and inter are this rank's; o_proj / down_proj row-parallel,
 * the rest column-parallel) and the exchanges of the per-kernel tensor-parallel step inside the
 * launch -- replaces, per layer, mvb_tp_gemm_bf16 (o_proj push) -> mvb_tp_fused_add_rmsnorm_gemm
 * -> mvb_tp_gemm_bf16 (gate_up) -> mvb_gated_gemm -> mvb_tp_gemm_bf16 (down push) ->
 * mvb_tp_fused_add_rmsnorm_gemm -> mvb_tp_gemm_bf16 (next q|k|v) -> QK-norm/RoPE/KV write.
 *   o_proj and down_proj push their fp32 partials into the receive areas (heap offsets
 *   recv_o_offset / recv_down_offset, sized by mvb_tp_recv_bytes) of the ranks that own the batch
 *   rows (m / nranks each); each owner adds them to its residual rows, normalises them and writes
 *   them into every rank's xn (heap offset xn_offset); signal points 4 * layer .. 4 * layer + 3
 *   (o_proj pushed, rows gathered, down_proj pushed, rows gathered), as the per-kernel step uses
 *   them.  mvb_tp_begin_step must have started the step.  Waits for other ranks give up after
 *   their time limit with MVB_DEV_WAIT_TIMEOUT. */
int mvb_tp_decoder_layer_tail(mvb_tp_comm* comm, int layer, const void* attn, int64_t attn_stride, const void* wo,
                              const void* ln2, const void* wgu, const void* wdown, const void* ln_next,
                              const void* wqkv_next, const void* q_norm_next, const void* k_norm_next, void* residual,
                              int64_t xn_offset, void* h, void* q_out, void* kv_cache, const void* cos,
                              const void* sin, int64_t table_len, const int32_t* positions,
                              const int32_t* block_tables, int64_t max_blocks, int64_t m, int64_t hidden,
                              int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim, int64_t inter,
                              int64_t num_layers, int64_t next_layer, int64_t num_blocks, int64_t block_size,
                              float eps, int64_t recv_o_offset, int64_t recv_down_offset, void* workspace,
                              int64_t workspace_bytes, void* barrier, mvb_stream_t stream);

/* Expert parallelism of the sparse MoE block over the group (Qwen3MoeSparseMoe.forward,
 * models/qwen3_moe_model.py:39-65, with its experts split evenly over the ranks): each rank
 * combines the slots of its experts first_expert .. first_expert + local_experts - 1 for every
 * row (as mvb_moe_combine, ascending expert index, acc = bf16(acc + w * y)) and pushes the fp32
 * partial into the receive area (heap offset recv_offset, mvb_tp_recv_bytes(rows, hidden, 64,
 * nranks) bytes) of the rank that owns the row; then signals `signal_point` once per rank.  The
 * owner's mvb_tp_fused_add_rmsnorm_gemm with gemm_k = 64 adds the ranks' partials.
 * rows % nranks == 0, hidden % 128 == 0. */
int mvb_tp_moe_combine(mvb_tp_comm* comm, const void* y, const float* topk_w, const int32_t* topk_ids,
                       const int32_t* pair_row, int64_t rows, int64_t top_k, int64_t hidden, int64_t first_expert,
                       int64_t local_experts, int64_t recv_offset, int signal_point, mvb_stream_t stream);
/* Bytes of the receive area of a row-parallel (push) GEMM of shape [m, n, k_local]. */
int64_t mvb_tp_recv_bytes(int64_t m, int64_t n, int64_t k, int nranks, int device);
/* The tcgen05 GEMM of mvb_gemm_bf16 with the exchanges of a tensor-parallel step:
 *   wait_point >= 0       X (a local buffer, e.g. inside the heap) is only read after every
 *                         rank signalled wait_point this step;
 *   MVB_EPI_PARTIALS with out_offset >= 0  (row-parallel o_proj / down_proj, model.py:180, :328)
 *                         push: the fp32 split-K partials of batch row b go to the receive area
 *                         at out_offset in the heap of rank b / (m / nranks); then signal_point;
 *   MVB_EPI_STORE with out_offset >= 0  (vocab-parallel lm_head, model_cuda.py:413)
 *                         all-gather: Y (this rank's n columns, row stride ldy) is stored at
 *                         out_offset in every rank's heap; then signal_point;
 *   MVB_EPI_PARTIALS / MVB_EPI_SWIGLU_PARTIALS with out_offset < 0  local partials in
 *                         `workspace`, as mvb_gemm_bf16 (column-parallel q/k/v, gate/up). */
int mvb_tp_gemm_bf16(mvb_tp_comm* comm, const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t m, int64_t n,
                     int64_t k, int epilogue, void* workspace, int64_t workspace_bytes, int64_t out_offset,
                     int64_t ldy, int wait_point, int signal_point, mvb_stream_t stream);
/* The all-reduce + residual add + RMSNorm after a push GEMM of shape [rows, hidden, gemm_k]
 * (model.py:319-322, :328 + the next RMSNorm): for the rows this rank owns, waits for
 * wait_point, sums the pushed partials over ranks, residual += bf16(sum) (the residual of a row
 * is kept by its owner only), and writes RMSNorm(residual) into every rank's [rows, hidden]
 * bf16 buffer at out_offset; then signal_point. */
int mvb_tp_fused_add_rmsnorm_gemm(mvb_tp_comm* comm, void* residual, int64_t rows, int64_t hidden, int64_t gemm_k,
                                  const void* weight, float eps, int plus_one, int64_t recv_offset, int wait_point,
                                  int64_t out_offset, int signal_point, mvb_stream_t stream);
/* The same with Gemma's post-norm (mvb_fused_norm_add_rmsnorm_gemm): the row's summed output is
 * normalised with post_weight before the residual add. */
int mvb_tp_fused_norm_add_rmsnorm_gemm(mvb_tp_comm* comm, void* residual, int64_t rows, int64_t hidden,
                                       int64_t gemm_k, const void* post_weight, const void* weight, float eps,
                                       int plus_one, int64_t recv_offset, int wait_point, int64_t out_offset,
                                       int signal_point, mvb_stream_t stream);
/* Stream-ordered wait (one tiny kernel) until every rank signalled `point` this step. */
int mvb_tp_wait(mvb_tp_comm* comm, int point, mvb_stream_t stream);

/* ---- programmatic dependent launch -------------------------------------------
 * When enabled (default off), kernels of this library are launched with the PDL
 * attribute so that, inside a stream or CUDA graph, a kernel's prologue overlaps the
 * tail of the previous one.  A kernel then reads its step metadata (positions, context
 * lengths, block tables) and constant tables (weights, cos/sin) before it waits for the
 * previous kernel.  With PDL enabled, those inputs must therefore not be written by the
 * kernel launched just before it in the stream when that kernel lets its dependents start
 * early, as every kernel of this library does.  Host copies, and kernels that let
 * dependents start only at their end, are fine.  Returns the previous setting. */
int mvb_set_pdl(int enable);

#ifdef __cplusplus
}
#endif

#endif /* MVB200_H_ */
