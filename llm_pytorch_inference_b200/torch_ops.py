"""``torch.ops.mini_vllm_ops`` on the sm_100a kernels.

Registers, under the reference's namespace, the 15 schemas of
``csrc/bindings/ops_binding.cpp:10-26`` with the same names and schema strings, plus
the decode-path ops the reference implements in Python / cuBLAS.  Implementations are
registered for the CUDA dispatch key only and call the C ABI (``libmvb200.so``); a CPU
tensor raises.  Importing this module is what a ``mini_vllm`` checkout would do instead
of ``torch.ops.load_library(_C*.pyd)`` (``mini_vllm/ops/_utils.py:20-58``).

As in the reference, ``fused_add_rmsnorm_forward`` updates ``residual`` in place and
``top_k_top_p_filter`` filters ``logits`` in place although their schemas carry no
mutation annotation (kept verbatim for drop-in compatibility; eager use only).
"""
from __future__ import annotations

import torch

from . import _native as N
from . import ops

NAMESPACE = "mini_vllm_ops"

REFERENCE_SCHEMAS = [
    "rmsnorm_forward(Tensor input, Tensor weight, float eps) -> Tensor",
    "rmsnorm_plus_one_forward(Tensor input, Tensor weight, float eps) -> Tensor",
    "fused_add_rmsnorm_forward(Tensor residual, Tensor input, Tensor weight, float eps) -> (Tensor, Tensor)",
    "fused_add_rmsnorm_plus_one_forward(Tensor residual, Tensor input, Tensor weight, float eps) -> (Tensor, Tensor)",
    "rotary_pos_emb_forward(Tensor input, Tensor cos, Tensor sin) -> Tensor",
    "silu_forward(Tensor input) -> Tensor",
    "gelu_forward(Tensor input) -> Tensor",
    "swiglu_forward(Tensor gate, Tensor up) -> Tensor",
    "geglu_forward(Tensor gate, Tensor up) -> Tensor",
    "greedy_sample(Tensor logits) -> Tensor",
    "top_k_top_p_filter(Tensor logits, int top_k, float top_p) -> ()",
    "softmax_multinomial_sample(Tensor logits, float temperature) -> Tensor",
    "embedding_forward(Tensor input_ids, Tensor weight, float scale) -> Tensor",
    "softmax_forward(Tensor input) -> Tensor",
    "fused_mlp_forward(Tensor gate_up, int intermediate_size, int activation) -> Tensor",
]

DECODE_SCHEMAS = [
    "gemm_bf16(Tensor x, Tensor weight, int epilogue, Tensor? aux) -> Tensor",
    "qk_norm_rope_kv_write(Tensor qkv, Tensor(a!) kv_cache, int layer, Tensor positions, Tensor block_tables, "
    "Tensor cos, Tensor sin, int num_q_heads, int num_kv_heads, Tensor? q_norm_w, Tensor? k_norm_w, float eps) "
    "-> Tensor",
    "paged_attention_decode(Tensor q, Tensor kv_cache, int layer, Tensor block_tables, Tensor ctx_lens, "
    "float scale) -> Tensor",
    "fused_sample(Tensor logits, Tensor temperature, Tensor top_k, Tensor top_p, int seed, int offset) -> Tensor",
]


def _rope_rows(input: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    # rope_kernel.cu:44-61 contract: input/cos/sin are [N, head_dim] rows
    N.require_cuda(input, cos, sin)
    x = input.contiguous()
    out = torch.empty_like(x)
    with torch.cuda.device(x.device):
        N.check(N.lib().mvb_rotary_pos_emb(out.data_ptr(), x.data_ptr(), cos.contiguous().data_ptr(),
                                           sin.contiguous().data_ptr(), x.shape[0], x.shape[-1], N.dtype_code(x),
                                           N.stream_handle(x.device)), "rotary_pos_emb")
    return out


def _filter_inplace(logits: torch.Tensor, top_k: int, top_p: float) -> None:
    N.require_cuda(logits)
    if not logits.is_contiguous():
        raise RuntimeError("top_k_top_p_filter: logits must be contiguous")
    V = logits.shape[-1]
    with torch.cuda.device(logits.device):
        N.check(N.lib().mvb_top_k_top_p_filter(logits.data_ptr(), logits.numel() // V, V, int(top_k), float(top_p),
                                               N.dtype_code(logits), N.stream_handle(logits.device)),
                "top_k_top_p_filter")


IMPLS = {
    "rmsnorm_forward": lambda input, weight, eps: ops.rmsnorm(input, weight, eps),
    "rmsnorm_plus_one_forward": lambda input, weight, eps: ops.rmsnorm_plus_one(input, weight, eps),
    "fused_add_rmsnorm_forward": lambda residual, input, weight, eps: ops.fused_add_rmsnorm(residual, input, weight,
                                                                                             eps),
    "fused_add_rmsnorm_plus_one_forward": lambda residual, input, weight, eps: ops.fused_add_rmsnorm_plus_one(
        residual, input, weight, eps),
    "rotary_pos_emb_forward": _rope_rows,
    "silu_forward": ops.silu,
    "gelu_forward": ops.gelu,
    "swiglu_forward": ops.swiglu,
    "geglu_forward": ops.geglu,
    "greedy_sample": ops.greedy_sample,
    "top_k_top_p_filter": _filter_inplace,
    "softmax_multinomial_sample": ops.softmax_multinomial_sample,
    "embedding_forward": lambda input_ids, weight, scale: ops.embedding(input_ids, weight, scale),
    "softmax_forward": lambda input: ops.softmax(input),
    "fused_mlp_forward": ops.fused_mlp_forward,
    "gemm_bf16": lambda x, weight, epilogue, aux: ops.linear(x, weight, epilogue, aux),
    "qk_norm_rope_kv_write": lambda qkv, kv_cache, layer, positions, block_tables, cos, sin, nq, nkv, qn, kn, eps:
        ops.qk_norm_rope_kv_write(qkv, kv_cache, layer, positions, block_tables, cos, sin, nq, nkv, qn, kn, eps),
    "paged_attention_decode": lambda q, kv_cache, layer, block_tables, ctx_lens, scale:
        ops.paged_attention_decode(q, kv_cache, layer, block_tables, ctx_lens, scale),
    "fused_sample": lambda logits, t, k, p, seed, offset: ops.sample(logits, t, k, p, seed, offset),
}

_LIB: torch.library.Library | None = None


def register() -> bool:
    """Defines the namespace and its CUDA implementations once; False if another library
    (e.g. the reference's own ``mini_vllm._C``) already owns the namespace."""
    global _LIB
    if _LIB is not None:
        return True
    try:
        lib = torch.library.Library(NAMESPACE, "DEF")
    except RuntimeError:
        return False
    for schema in REFERENCE_SCHEMAS + DECODE_SCHEMAS:
        lib.define(schema)
    for name, fn in IMPLS.items():
        lib.impl(name, fn, "CUDA")
    _LIB = lib
    return True


register()
