"""Model architectures served by the decode path, as HuggingFace-style config dicts.

The keys follow the ``config.json`` fields the reference's loader reads
(``mini_vllm/models/loader.py:232-266``) plus the private ``_qk_norm`` flag that
the reference auto-detects from checkpoint keys (``loader.py:137-141``).  With
random-init weights there is no checkpoint to detect from, so the flag is set
explicitly for the Qwen3 family.
"""
from __future__ import annotations

import copy

_QWEN3_COMMON = {
    "model_type": "qwen3",
    "hidden_act": "silu",
    "attention_bias": False,
    "rms_norm_eps": 1e-6,
    "rope_theta": 1000000.0,
    "max_position_embeddings": 40960,
    "head_dim": 128,
    "_qk_norm": True,
}

ARCHS: dict[str, dict] = {
    # Qwen3-0.6B architecture: CPU plumbing workload (fp32, 4x128 prompts, greedy 64).
    "qwen3-0.6b": {
        **_QWEN3_COMMON,
        "num_hidden_layers": 28,
        "hidden_size": 1024,
        "num_attention_heads": 16,
        "num_key_value_heads": 8,
        "intermediate_size": 3072,
        "vocab_size": 151936,
        "tie_word_embeddings": True,
    },
    # Qwen3-8B architecture: the headline decode workload (bf16, batch 64, context 2048).
    "qwen3-8b": {
        **_QWEN3_COMMON,
        "num_hidden_layers": 36,
        "hidden_size": 4096,
        "num_attention_heads": 32,
        "num_key_value_heads": 8,
        "intermediate_size": 12288,
        "vocab_size": 151936,
        "tie_word_embeddings": False,
    },
    # Llama-3-8B architecture (no QK-norm, theta 5e5).
    "llama3-8b": {
        "model_type": "llama",
        "hidden_act": "silu",
        "attention_bias": False,
        "rms_norm_eps": 1e-5,
        "rope_theta": 500000.0,
        "max_position_embeddings": 8192,
        "head_dim": 128,
        "num_hidden_layers": 32,
        "hidden_size": 4096,
        "num_attention_heads": 32,
        "num_key_value_heads": 8,
        "intermediate_size": 14336,
        "vocab_size": 128256,
        "tie_word_embeddings": False,
    },
    # Small Qwen3-family shapes used by the parity tests (head_dim stays 128, the
    # kernels' native width; vocab is cut so the CPU oracle finishes in seconds).
    "qwen3-tiny": {
        **_QWEN3_COMMON,
        "num_hidden_layers": 2,
        "hidden_size": 512,
        "num_attention_heads": 8,
        "num_key_value_heads": 4,
        "intermediate_size": 1024,
        "vocab_size": 4096,
        "tie_word_embeddings": False,
    },
    "qwen3-8b-2l": None,  # filled below: Qwen3-8B dims with 2 layers
    # Qwen3-30B-A3B architecture: sparse MoE MLP (qwen3_moe_model.py), 128 experts, top-8.
    "qwen3-30b-a3b": {
        **_QWEN3_COMMON,
        "model_type": "qwen3_moe",
        "num_hidden_layers": 48,
        "hidden_size": 2048,
        "num_attention_heads": 32,
        "num_key_value_heads": 4,
        "intermediate_size": 6144,
        "moe_intermediate_size": 768,
        "num_experts": 128,
        "num_experts_per_tok": 8,
        "norm_topk_prob": True,
        "vocab_size": 151936,
        "tie_word_embeddings": False,
    },
    # Small MoE shapes for the parity tests.
    "qwen3-moe-tiny": {
        **_QWEN3_COMMON,
        "model_type": "qwen3_moe",
        "num_hidden_layers": 2,
        "hidden_size": 512,
        "num_attention_heads": 8,
        "num_key_value_heads": 2,
        "intermediate_size": 1024,
        "moe_intermediate_size": 128,
        "num_experts": 16,
        "num_experts_per_tok": 4,
        "norm_topk_prob": True,
        "vocab_size": 4096,
        "tie_word_embeddings": False,
    },
}

_GEMMA_COMMON = {
    "hidden_act": "gelu_new",                  # tanh GELU (loader.py:149-157 maps gelu_pytorch_tanh)
    "hidden_activation": "gelu_pytorch_tanh",
    "rms_norm_eps": 1e-6,
    "head_dim": 256,
    "query_pre_attn_scalar": 256,
    "_rms_norm_plus_one": True,               # (1 + w) norms, zero-initialised
    "_has_feedforward_layernorms": True,      # pre/post feed-forward norms (loader.py:143-147)
}

# Gemma-2-9B architecture: alternating 4096-token sliding-window / global layers (even layers
# slide), attention logits soft-capped at 50 and final logits at 30, no QK-norm, one RoPE theta.
ARCHS["gemma2-9b"] = {
    **_GEMMA_COMMON,
    "model_type": "gemma2",
    "num_hidden_layers": 42,
    "hidden_size": 3584,
    "num_attention_heads": 16,
    "num_key_value_heads": 8,
    "intermediate_size": 14336,
    "vocab_size": 256000,
    "rope_theta": 10000.0,
    "max_position_embeddings": 8192,
    "sliding_window": 4096,
    "attn_logit_softcapping": 50.0,
    "final_logit_softcapping": 30.0,
    "tie_word_embeddings": True,
    "_qk_norm": False,
}
# Small Gemma-2 shapes for the parity tests: 4 layers (2 sliding, 2 global), a 32-token window,
# an untied lm_head (tied random weights mostly echo the input token).
ARCHS["gemma2-tiny"] = {
    **ARCHS["gemma2-9b"],
    "num_hidden_layers": 4,
    "hidden_size": 512,
    "num_attention_heads": 4,
    "num_key_value_heads": 2,
    "intermediate_size": 1024,
    "vocab_size": 4096,
    "sliding_window": 32,
    "tie_word_embeddings": False,
}
# The reference's own Gemma 3 model (models/gemma3_model.py, model_type gemma3_text): QK-norm,
# local/global RoPE theta every `sliding_window_pattern` layers, no soft-capping and no window.
ARCHS["gemma3-tiny"] = {
    **_GEMMA_COMMON,
    "model_type": "gemma3_text",
    "num_hidden_layers": 2,
    "hidden_size": 512,
    "num_attention_heads": 4,
    "num_key_value_heads": 2,
    "intermediate_size": 1024,
    "vocab_size": 4096,
    "rope_theta": 1000000.0,
    "rope_local_base_freq": 10000.0,
    "sliding_window_pattern": 2,
    "max_position_embeddings": 32768,
    "tie_word_embeddings": False,
    "_qk_norm": True,
}
ARCHS["qwen3-8b-2l"] = {**ARCHS["qwen3-8b"], "num_hidden_layers": 2}
ARCHS["gemma2-9b-2l"] = {**ARCHS["gemma2-9b"], "num_hidden_layers": 2}


def get_config(name: str, **overrides) -> dict:
    """Return a fresh copy of a named architecture, with optional overrides."""
    if name not in ARCHS:
        raise KeyError(f"unknown architecture {name!r}; known: {sorted(ARCHS)}")
    cfg = copy.deepcopy(ARCHS[name])
    cfg.update(overrides)
    return cfg


def is_gemma(cfg: dict) -> bool:
    """Gemma-family decoder: (1 + w) sandwich norms, GeGLU, sqrt(hidden) embedding scale."""
    return cfg.get("model_type") in ("gemma2", "gemma3_text")


def layer_rope_theta(cfg: dict, i: int) -> float:
    """RoPE base of layer i: Gemma 3 uses the global theta on every ``sliding_window_pattern``-th
    layer and the local one elsewhere (models/gemma3_model.py:307-320); the rest use one theta."""
    if cfg.get("model_type") == "gemma3_text":
        pattern = cfg.get("sliding_window_pattern", 6)
        glob = i % pattern == pattern - 1
        return float(cfg.get("rope_theta", 1000000.0)) if glob else float(cfg.get("rope_local_base_freq", 10000.0))
    return float(cfg.get("rope_theta", 10000.0))


def layer_window(cfg: dict, i: int) -> int:
    """Sliding window of layer i (0 = global): Gemma-2 alternates, even layers sliding."""
    if cfg.get("model_type") == "gemma2" and cfg.get("sliding_window"):
        return int(cfg["sliding_window"]) if i % 2 == 0 else 0
    return 0


def embed_scale(cfg: dict) -> float:
    """Embedding multiplier: sqrt(hidden) for Gemma (models/gemma3_model.py:295-299), else 1.  The
    reference keeps it in a buffer that ``model.to(dtype)`` casts, so a bf16 model multiplies by
    bf16(sqrt(hidden)); the value returned here is that bf16-rounded one."""
    if not is_gemma(cfg):
        return 1.0
    import torch

    return float(torch.tensor(float(cfg["hidden_size"]) ** 0.5).to(torch.bfloat16))


def head_dim(cfg: dict) -> int:
    return cfg.get("head_dim", cfg["hidden_size"] // cfg["num_attention_heads"])


def num_kv_heads(cfg: dict) -> int:
    return cfg.get("num_key_value_heads", cfg["num_attention_heads"])
