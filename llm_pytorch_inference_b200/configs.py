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

ARCHS["qwen3-8b-2l"] = {**ARCHS["qwen3-8b"], "num_hidden_layers": 2}


def get_config(name: str, **overrides) -> dict:
    """Return a fresh copy of a named architecture, with optional overrides."""
    if name not in ARCHS:
        raise KeyError(f"unknown architecture {name!r}; known: {sorted(ARCHS)}")
    cfg = copy.deepcopy(ARCHS[name])
    cfg.update(overrides)
    return cfg


def head_dim(cfg: dict) -> int:
    return cfg.get("head_dim", cfg["hidden_size"] // cfg["num_attention_heads"])


def num_kv_heads(cfg: dict) -> int:
    return cfg.get("num_key_value_heads", cfg["num_attention_heads"])
