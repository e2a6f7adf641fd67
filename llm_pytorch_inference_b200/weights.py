"""Canonical random-init weights with HuggingFace key names.

Every Linear / Embedding weight is drawn N(0, 0.02) in sorted-key order from one
seeded generator, in fp32, then cast; norm weights keep their constructor values
(ones, or zeros for the (1+w) form, ``mini_vllm/models/model.py:10-17``).  The
same seed therefore gives the same tensors to the oracle, the golden-fixture
script and the CUDA path.  The reference's ``Embedding.reset_parameters``
(``mini_vllm/ops/embedding.py:47``) uses the same N(0, 0.02) law.

For the full-size benchmark the draw can run on the GPU instead (``device="cuda"``):
same law, different values, no 33 GB fp32 staging on the host.
"""
from __future__ import annotations

import torch

from .configs import head_dim, num_kv_heads


def weight_shapes(cfg: dict) -> dict[str, tuple[int, ...]]:
    """HF key -> shape for a Llama/Qwen-family decoder (``model.py:120-424``)."""
    H = cfg["hidden_size"]
    hd = head_dim(cfg)
    nq = cfg["num_attention_heads"]
    nkv = num_kv_heads(cfg)
    inter = cfg["intermediate_size"]
    V = cfg["vocab_size"]
    shapes: dict[str, tuple[int, ...]] = {"model.embed_tokens.weight": (V, H), "model.norm.weight": (H,)}
    if not cfg.get("tie_word_embeddings", False):
        shapes["lm_head.weight"] = (V, H)
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}."
        shapes[p + "self_attn.q_proj.weight"] = (nq * hd, H)
        shapes[p + "self_attn.k_proj.weight"] = (nkv * hd, H)
        shapes[p + "self_attn.v_proj.weight"] = (nkv * hd, H)
        shapes[p + "self_attn.o_proj.weight"] = (H, nq * hd)
        if cfg.get("_qk_norm", False):
            shapes[p + "self_attn.q_norm.weight"] = (hd,)
            shapes[p + "self_attn.k_norm.weight"] = (hd,)
        if cfg.get("num_experts"):   # sparse MoE block (qwen3_moe_model.py:23-65)
            E, mi = cfg["num_experts"], cfg["moe_intermediate_size"]
            shapes[p + "mlp.gate.weight"] = (E, H)
            for e in range(E):
                q = f"{p}mlp.experts.{e}."
                shapes[q + "gate_proj.weight"] = (mi, H)
                shapes[q + "up_proj.weight"] = (mi, H)
                shapes[q + "down_proj.weight"] = (H, mi)
        else:
            shapes[p + "mlp.gate_proj.weight"] = (inter, H)
            shapes[p + "mlp.up_proj.weight"] = (inter, H)
            shapes[p + "mlp.down_proj.weight"] = (H, inter)
        shapes[p + "input_layernorm.weight"] = (H,)
        shapes[p + "post_attention_layernorm.weight"] = (H,)
        if cfg.get("_has_feedforward_layernorms"):   # Gemma sandwich norms (gemma3_model.py:265-268)
            shapes[p + "pre_feedforward_layernorm.weight"] = (H,)
            shapes[p + "post_feedforward_layernorm.weight"] = (H,)
    return shapes


def jitter_norms(sd: dict[str, torch.Tensor], seed: int = 1, std: float = 0.1) -> dict[str, torch.Tensor]:
    """Adds seeded N(0, std) noise to every norm weight (in place of their constant init) so that
    parity tests exercise the norm scales; same seed, same values on every side."""
    gen = torch.Generator().manual_seed(seed)
    out = dict(sd)
    for key in sorted(sd):
        if _is_norm(key):
            t = sd[key]
            out[key] = (t.float().cpu() + torch.randn(t.shape, generator=gen) * std).to(t.dtype).to(t.device)
    return out


def _is_norm(key: str) -> bool:
    return key.endswith("norm.weight")


def stacked_expert_shapes(cfg: dict) -> dict[str, tuple[int, ...]]:
    """``weight_shapes`` with each MoE layer's experts stacked: ``mlp.experts.gate_up_proj.weight``
    ``[E, 2I, H]`` (per expert ``cat(gate, up)``) and ``mlp.experts.down_proj.weight`` ``[E, H, I]``."""
    shapes = {k: v for k, v in weight_shapes(cfg).items() if ".mlp.experts." not in k}
    E, mi, H = cfg["num_experts"], cfg["moe_intermediate_size"], cfg["hidden_size"]
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}.mlp.experts."
        shapes[p + "gate_up_proj.weight"] = (E, 2 * mi, H)
        shapes[p + "down_proj.weight"] = (E, H, mi)
    return shapes


def canonical_state_dict(cfg: dict, seed: int = 0, dtype: torch.dtype = torch.float32,
                         device: str | torch.device = "cpu", stacked_experts: bool = False) -> dict[str, torch.Tensor]:
    """Seeded random-init state dict (sorted keys, N(0, 0.02), norms at ones).  With
    ``stacked_experts`` (MoE only) the experts come pre-stacked (``stacked_expert_shapes``): same
    law, different values, and no second copy of the experts when the decode weights are built."""
    plus_one = cfg.get("_rms_norm_plus_one", False)
    shapes = stacked_expert_shapes(cfg) if stacked_experts and cfg.get("num_experts") else weight_shapes(cfg)
    dev = torch.device(device)
    gen = torch.Generator(device=dev).manual_seed(seed)
    out: dict[str, torch.Tensor] = {}
    for key in sorted(shapes):
        shape = shapes[key]
        if _is_norm(key):
            t = torch.zeros(shape, device=dev) if plus_one else torch.ones(shape, device=dev)
            out[key] = t.to(dtype)
        elif dev.type == "cpu":
            t = torch.empty(shape, dtype=torch.float32)
            t.normal_(0.0, 0.02, generator=gen)
            out[key] = t.to(dtype)
        else:
            # GPU draw straight into the target dtype: avoids an fp32 copy of 8B params.
            t = torch.empty(shape, dtype=dtype, device=dev)
            t.normal_(0.0, 0.02, generator=gen)
            out[key] = t
    return out
