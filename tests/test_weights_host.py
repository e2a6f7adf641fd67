"""Weight packing on the CPU: the layouts the GEMM kernels read (``wqkv = cat(q, k, v)``, the
reference's fused-MLP ``cat([gate, up])`` of ``ops/mlp.py:87-121``, experts stacked ``[E, 2I, H]``
with gate rows first), and the streamed-bytes figure the step roofline is taken against."""
import pytest
import torch

from llm_pytorch_inference_b200.configs import get_config
from llm_pytorch_inference_b200.runner import DecodeWeights
from llm_pytorch_inference_b200.weights import canonical_state_dict, stacked_expert_shapes, weight_shapes


@pytest.mark.parametrize("arch", ["qwen3-tiny", "gemma2-tiny", "qwen3-moe-tiny"])
def test_packed_layouts(arch):
    cfg = get_config(arch)
    sd = canonical_state_dict(cfg, 0, torch.float32)
    w = DecodeWeights(cfg, sd, "cpu", torch.bfloat16)
    bf = torch.bfloat16
    for i in range(cfg["num_hidden_layers"]):
        a = f"model.layers.{i}.self_attn."
        assert torch.equal(w.wqkv[i], torch.cat([sd[a + "q_proj.weight"], sd[a + "k_proj.weight"],
                                                 sd[a + "v_proj.weight"]]).to(bf))
        assert torch.equal(w.wo[i], sd[a + "o_proj.weight"].to(bf))
        m = f"model.layers.{i}.mlp."
        if cfg.get("num_experts"):
            E = cfg["num_experts"]
            assert w.egu[i].shape == (E, 2 * cfg["moe_intermediate_size"], cfg["hidden_size"])
            for e in (0, E - 1):
                q = f"{m}experts.{e}."
                assert torch.equal(w.egu[i][e], torch.cat([sd[q + "gate_proj.weight"],
                                                           sd[q + "up_proj.weight"]]).to(bf))
                assert torch.equal(w.edown[i][e], sd[q + "down_proj.weight"].to(bf))
            assert torch.equal(w.router[i], sd[m + "gate.weight"].to(bf))
        else:
            assert torch.equal(w.wgu[i], torch.cat([sd[m + "gate_proj.weight"], sd[m + "up_proj.weight"]]).to(bf))
            assert torch.equal(w.wdown[i], sd[m + "down_proj.weight"].to(bf))
    if cfg.get("tie_word_embeddings"):
        assert w.lm_head is w.embed


def test_stacked_expert_state_dict_keeps_the_stacked_layout():
    cfg = get_config("qwen3-moe-tiny")
    shapes = stacked_expert_shapes(cfg)
    E, I, H = cfg["num_experts"], cfg["moe_intermediate_size"], cfg["hidden_size"]
    assert shapes["model.layers.0.mlp.experts.gate_up_proj.weight"] == (E, 2 * I, H)
    assert shapes["model.layers.0.mlp.experts.down_proj.weight"] == (E, H, I)
    sd = canonical_state_dict(cfg, 0, torch.float32, stacked_experts=True)
    w = DecodeWeights(cfg, sd, "cpu", torch.bfloat16)
    assert torch.equal(w.egu[0], sd["model.layers.0.mlp.experts.gate_up_proj.weight"].to(torch.bfloat16))


def test_streamed_bytes_of_the_qwen3_8b_step():
    """Every layer's matrices and norms, the final norm and lm_head; the embedding table is only
    gathered.  From the shapes alone (no 16 GB allocation): 15.1 GB."""
    cfg = get_config("qwen3-8b")
    shapes = weight_shapes(cfg)
    total = sum(2 * torch.Size(s).numel() for k, s in shapes.items() if k != "model.embed_tokens.weight")
    L, H, V = cfg["num_hidden_layers"], cfg["hidden_size"], cfg["vocab_size"]
    per_layer = 2 * (6144 * H + H * H + 2 * 12288 * H + H * 12288) + 2 * (2 * H + 2 * 128)
    assert total == L * per_layer + 2 * (V * H + H)
    assert 15.1e9 < total < 15.2e9
    # the same figure from the packed weights of a 2-layer model, scaled by layers
    small = get_config("qwen3-tiny")
    w = DecodeWeights(small, canonical_state_dict(small, 0, torch.float32), "cpu", torch.bfloat16)
    s2 = weight_shapes(small)
    assert w.streamed_bytes() == sum(2 * torch.Size(s).numel() for k, s in s2.items()
                                     if k != "model.embed_tokens.weight" or small.get("tie_word_embeddings"))
