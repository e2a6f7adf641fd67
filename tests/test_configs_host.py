"""Per-layer architecture facts on the CPU: the product's helpers (which pick each layer's RoPE
table, attention window and embedding scale on the GPU path) agree with the oracle's own
restatement of the reference (``models/gemma3_model.py:295-320``) for every named architecture,
and the RoPE tables (``models/model.py:28-81``)."""
import math

import pytest
import torch

from llm_pytorch_inference_b200 import configs as C
from oracle import model as om


@pytest.mark.parametrize("name", sorted(C.ARCHS))
def test_layer_facts_match_the_oracle(name):
    cfg = C.get_config(name)
    assert C.is_gemma(cfg) == om.is_gemma(cfg)
    for i in range(cfg["num_hidden_layers"]):
        assert C.layer_rope_theta(cfg, i) == float(om.layer_rope_theta(cfg, i)), (name, i)
        assert C.layer_window(cfg, i) == om.layer_window(cfg, i), (name, i)


@pytest.mark.parametrize("name", sorted(C.ARCHS))
def test_embedding_scale(name):
    cfg = C.get_config(name)
    if not C.is_gemma(cfg):
        assert C.embed_scale(cfg) == 1.0
        return
    s = C.embed_scale(cfg)   # the bf16-rounded sqrt(hidden) a bf16 model multiplies by
    assert s == float(torch.tensor(math.sqrt(cfg["hidden_size"])).to(torch.bfloat16))
    assert abs(s - math.sqrt(cfg["hidden_size"])) <= math.sqrt(cfg["hidden_size"]) * 2 ** -8


def test_gemma2_alternates_sliding_and_global_layers():
    cfg = C.get_config("gemma2-9b")
    w = [C.layer_window(cfg, i) for i in range(cfg["num_hidden_layers"])]
    assert w[0::2] == [cfg["sliding_window"]] * len(w[0::2]) and set(w[1::2]) == {0}


def test_overrides_do_not_leak_between_calls():
    a = C.get_config("qwen3-8b", num_hidden_layers=2)
    b = C.get_config("qwen3-8b")
    assert a["num_hidden_layers"] == 2 and b["num_hidden_layers"] != 2
    with pytest.raises(KeyError):
        C.get_config("no-such-arch")


@pytest.mark.parametrize("head_dim,theta,length", [(128, 1e6, 4200), (256, 10000.0, 9000), (128, 10000.0, 64)])
def test_rope_tables_match_the_oracle(head_dim, theta, length):
    """The cos/sin tables the GPU path uploads (bf16, positions rounded to bf16 as the reference's
    ``model.to(dtype)`` leaves them) equal the oracle's, which the golden fixtures pin."""
    from llm_pytorch_inference_b200.runner import rope_tables

    cos, sin = rope_tables(head_dim, theta, length, torch.bfloat16, "cpu")
    ocos, osin = om.rope_tables(head_dim, theta, length, torch.bfloat16)
    assert torch.equal(cos, ocos) and torch.equal(sin, osin)
