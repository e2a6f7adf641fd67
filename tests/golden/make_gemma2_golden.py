"""Pin the oracle's Gemma-2 features to the transformers implementation of Gemma-2.

The reference (mini_vllm) has no Gemma-2 model: its Gemma 3 (``models/gemma3_model.py``)
has neither attention / final-logit soft-capping nor sliding-window layers.  Those
features are restated in ``oracle/model.py`` from Gemma-2's published definition; this
script runs ``transformers``' ``Gemma2ForCausalLM`` (eager attention, fp32, CPU) on the
``gemma2-tiny`` architecture with the canonical seeded weights and records, for greedy
generation, every step's full logits and token.  Each step is a full forward over the
sequence so far (no KV cache), so the fixture is independent of paging.

Usage:  python tests/golden/make_gemma2_golden.py
Writes tests/golden/gemma2_tiny_hf_f32.pt.
"""
from __future__ import annotations

import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from llm_pytorch_inference_b200.configs import get_config  # noqa: E402
from llm_pytorch_inference_b200.weights import canonical_state_dict, jitter_norms  # noqa: E402

PROMPT_LENS = [40, 51, 9, 70]
STEPS = 12


def hf_model(cfg: dict, sd: dict):
    import transformers
    from transformers import Gemma2Config, Gemma2ForCausalLM

    hc = Gemma2Config(
        vocab_size=cfg["vocab_size"], hidden_size=cfg["hidden_size"], intermediate_size=cfg["intermediate_size"],
        num_hidden_layers=cfg["num_hidden_layers"], num_attention_heads=cfg["num_attention_heads"],
        num_key_value_heads=cfg["num_key_value_heads"], head_dim=cfg["head_dim"], rms_norm_eps=cfg["rms_norm_eps"],
        rope_theta=cfg["rope_theta"], max_position_embeddings=cfg["max_position_embeddings"],
        query_pre_attn_scalar=cfg["query_pre_attn_scalar"], sliding_window=cfg["sliding_window"],
        attn_logit_softcapping=cfg["attn_logit_softcapping"], final_logit_softcapping=cfg["final_logit_softcapping"],
        hidden_activation="gelu_pytorch_tanh", tie_word_embeddings=cfg["tie_word_embeddings"])
    hc._attn_implementation = "eager"
    m = Gemma2ForCausalLM(hc).float().eval()
    missing, unexpected = m.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert all(k == "lm_head.weight" for k in missing) and (missing == [] or cfg["tie_word_embeddings"]), missing
    assert [m.model.layers[i].self_attn.sliding_window for i in range(cfg["num_hidden_layers"])] == \
        [cfg["sliding_window"] if i % 2 == 0 else None for i in range(cfg["num_hidden_layers"])]
    return m, transformers.__version__


def main() -> None:
    torch.manual_seed(0)
    cfg = get_config("gemma2-tiny")
    sd = jitter_norms(canonical_state_dict(cfg, seed=0, dtype=torch.float32))
    model, version = hf_model(cfg, sd)
    g = torch.Generator().manual_seed(13)
    prompts = [torch.randint(0, cfg["vocab_size"], (n,), generator=g).tolist() for n in PROMPT_LENS]
    tokens, logits = [], []
    with torch.no_grad():
        for p in prompts:
            seq = list(p)
            rows = []
            for _ in range(STEPS):
                out = model(input_ids=torch.tensor([seq]), use_cache=False).logits[0, -1].float()
                rows.append(out)
                seq.append(int(torch.argmax(out)))
            tokens.append(seq[len(p):])
            logits.append(torch.stack(rows))
    fx = {"arch": "gemma2-tiny", "transformers": version, "prompts": [torch.tensor(p) for p in prompts],
          "tokens": torch.tensor(tokens), "logits": torch.stack(logits)}   # [B, STEPS, V]
    torch.save(fx, HERE / "gemma2_tiny_hf_f32.pt")
    print("gemma2_tiny_hf_f32.pt written, transformers", version, "tokens", fx["tokens"][:, :6].tolist())


if __name__ == "__main__":
    main()
