"""Generate the golden fixtures under tests/golden/ by running the reference itself.

Runs the unmodified reference (``mini_vllm``) on this machine's CPU through its
PyTorch path (``MINI_VLLM_BACKEND=pytorch``, ``mini_vllm/ops/_utils.py:74``):

* ``ops_golden.pt``    -- the reference ops' PyTorch fallbacks on seeded inputs
  (rmsnorm family ``ops/rmsnorm.py:12-42``, RoPE ``ops/rope.py`` + the model's
  bf16 cos/sin tables ``models/model.py:28-81``, embedding, softmax, activations,
  FusedMLP fallback, greedy / top-k / top-p / softmax sampling ``ops/sampling.py``).
* ``kv_golden.json``   -- KVCacheManager traces (``engine/kv_cache.py:6-81``):
  block tables under a shuffled pool, exhaustion, growth.
* ``decode_qwen3_0.6b_f32.pt`` -- Qwen3-0.6B-architecture fp32 greedy generation through
  ``LLMEngine._step`` (``engine/engine.py:241-360``): 4 prompts x 128 ids, 64 tokens.
* ``decode_qwen3_0.6b_bf16.pt`` -- the same model, prompts and engine path in bf16: greedy,
  33 tokens (the prefill's token and 32 decode steps), top-16 logits of every step.
* ``decode_tiny_bf16.pt`` -- a 2-layer Qwen3-family bf16 model, ragged prompts,
  greedy 24 tokens, full per-step logits.
* ``engine_trace.json`` -- continuous batching through ``LLMEngine._step``: sequences finishing
  at different steps (max_tokens, a stop id), joining mid-run, one that cannot be allocated;
  per-step decoded rows, tokens, block tables, free list and finished set.
* ``decode_moe_tiny_f32.pt`` -- a 2-layer Qwen3-MoE model (``models/qwen3_moe_model.py``,
  16 experts, top-4) in fp32: its MoE block alone, and greedy decoding with full logits.
* ``decode_gemma3_tiny.pt`` -- the reference's Gemma 3 model (``models/gemma3_model.py``, head
  dim 256, QK-norm, local/global RoPE theta) with seeded non-trivial norm weights: greedy
  decoding in fp32 and in bf16, full logits.

Usage (only where the reference is mounted; its checkout path is required):
    python tests/golden/make_golden.py --reference <path to the reference checkout> [--only name,...]
    (or set MINI_VLLM_REFERENCE to that path)

The reference cannot travel with the repository; the fixtures it produced are
committed, and this script is how they were made.
"""
from __future__ import annotations

import argparse
import json
import os
import random
import sys
from collections import deque
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from llm_pytorch_inference_b200.configs import get_config, head_dim, num_kv_heads  # noqa: E402
from llm_pytorch_inference_b200.weights import canonical_state_dict, jitter_norms  # noqa: E402


def _import_reference(path: str):
    os.environ["MINI_VLLM_BACKEND"] = "pytorch"
    sys.path.insert(0, path)
    import mini_vllm  # noqa: F401
    from mini_vllm.ops._utils import is_ext_loaded
    assert not is_ext_loaded(), "reference must run its PyTorch path"


# --------------------------------------------------------------------------- ops
def make_ops_golden() -> dict:
    import importlib
    R = importlib.import_module("mini_vllm.ops.rmsnorm")
    S = importlib.import_module("mini_vllm.ops.sampling")
    E = importlib.import_module("mini_vllm.ops.embedding")
    A = importlib.import_module("mini_vllm.ops.activation")
    SM = importlib.import_module("mini_vllm.ops.softmax")
    from mini_vllm.ops.mlp import FusedMLP
    from mini_vllm.models.model import RotaryEmbedding, apply_rotary_pos_emb

    g = torch.Generator().manual_seed(1234)
    out: dict[str, torch.Tensor] = {}

    def rn(*shape, dtype=torch.bfloat16, scale=1.0):
        return (torch.randn(*shape, generator=g) * scale).to(dtype)

    for dt, tag in ((torch.bfloat16, "bf16"), (torch.float32, "f32")):
        x = rn(6, 4096, dtype=dt)
        w = (1.0 + 0.1 * torch.randn(4096, generator=g)).to(dt)
        res = rn(6, 4096, dtype=dt)
        out[f"rms_x_{tag}"], out[f"rms_w_{tag}"], out[f"rms_res_{tag}"] = x, w, res
        out[f"rmsnorm_{tag}"] = R.rmsnorm(x, w, 1e-6)
        out[f"rmsnorm_p1_{tag}"] = R.rmsnorm_plus_one(x, w, 1e-6)
        y, r = R.fused_add_rmsnorm(res.clone(), x, w, 1e-6)
        out[f"fadd_y_{tag}"], out[f"fadd_r_{tag}"] = y, r
        y, r = R.fused_add_rmsnorm_plus_one(res.clone(), x, w, 1e-6)
        out[f"fadd_p1_y_{tag}"], out[f"fadd_p1_r_{tag}"] = y, r

    # RoPE with the model's own cos/sin cache, cast to bf16 like model.to(bf16) does.
    rope = RotaryEmbedding(128, base=1000000.0).to(torch.bfloat16)
    positions = torch.tensor([[0], [1], [17], [2047], [2048], [2049], [2300], [4095]], dtype=torch.long)
    cos, sin = rope(positions)
    cos_p, sin_p = cos[positions].unsqueeze(1), sin[positions].unsqueeze(1)  # [B,1,1,128]
    q = rn(8, 32, 1, 128)
    k = rn(8, 8, 1, 128)
    qe, ke = apply_rotary_pos_emb(q, k, cos_p, sin_p)
    rows = torch.cat([torch.arange(0, 256), positions[:, 0]])
    out.update(rope_positions=positions, rope_table_rows=rows, rope_cos_rows=cos[rows], rope_sin_rows=sin[rows],
               rope_table_len=torch.tensor(cos.shape[0]), rope_q=q, rope_k=k, rope_q_out=qe, rope_k_out=ke)

    ids = torch.randint(0, 1000, (7,), generator=g)
    W = rn(1000, 256)
    out.update(emb_ids=ids, emb_w=W, emb_out=E.embedding(ids, W, 1.0), emb_out_scaled=E.embedding(ids, W, 2.5))

    sx = rn(5, 3000, dtype=torch.float32, scale=3.0)
    out.update(softmax_x=sx, softmax_out=SM.softmax(sx))
    ax = rn(4, 1000)
    ay = rn(4, 1000)
    out.update(act_x=ax, act_y=ay, silu=A.silu(ax), gelu=A.gelu(ax), swiglu=A.swiglu(ax, ay), geglu=A.geglu(ax, ay))

    mlp = FusedMLP(256, 384, "silu").to(torch.bfloat16)
    with torch.no_grad():
        mlp.gate_up_proj.weight.copy_(rn(768, 256, scale=0.05))
        mlp.down_proj.weight.copy_(rn(256, 384, scale=0.05))
        mx = rn(3, 256)
        out.update(mlp_x=mx, mlp_gate_up_w=mlp.gate_up_proj.weight.detach().clone(),
                   mlp_down_w=mlp.down_proj.weight.detach().clone(), mlp_out=mlp(mx))

    # Sampling: logits are bf16-rounded then .float(), as engine.py:353 hands them to the sampler.
    V = 151936
    logits = (torch.randn(4, V, generator=g) * 1.3).to(torch.bfloat16).float()
    logits[1, 500] = logits[1].max() + 1.0      # a clear winner
    logits[2, 10:14] = logits[2].max() + 0.5    # exact ties: argmax keeps the first index
    out["samp_logits_bf16"] = logits.to(torch.bfloat16)   # exact: the values are bf16-rounded
    out["greedy"] = S.greedy_sample(logits)
    # Filters either keep a logit unchanged or set it to -inf: store the kept indices per row.
    for k_, p_ in ((50, 0.95), (50, 1.0), (0, 0.9), (1, 1.0), (5, 0.5)):
        filt = S.top_k_top_p_filter(logits, k_, p_)
        kept = torch.isfinite(filt)
        assert torch.equal(filt[kept], logits[kept])
        out[f"filter_k{k_}_p{int(p_ * 100)}_kept_bits"] = torch.from_numpy(np.packbits(kept.numpy(), axis=-1))
    filt = S.top_k_top_p_filter(logits, 50, 0.95)
    probs = S.torch.softmax(filt / 0.8, dim=-1)
    for r in range(logits.shape[0]):
        nz = probs[r].nonzero()[:, 0]
        out[f"probs_t08_k50_p95_row{r}_idx"] = nz
        out[f"probs_t08_k50_p95_row{r}_val"] = probs[r, nz]
    return out


# ----------------------------------------------------------------------- kv cache
def make_kv_golden() -> dict:
    from mini_vllm.engine.kv_cache import KVCacheManager

    traces = {}
    kv = KVCacheManager(num_blocks=64, block_size=16, num_layers=1, num_heads=1, head_dim=8, device="cpu")
    order = list(range(64))
    random.Random(0).shuffle(order)
    kv.free_blocks = deque(order)
    log = []
    def snap(bt):  # allocate() returns the live table that append_token() later grows
        return None if bt is None else list(bt)

    for sid, n in enumerate([200, 17, 16]):
        log.append(["allocate", sid, n, snap(kv.allocate(sid, n))])
    for step in range(40):
        for sid in range(3):
            ok = kv.append_token(sid)
            log.append(["append", sid, ok, list(kv.get_block_table(sid))])
    kv.free(1)
    log.append(["free", 1, list(kv.free_blocks)])
    log.append(["allocate", 3, 100, snap(kv.allocate(3, 100))])
    log.append(["allocate", 4, 2000, snap(kv.allocate(4, 2000))])   # exhaustion -> None
    traces["shuffled_pool"] = {"order": order, "log": log, "free_end": list(kv.free_blocks)}
    return traces


# ------------------------------------------------------------------------- decode
def _build_reference_engine(cfg: dict, dtype: torch.dtype, num_blocks: int, pool_seed: int = 0,
                            norm_jitter: int | None = None):
    from mini_vllm.models.loader import _ensure_builtin_models, _BUILTIN_MODELS
    from mini_vllm.engine.engine import LLMEngine
    from mini_vllm.engine.kv_cache import KVCacheManager
    from mini_vllm.engine.scheduler import Scheduler
    from mini_vllm.engine.sampler import Sampler
    from mini_vllm.utils.config import EngineConfig

    _ensure_builtin_models()
    model = _BUILTIN_MODELS[cfg["model_type"]](dict(cfg))
    sd = canonical_state_dict(cfg, seed=0, dtype=torch.float32)
    if norm_jitter is not None:
        sd = jitter_norms(sd, norm_jitter)
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert all(k == "lm_head.weight" for k in missing), missing
    model = model.to(dtype=dtype).eval()

    eng = LLMEngine.__new__(LLMEngine)
    eng.config = EngineConfig(model_path="synthetic", device="cpu",
                              dtype={torch.float32: "float32", torch.bfloat16: "bfloat16"}[dtype])
    eng.model = model
    eng.device = "cpu"
    eng._torch_dtype = dtype
    eng.kv_cache = KVCacheManager(num_blocks=num_blocks, block_size=16, num_layers=cfg["num_hidden_layers"],
                                  num_heads=num_kv_heads(cfg), head_dim=head_dim(cfg), device="cpu", dtype=dtype)
    order = list(range(num_blocks))
    random.Random(pool_seed).shuffle(order)
    eng.kv_cache.free_blocks = deque(order)
    eng.scheduler = Scheduler(eng.config)
    eng.sampler = Sampler()
    eng.eos_token_ids = []
    return eng


class _Recorder(torch.nn.Module):
    def __init__(self, inner):
        super().__init__()
        self.inner = inner
        self.calls = []

    def forward(self, input_ids, positions, **kw):
        logits = self.inner(input_ids, positions, **kw)
        self.calls.append({
            "input_ids": input_ids.clone(), "positions": positions.clone(),
            "block_tables": kw.get("block_tables"), "slot_idx": kw.get("slot_idx"),
            "use_cache": kw.get("use_cache"), "logits": logits[:, -1, :].float().clone(),
        })
        return logits


def run_reference_decode(cfg, dtype, prompts, max_tokens, num_blocks=256, norm_jitter=None):
    from mini_vllm.engine.sequence import Sequence
    from mini_vllm.utils.config import SamplingParams

    eng = _build_reference_engine(cfg, dtype, num_blocks, norm_jitter=norm_jitter)
    rec = _Recorder(eng.model)
    eng.model = rec
    seqs = []
    for i, p in enumerate(prompts):
        s = Sequence(prompt_token_ids=list(p), sampling_params=SamplingParams(temperature=0.0, max_tokens=max_tokens),
                     seq_id=i)
        s.set_stop_conditions([])
        eng.scheduler.add_sequence(s)
        seqs.append(s)
    with torch.no_grad():
        while eng.scheduler.has_unfinished:
            eng._step()
    return seqs, rec.calls


def _decode_fixture(cfg, dtype, prompts, max_tokens, keep_full_logits, norm_jitter=None):
    seqs, calls = run_reference_decode(cfg, dtype, prompts, max_tokens, norm_jitter=norm_jitter)
    prefill = [c for c in calls if not c["use_cache"]]
    decode = [c for c in calls if c["use_cache"]]
    fx: dict = {
        "prompts": [torch.tensor(p, dtype=torch.long) for p in prompts],
        "output_tokens": torch.tensor([s.get_output_token_ids() for s in seqs], dtype=torch.long),
        "prefill_logits_top": torch.stack([torch.topk(c["logits"][0], 16).values for c in prefill]),
        "prefill_logits_top_idx": torch.stack([torch.topk(c["logits"][0], 16).indices for c in prefill]),
        "decode_positions": torch.stack([c["positions"][:, 0] for c in decode]),
        "decode_slot_idx": torch.tensor([c["slot_idx"] for c in decode], dtype=torch.long),
        "decode_block_tables": json.dumps([c["block_tables"] for c in decode]),
        "decode_input_ids": torch.stack([c["input_ids"][:, 0] for c in decode]),
    }
    L = torch.stack([c["logits"] for c in decode])  # [steps, B, V]
    fx["decode_logits_top"] = torch.topk(L, 16, dim=-1).values
    fx["decode_logits_top_idx"] = torch.topk(L, 16, dim=-1).indices
    fx["decode_logits_sum"] = L.double().sum(-1)
    fx["decode_logits_sumsq"] = L.double().pow(2).sum(-1)
    fx["decode_logits_head"] = L[..., :256].clone()
    if keep_full_logits:
        fx["decode_logits"] = L.to(torch.bfloat16) if dtype == torch.bfloat16 else L
    return fx


def make_engine_trace_golden() -> dict:
    """Continuous batching through the reference's ``LLMEngine._step`` (``engine/engine.py:241-360``,
    ``engine/scheduler.py:27-57``): qwen3-tiny in fp32 on a shuffled 20-block pool, sequences
    finishing at different steps (each its own ``max_tokens``, one with a stop id that it
    generates), two sequences joining while others run, one whose prompt does not fit.  After
    every ``_step`` the trace records the prefilled sequences with their first tokens, the decoded
    sequences in batch order with their tokens and block tables, the free list and the finished
    set."""
    from mini_vllm.engine.sequence import Sequence
    from mini_vllm.utils.config import SamplingParams

    cfg = get_config("qwen3-tiny")
    g = torch.Generator().manual_seed(23)
    lens = [37, 50, 16, 64, 20, 33, 400]
    prompts = [torch.randint(0, cfg["vocab_size"], (n,), generator=g).tolist() for n in lens]
    max_toks = [3, 9, 5, 14, 6, 8, 4]
    joins = {0: [0, 1, 2, 3], 4: [4, 5, 6]}      # _step index -> sequences added before it

    def run(stop: dict[int, list[int]]):
        eng = _build_reference_engine(cfg, torch.float32, num_blocks=20, pool_seed=3)
        seqs = {}
        trace = []
        cur = {}
        orig_prefill, orig_decode = eng._run_prefill, eng._run_decode

        def rec_prefill(seq):
            orig_prefill(seq)
            cur["prefill"].append([seq.seq_id, seq.token_ids[-1] if seq.output_len else None])

        model = eng.model

        def forward(input_ids, positions, **kw):      # the tables the decode forward is given
            if kw.get("use_cache"):
                cur["block_tables"] = [list(t) for t in kw["block_tables"]]
                cur["slot_idx"] = list(kw["slot_idx"])
            return model(input_ids, positions, **kw)

        def rec_decode(batch):
            before = {q.seq_id: q.output_len for q in batch}
            orig_decode(batch)
            cur["decode"] = [q.seq_id for q in batch if q.output_len > before[q.seq_id]]
            cur["decode_tokens"] = {str(q.seq_id): q.token_ids[-1] for q in batch if q.output_len > before[q.seq_id]}

        eng.model = forward

        eng._run_prefill, eng._run_decode = rec_prefill, rec_decode
        step = 0
        with torch.no_grad():
            while step == 0 or eng.scheduler.has_unfinished or step in joins:
                for i in joins.get(step, []):
                    q = Sequence(prompt_token_ids=prompts[i], seq_id=i,
                                 sampling_params=SamplingParams(temperature=0.0, max_tokens=max_toks[i]))
                    q.set_stop_conditions(stop.get(i, []))
                    eng.scheduler.add_sequence(q)
                    seqs[i] = q
                cur.clear()
                cur.update(prefill=[], decode=[], block_tables=[], slot_idx=[], decode_tokens={})
                eng._step()
                cur["free_after"] = list(eng.kv_cache.free_blocks)
                cur["finished_after"] = sorted(i for i, q in seqs.items() if q.is_finished())
                trace.append(dict(cur))
                step += 1
        return trace, {i: q.token_ids[q.prompt_len:] for i, q in seqs.items()}

    _, dry = run({})
    stop_tok = dry[3][5]            # sequence 3 stops at its first occurrence of its 6th token
    trace, outs = run({3: [stop_tok]})
    return {"arch": "qwen3-tiny", "num_blocks": 20, "pool_seed": 3, "prompts": prompts, "max_tokens": max_toks,
            "stop": {"3": [stop_tok]}, "joins": {str(k): v for k, v in joins.items()}, "trace": trace,
            "outputs": {str(k): v for k, v in outs.items()}}


def make_moe_golden() -> dict:
    """The reference's sparse-MoE model (``models/qwen3_moe_model.py``) in fp32: the MoE block of
    layer 0 on seeded hidden states, and greedy decoding through ``LLMEngine._step`` (the engine
    picks the model class by ``model_type`` = ``qwen3_moe``)."""
    from mini_vllm.models.qwen3_moe_model import Qwen3MoeSparseMoe

    cfg = get_config("qwen3-moe-tiny")
    sd = canonical_state_dict(cfg, seed=0, dtype=torch.float32)
    block = Qwen3MoeSparseMoe(dict(cfg))
    pre = "model.layers.0.mlp."
    block.load_state_dict({k[len(pre):]: v for k, v in sd.items() if k.startswith(pre)}, strict=True)
    g = torch.Generator().manual_seed(5)
    x = torch.randn(1, 6, cfg["hidden_size"], generator=g)
    with torch.no_grad():
        y = block(x)
    g = torch.Generator().manual_seed(11)
    lens = [21, 40, 9, 33]
    prompts = [torch.randint(0, cfg["vocab_size"], (n,), generator=g).tolist() for n in lens]
    fx = _decode_fixture(cfg, torch.float32, prompts, 12, keep_full_logits=True)
    fx["arch"] = "qwen3-moe-tiny"
    fx["block_x"] = x
    fx["block_y"] = y
    return fx


def make_gemma3_golden() -> dict:
    """The reference's Gemma 3 model (``model_type`` gemma3_text, ``loader.py:70``) through
    ``LLMEngine._step``, in fp32 and bf16, with norm weights jittered (seed 1) so that every
    (1 + w) scale matters."""
    cfg = get_config("gemma3-tiny")
    g = torch.Generator().manual_seed(17)
    lens = [37, 50, 16, 64]
    prompts = [torch.randint(0, cfg["vocab_size"], (n,), generator=g).tolist() for n in lens]
    out = {"arch": "gemma3-tiny", "norm_jitter": 1}
    for dt, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
        fx = _decode_fixture(cfg, dt, prompts, 16, keep_full_logits=True, norm_jitter=1)
        out.update({f"{k}_{tag}": v for k, v in fx.items()})
    out["prompts"] = out["prompts_f32"]
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MINI_VLLM_REFERENCE"),
                    help="path of the reference checkout (default: $MINI_VLLM_REFERENCE)")
    ap.add_argument("--only", default="", help="comma list of fixtures to (re)make")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or MINI_VLLM_REFERENCE) must name the reference checkout")
    _import_reference(args.reference)
    torch.set_num_threads(os.cpu_count() or 8)
    only = set(filter(None, args.only.split(",")))

    def want(name):
        return not only or name in only

    if want("ops"):
        torch.save(make_ops_golden(), HERE / "ops_golden.pt")
        print("ops_golden.pt written")
    if want("kv"):
        (HERE / "kv_golden.json").write_text(json.dumps(make_kv_golden()))
        print("kv_golden.json written")
    if want("tiny"):
        cfg = get_config("qwen3-tiny")
        g = torch.Generator().manual_seed(7)
        lens = [37, 50, 16, 64]
        prompts = [torch.randint(0, cfg["vocab_size"], (n,), generator=g).tolist() for n in lens]
        fx = _decode_fixture(cfg, torch.bfloat16, prompts, 24, keep_full_logits=True)
        fx["arch"] = "qwen3-tiny"
        torch.save(fx, HERE / "decode_tiny_bf16.pt")
        print("decode_tiny_bf16.pt written")
    if want("engine-trace"):
        (HERE / "engine_trace.json").write_text(json.dumps(make_engine_trace_golden()))
        print("engine_trace.json written")
    if want("moe"):
        torch.save(make_moe_golden(), HERE / "decode_moe_tiny_f32.pt")
        print("decode_moe_tiny_f32.pt written")
    if want("gemma3"):
        torch.save(make_gemma3_golden(), HERE / "decode_gemma3_tiny.pt")
        print("decode_gemma3_tiny.pt written")
    if want("qwen3-0.6b"):
        cfg = get_config("qwen3-0.6b")
        g = torch.Generator().manual_seed(0)
        prompts = [torch.randint(0, cfg["vocab_size"], (128,), generator=g).tolist() for _ in range(4)]
        fx = _decode_fixture(cfg, torch.float32, prompts, 64, keep_full_logits=False)
        fx["arch"] = "qwen3-0.6b"
        torch.save(fx, HERE / "decode_qwen3_0.6b_f32.pt")
        print("decode_qwen3_0.6b_f32.pt written")
    if want("qwen3-0.6b-bf16"):
        # the same architecture, weights and prompts in bf16: greedy, the prefill's token + 32 decode steps
        cfg = get_config("qwen3-0.6b")
        g = torch.Generator().manual_seed(0)
        prompts = [torch.randint(0, cfg["vocab_size"], (128,), generator=g).tolist() for _ in range(4)]
        fx = _decode_fixture(cfg, torch.bfloat16, prompts, 33, keep_full_logits=False)
        fx["arch"] = "qwen3-0.6b"
        torch.save(fx, HERE / "decode_qwen3_0.6b_bf16.pt")
        print("decode_qwen3_0.6b_bf16.pt written")


if __name__ == "__main__":
    main()
