"""The drop-in boundary on the GPU, called the way the reference calls it.

* ``torch.ops.mini_vllm_ops.*`` (the 15 schemas of ``csrc/bindings/ops_binding.cpp:11-25``) on CUDA
  tensors, against the outputs the reference's own ops produced (``tests/golden/ops_golden.pt``).
* ``Sampler.sample(logits, SamplingParams)`` (``engine/sampler.py:21``) in its reference mode, and
  the engine's parity sampling mode: given the same logits and the same generator seed, the tokens
  are the ones the reference's CUDA-tensor path draws (``ops/sampling.py:24-73``: top-k, top-p on
  untempered logits, ``/T``, softmax, ``torch.multinomial``), that path run here on the same device.
* ``ForCausalLM.forward`` / ``Attention.forward`` (``models/model_cuda.py:108-121``, ``:412-415``)
  driven like ``LLMEngine`` drives them: the reference's block manager, block tables, slot
  indices, cached-token counts and float mask, on a caller-owned pool.
"""
import random

import numpy as np
import pytest
import torch
from torch.nn.attention import SDPBackend

from llm_pytorch_inference_b200 import _native as N
from llm_pytorch_inference_b200 import torch_ops  # noqa: F401  (registers torch.ops.mini_vllm_ops)
from llm_pytorch_inference_b200.configs import get_config, head_dim, num_kv_heads
from llm_pytorch_inference_b200.engine import DecodeEngine
from llm_pytorch_inference_b200.model_cuda import Attention, ForCausalLM
from llm_pytorch_inference_b200.sampler import Sampler, SamplingParams
from llm_pytorch_inference_b200.weights import canonical_state_dict
from oracle import model as om
from oracle import sampling as osamp
from oracle.engine import OracleEngine

pytestmark = pytest.mark.gpu
DEV = "cuda"
OPS = torch.ops.mini_vllm_ops


@pytest.fixture(scope="module")
def golden(golden_dir):
    return torch.load(golden_dir / "ops_golden.pt")


@pytest.fixture(autouse=True)
def _status_clean():
    N.device_status(clear=True)
    yield
    assert N.device_status(clear=True) == 0, "a kernel reported a device-side error"


def _ulps(a, b):
    ia = a.contiguous().view(torch.int16).to(torch.int32)
    ib = b.contiguous().view(torch.int16).to(torch.int32)
    ia = torch.where(ia < 0, -(ia & 0x7FFF), ia)
    ib = torch.where(ib < 0, -(ib & 0x7FFF), ib)
    return int((ia - ib).abs().max())


# ------------------------------------------------------------------ op namespace
@pytest.mark.parametrize("tag", ["bf16", "f32"])
def test_op_namespace_norms_on_cuda(golden, tag):
    x, w, res = (golden[f"rms_{k}_{tag}"].to(DEV) for k in ("x", "w", "res"))
    out = OPS.rmsnorm_forward(x, w, 1e-6).cpu()
    if tag == "bf16":
        assert _ulps(out, golden["rmsnorm_bf16"]) <= 1
    else:
        torch.testing.assert_close(out, golden["rmsnorm_f32"], rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(OPS.rmsnorm_plus_one_forward(x, w, 1e-6).cpu().float(),
                               golden[f"rmsnorm_p1_{tag}"].float(), rtol=1e-2, atol=2e-2)
    for op, key in ((OPS.fused_add_rmsnorm_forward, "fadd"), (OPS.fused_add_rmsnorm_plus_one_forward, "fadd_p1")):
        r = res.clone()
        y, r2 = op(r, x, w, 1e-6)
        assert torch.equal(r.cpu(), golden[f"{key}_r_{tag}"])       # residual updated in place
        assert torch.equal(r2.cpu(), golden[f"{key}_r_{tag}"])
        torch.testing.assert_close(y.cpu().float(), golden[f"{key}_y_{tag}"].float(), rtol=1e-2, atol=2e-2)


def test_op_namespace_rope_activations_embedding_softmax_mlp(golden):
    q, k = golden["rope_q"], golden["rope_k"]
    pos = golden["rope_positions"][:, 0]
    cos, sin = om.rope_tables(128, 1e6, int(golden["rope_table_len"]), torch.bfloat16)
    # rope_kernel.cu:44-61 contract: [N, D] rows with their cos/sin rows
    qr = q[:, :, 0].reshape(-1, 128)
    cr = cos[pos].repeat_interleave(32, 0)
    sr = sin[pos].repeat_interleave(32, 0)
    out = OPS.rotary_pos_emb_forward(qr.to(DEV), cr.to(DEV), sr.to(DEV)).cpu()
    assert torch.equal(out, golden["rope_q_out"][:, :, 0].reshape(-1, 128))
    ax, ay = golden["act_x"].to(DEV), golden["act_y"].to(DEV)
    assert _ulps(OPS.silu_forward(ax).cpu(), golden["silu"]) <= 1
    assert _ulps(OPS.gelu_forward(ax).cpu(), golden["gelu"]) <= 1
    assert _ulps(OPS.swiglu_forward(ax, ay).cpu(), golden["swiglu"]) <= 1
    assert _ulps(OPS.geglu_forward(ax, ay).cpu(), golden["geglu"]) <= 1
    ids, W = golden["emb_ids"].to(DEV), golden["emb_w"].to(DEV)
    assert torch.equal(OPS.embedding_forward(ids, W, 1.0).cpu(), golden["emb_out"])
    assert torch.equal(OPS.embedding_forward(ids, W, 2.5).cpu(), golden["emb_out_scaled"])
    torch.testing.assert_close(OPS.softmax_forward(golden["softmax_x"].to(DEV)).cpu(), golden["softmax_out"],
                               rtol=1e-5, atol=1e-7)
    gu = (golden["mlp_x"].float() @ golden["mlp_gate_up_w"].float().T).to(torch.bfloat16)
    h = OPS.fused_mlp_forward(gu.to(DEV), 384, 0).cpu()
    g_, u_ = gu.chunk(2, -1)
    assert _ulps(h, torch.nn.functional.silu(g_) * u_) <= 1


def test_op_namespace_sampling(golden):
    logits = golden["samp_logits_bf16"].to(DEV)
    assert torch.equal(OPS.greedy_sample(logits).cpu(), golden["greedy"])
    for k, p in ((50, 0.95), (50, 1.0), (0, 0.9), (1, 1.0), (5, 0.5)):
        x = logits.float().contiguous()
        OPS.top_k_top_p_filter(x, k, p)                                  # in place (ops/sampling.py:35)
        kept = torch.isfinite(x)
        # the reference's own call on the same CUDA tensor (its sort on CUDA orders equal logits by
        # index, the kernel's rule); on the CPU it may keep another member of a tie at the cutoff,
        # so against the CPU-made fixture only the kept count is compared
        assert torch.equal(kept, torch.isfinite(osamp.top_k_top_p_filter(logits.float(), k, p))), (k, p)
        want = np.unpackbits(golden[f"filter_k{k}_p{int(p * 100)}_kept_bits"].numpy(), axis=-1)[:, :x.shape[1]]
        # a nucleus over the whole vocabulary: the CPU's fp32 cumsum over 152k terms moves its
        # cutoff by a few tokens (the kernel's count is checked against exact arithmetic in
        # test_kernels_gpu); with top-k first the counts are equal
        slack = 16 if k <= 0 else 0
        assert np.abs(kept.sum(-1).cpu().numpy() - want.sum(-1)).max() <= slack, (k, p)
        assert torch.equal(x[kept], logits.float()[kept])
    filt = logits.float().contiguous()
    OPS.top_k_top_p_filter(filt, 50, 0.95)
    tok = OPS.softmax_multinomial_sample(filt, 0.8).cpu()
    assert all(torch.isfinite(filt[r, int(tok[r])]) for r in range(tok.shape[0]))


# ---------------------------------------------------------------------- sampling
def _reference_draw(logits_row: torch.Tensor, T: float, k: int, p: float, gen: torch.Generator) -> int:
    """The reference's CUDA-tensor sampling of one sequence (``sampler.py:40-48`` with the
    ``ops/sampling.py`` fallbacks), run on the same device: filter, ``/T``, softmax, multinomial."""
    x = logits_row.float()
    if k > 0 or p < 1.0:
        x = osamp.top_k_top_p_filter(x, k, p)
    if T > 0 and T != 1.0:
        x = x / T
    probs = torch.softmax(x, dim=-1)
    return int(torch.multinomial(probs, num_samples=1, generator=gen).squeeze(-1))


def test_sampler_reference_mode_draws_the_reference_tokens(golden):
    """Same logits, same generator seed: the drop-in ``Sampler`` and the reference's path give the
    same token, for 4 rows x 3 parameter sets x 100 seeds.  The kernel's probabilities equal the
    reference's (tests/golden) to fp32 rounding."""
    logits = golden["samp_logits_bf16"].to(DEV).float()
    probs = torch.empty_like(logits)
    from llm_pytorch_inference_b200 import ops

    ops.sample(logits, 0.8, 50, 0.95, 0, 0, probs_out=probs)
    ref = torch.softmax(osamp.top_k_top_p_filter(logits, 50, 0.95) / 0.8, dim=-1)   # reference path, on CUDA
    for r in range(4):
        assert torch.equal(probs[r].nonzero(), ref[r].nonzero())
        torch.testing.assert_close(probs[r], ref[r], rtol=2e-6, atol=1e-9)
        # the CPU-made fixture: the same number of survivors (a tie at the cutoff may resolve to
        # another index there) and the same probability values
        val = golden[f"probs_t08_k50_p95_row{r}_val"]
        nz = probs[r].nonzero()[:, 0]
        assert len(nz) == len(val)
        torch.testing.assert_close(probs[r, nz].sort().values.cpu(), val.sort().values, rtol=2e-6, atol=1e-9)
    mismatches = 0
    for T, k, p in ((0.8, 50, 0.95), (1.0, -1, 0.9), (0.6, 5, 1.0)):
        for seed in range(100):
            for r in range(4):
                g_ref = torch.Generator(device=DEV).manual_seed(seed)
                g_ours = torch.Generator(device=DEV).manual_seed(seed)
                want = _reference_draw(logits[r:r + 1], T, k, p, g_ref)
                got = Sampler("reference", g_ours).sample(logits[r:r + 1], SamplingParams(T, k, p))[0]
                mismatches += got != want
    assert mismatches == 0
    assert Sampler().sample(logits, SamplingParams(temperature=0.0)) == golden["greedy"].tolist()


def test_engine_parity_sampling_follows_the_reference_draw():
    """A decode engine in parity mode (T 0.8 / top-k 50 / top-p 0.95, 16 sequences): each step's
    tokens equal the reference's per-sequence draws from that step's logits with a generator of
    the same seed, row after row (``engine.py:352-354``)."""
    cfg = get_config("qwen3-tiny")
    sd = {k: v.to(torch.bfloat16) for k, v in canonical_state_dict(cfg, 0, torch.float32).items()}
    eng = DecodeEngine(cfg, sd, max_batch=16, max_model_len=256, num_blocks=256, device=DEV)
    g = torch.Generator().manual_seed(5)
    for s in range(16):
        eng.add_sequence(s, torch.randint(0, cfg["vocab_size"], (int(torch.randint(5, 80, (1,), generator=g)),),
                                          generator=g).tolist())
        eng.append_first_token(s, int(torch.randint(0, cfg["vocab_size"], (1,), generator=g)))
    eng.prefill_synthetic(seed=1)
    gen = torch.Generator(device=DEV).manual_seed(1234)
    ref_gen = torch.Generator(device=DEV).manual_seed(1234)
    eng.set_sampling(0.8, 50, 0.95, parity=True, generator=gen)
    eng.start()
    for step in range(4):
        got = eng.step(use_graph=step > 0)
        logits = eng.runner.logits[:16].clone()
        want = [_reference_draw(logits[r:r + 1], 0.8, 50, 0.95, ref_gen) for r in range(16)]
        assert got == want, step


# ------------------------------------------------------------------- model drop-ins
def _oracles(cfg, sd, P, order):
    o = OracleEngine(cfg, sd, torch.bfloat16, P, 16, list(order), prefill_last_only=True)
    a = OracleEngine(cfg, sd, torch.bfloat16, P, 16, list(order), sdpa_backend=SDPBackend.MATH,
                     prefill_last_only=True)
    return o, a


def _bars(got, ref, ref_alt, where):
    d, n = (got - ref).abs(), (ref_alt - ref).abs()
    assert float(d.max()) <= max(2e-2, 1.5 * float(n.max())), (where, float(d.max()), float(n.max()))
    assert float(d.mean()) <= max(2e-3, 1.25 * float(n.mean())), (where, float(d.mean()), float(n.mean()))


def test_for_causal_lm_drop_in_under_the_reference_engine_loop():
    """``ForCausalLM.forward`` called as ``LLMEngine._run_prefill`` / ``_run_decode`` call the
    reference model (``engine.py:275-283``, ``:339-349``): per-sequence prefill with a flat block
    table at slot 0, then batched decode with the manager's block tables, slot indices, cached
    counts and float mask, on a pool tensor owned by the caller.  Logits within the reference's
    own backend spread of the oracle's, teacher-forced on the oracle's greedy tokens."""
    cfg = get_config("qwen3-tiny")
    sd = canonical_state_dict(cfg, 0, torch.float32)
    P = 128
    order = list(range(P))
    random.Random(2).shuffle(order)
    oracle, alt = _oracles(cfg, sd, P, order)
    model = ForCausalLM(cfg, DEV)
    model.load_state_dict({k: v.to(torch.bfloat16) for k, v in sd.items()})
    pool = torch.zeros(cfg["num_hidden_layers"], 2, P, 16, num_kv_heads(cfg), head_dim(cfg), dtype=torch.bfloat16,
                       device=DEV)
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, cfg["vocab_size"], (n,), generator=g).tolist() for n in (33, 7, 64, 18)]
    for i, p in enumerate(prompts):
        ref, ref_alt = oracle.prefill(i, p), alt.prefill(i, p)
        bt = oracle.blocks.get_block_table(i)
        got = model(torch.tensor([p], device=DEV), torch.arange(len(p), device=DEV), kv_cache=pool,
                    block_tables=bt, slot_idx=0, use_cache=False)
        assert got.shape == (1, 1, cfg["vocab_size"])
        _bars(got[0, 0].float().cpu(), ref, ref_alt, ("prefill", i))
        tok = int(osamp.greedy(ref[None])[0])
        oracle.append(i, tok)
        alt.append(i, tok)
    alt.kv_pool.copy_(oracle.kv_pool)
    seqs = list(range(len(prompts)))
    for step in range(6):
        ref = oracle.decode(seqs)          # grows the tables (engine.py:299-309), then the forward
        ref_alt = alt.decode(seqs)
        bts = [oracle.blocks.get_block_table(s) for s in seqs]
        slot = [len(oracle.tokens[s]) - 1 for s in seqs]
        mask = torch.zeros(len(seqs), 1, 1, max(slot) + 1, dtype=torch.bfloat16, device=DEV)
        for b, n in enumerate(slot):
            mask[b, :, :, n + 1:] = float("-inf")
        ids = torch.tensor([[oracle.tokens[s][-1]] for s in seqs], device=DEV)
        got = model(ids, torch.tensor([[x] for x in slot], device=DEV), kv_cache=pool, block_tables=bts,
                    slot_idx=slot, use_cache=True, num_cached_tokens_list=list(slot), attn_mask=mask)
        _bars(got[:, 0].float().cpu(), ref, ref_alt, ("decode", step))
        for b, t in enumerate(osamp.greedy(ref).tolist()):
            oracle.append(seqs[b], t)
            alt.append(seqs[b], t)
    # the K/V the drop-in wrote sit in the reference's slots
    written = (pool.cpu() != 0).flatten(4).any(-1)
    assert torch.equal(written, (oracle.kv_pool != 0).flatten(4).any(-1))


def test_attention_drop_in_decode_and_prefill():
    """One ``Attention`` layer (Qwen3-8B head shape: 32 query / 8 KV heads of 128, QK-norm) against
    the oracle's ``Attention.forward`` on the same pool state: the batched decode form (per-sequence
    tables, slots, cached counts) and the single-sequence prefill form (flat table, slot 0)."""
    torch.manual_seed(0)
    H, Hq, Hkv, D, P = 1024, 32, 8, 128, 64
    cfg = {"hidden_size": H, "num_attention_heads": Hq, "num_key_value_heads": Hkv, "head_dim": D,
           "num_hidden_layers": 1, "vocab_size": 256, "intermediate_size": 256, "rms_norm_eps": 1e-6,
           "rope_theta": 1e6, "_qk_norm": True}
    att = Attention(H, Hq, Hkv, D, qk_norm=True).to(DEV)
    with torch.no_grad():
        for lin in (att.q_proj, att.k_proj, att.v_proj, att.o_proj):
            lin.weight.copy_(torch.randn_like(lin.weight) * 0.02)
        att.q_norm.weight.copy_(1 + 0.1 * torch.randn(D))
        att.k_norm.weight.copy_(1 + 0.1 * torch.randn(D))
    att = att.to(torch.bfloat16)
    pre = "model.layers.0.self_attn."
    w = {pre + n + ".weight": getattr(att, n).weight.detach().cpu() for n in ("q_proj", "k_proj", "v_proj", "o_proj",
                                                                             "q_norm", "k_norm")}
    w["model.embed_tokens.weight"] = torch.zeros(256, H, dtype=torch.bfloat16)
    dec = om.OracleDecoder(cfg, w, torch.bfloat16)
    pool = (torch.randn(1, 2, P, 16, Hkv, D) * 0.5).to(torch.bfloat16)
    gpool = pool.to(DEV)
    tables = [[5, 9, 2], [40], [7, 8, 11, 12]]
    slot = [37, 3, 60]
    x = (torch.randn(3, 1, H)).to(torch.bfloat16)
    cos_t, sin_t = om.rope_tables(D, 1e6, 256, torch.bfloat16)
    pos = torch.tensor(slot)
    cos, sin = cos_t[pos].unsqueeze(1).unsqueeze(1), sin_t[pos].unsqueeze(1).unsqueeze(1)
    mask = torch.zeros(3, 1, 1, max(slot) + 1, dtype=torch.bfloat16)     # engine.py:330-337
    for b, n in enumerate(slot):
        mask[b, :, :, n + 1:] = float("-inf")
    with torch.no_grad(), torch.autocast("cpu", dtype=torch.bfloat16):
        ref = dec.attention(0, x, cos, sin, pool, tables, slot, True, slot, mask)
    got = att(x.to(DEV), cos.to(DEV), sin.to(DEV), gpool, tables, slot, 0, use_cache=True,
              num_cached_tokens_list=slot, attn_mask=mask.to(DEV))
    torch.testing.assert_close(got.float().cpu(), ref.float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(gpool.float().cpu(), pool.float(), rtol=2e-2, atol=3e-2)   # same slots written
    # prefill: one sequence of 40 tokens at slot 0 into blocks 20, 21, 22
    xs = (torch.randn(1, 40, H)).to(torch.bfloat16)
    bt = [20, 21, 22]
    cos, sin = cos_t[:40].unsqueeze(0).unsqueeze(0), sin_t[:40].unsqueeze(0).unsqueeze(0)
    with torch.no_grad(), torch.autocast("cpu", dtype=torch.bfloat16):
        ref = dec.attention(0, xs, cos, sin, pool, bt, 0, False, None, None)
    got = att(xs.to(DEV), cos.to(DEV), sin.to(DEV), gpool, bt, 0, 0, use_cache=False)
    torch.testing.assert_close(got.float().cpu(), ref.float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(gpool.float().cpu(), pool.float(), rtol=2e-2, atol=3e-2)
