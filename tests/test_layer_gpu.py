"""The fused decoder-layer kernel (``mvb_decoder_layer_tail``) against the unfused kernels it
replaces: o_proj GEMM -> residual add + RMSNorm -> gate_up GEMM -> SwiGLU -> down GEMM -> residual
add + RMSNorm -> (next layer) q|k|v GEMM -> QK-norm + RoPE + paged KV write.  Same split-K plans,
same partial sums: the outputs agree to bf16 rounding (the fused add+norm sums its squares in
another order, a 1-ulp difference in a normalised activation propagates through the next GEMM),
the KV slots written are identical, and the kernel is deterministic."""
import math
import random

import pytest
import torch

from llm_pytorch_inference_b200 import _native as N
from oracle import model as om

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _weights(H, Hq, Hkv, D, I, g):
    def mat(n, k):
        return (torch.randn(n, k, device=DEV, generator=g) * 0.02).to(torch.bfloat16)

    def norm(n):
        return (1 + 0.1 * torch.randn(n, device=DEV, generator=g)).to(torch.bfloat16)

    return {"wo": mat(H, Hq * D), "ln2": norm(H), "wgu": mat(2 * I, H), "wdown": mat(H, I), "ln_next": norm(H),
            "wqkv": mat((Hq + 2 * Hkv) * D, H), "qn": norm(D), "kn": norm(D)}


def _setup(B, H=4096, Hq=32, Hkv=8, D=128, I=12288, L=2, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    w = _weights(H, Hq, Hkv, D, I, g)
    P = 4 * B + 8
    order = list(range(P))
    random.Random(seed).shuffle(order)
    bt = torch.tensor(order[:4 * B], dtype=torch.int32, device=DEV).view(B, 4)
    pos = torch.randint(0, 64, (B,), device=DEV, dtype=torch.int32, generator=g)
    cos, sin = om.rope_tables(D, 1e6, 256, torch.bfloat16, DEV)
    st = {"attn": (torch.randn(B, Hq * D, device=DEV, generator=g) * 0.5).to(torch.bfloat16),
          "residual": torch.randn(B, H, device=DEV, generator=g).to(torch.bfloat16),
          "pool": torch.zeros(L, 2, P + 1, 16, Hkv, D, dtype=torch.bfloat16, device=DEV),
          "bt": bt, "pos": pos, "cos": cos, "sin": sin, "P": P + 1}
    return w, st, dict(B=B, H=H, Hq=Hq, Hkv=Hkv, D=D, I=I, L=L)


def _unfused(w, st, c, with_next):
    lib, s = N.lib(), N.stream_handle()
    B, H, Hq, Hkv, D, I, L = (c[k] for k in ("B", "H", "Hq", "Hkv", "D", "I", "L"))
    ws = torch.zeros(max(lib.mvb_gemm_workspace_bytes(B, n, k, 0) for n, k in
                         ((H, Hq * D), (2 * I, H), (H, I), ((Hq + 2 * Hkv) * D, H))), dtype=torch.uint8, device=DEV)
    res, xn = st["residual"].clone(), torch.empty(B, H, dtype=torch.bfloat16, device=DEV)
    h = torch.empty(B, I, dtype=torch.bfloat16, device=DEV)
    q = torch.zeros(B, Hq, D, dtype=torch.bfloat16, device=DEV)
    pool = st["pool"].clone()

    def gemm(x, wt, epi):
        N.check(lib.mvb_gemm_bf16(None, 0, x.data_ptr(), x.stride(0), wt.data_ptr(), wt.stride(0), B, wt.shape[0],
                                  wt.shape[1], epi, None, 0, ws.data_ptr(), ws.numel(), s), "gemm")

    gemm(st["attn"], w["wo"], N.EPI_PARTIALS)
    N.check(lib.mvb_fused_add_rmsnorm_gemm(xn.data_ptr(), res.data_ptr(), ws.data_ptr(), B, H, Hq * D,
                                           w["ln2"].data_ptr(), 1e-6, 0, s), "fadd")
    gemm(xn, w["wgu"], N.EPI_SWIGLU_PARTIALS)
    N.check(lib.mvb_swiglu_gemm(h.data_ptr(), I, ws.data_ptr(), B, I, H, s), "swiglu")
    gemm(h, w["wdown"], N.EPI_PARTIALS)
    N.check(lib.mvb_fused_add_rmsnorm_gemm(xn.data_ptr(), res.data_ptr(), ws.data_ptr(), B, H, I,
                                           w["ln_next"].data_ptr(), 1e-6, 0, s), "fadd")
    if with_next:
        gemm(xn, w["wqkv"], N.EPI_PARTIALS)
        N.check(lib.mvb_qk_norm_rope_kv_write_gemm(
            q.data_ptr(), pool.data_ptr(), ws.data_ptr(), H, w["qn"].data_ptr(), w["kn"].data_ptr(),
            st["cos"].data_ptr(), st["sin"].data_ptr(), st["cos"].shape[0], st["pos"].data_ptr(), st["bt"].data_ptr(),
            4, B, Hq, Hkv, D, L, 1, st["P"], 16, 1e-6, 0, s), "qk")
    return res, xn, h, q, pool


def _fused(w, st, c, with_next, bar=None, ws=None):
    lib, s = N.lib(), N.stream_handle()
    B, H, Hq, Hkv, D, I, L = (c[k] for k in ("B", "H", "Hq", "Hkv", "D", "I", "L"))
    if ws is None:
        ws = torch.zeros(lib.mvb_decoder_layer_workspace_bytes(B, H, Hq * D, I, (Hq + 2 * Hkv) * D, 0),
                         dtype=torch.uint8, device=DEV)
    if bar is None:
        bar = torch.zeros(256, dtype=torch.uint8, device=DEV)
    res, xn = st["residual"].clone(), torch.empty(B, H, dtype=torch.bfloat16, device=DEV)
    h = torch.empty(B, I, dtype=torch.bfloat16, device=DEV)
    q = torch.zeros(B, Hq, D, dtype=torch.bfloat16, device=DEV)
    pool = st["pool"].clone()
    nxt = with_next
    N.check(lib.mvb_decoder_layer_tail(
        st["attn"].data_ptr(), st["attn"].stride(0), w["wo"].data_ptr(), w["ln2"].data_ptr(), w["wgu"].data_ptr(),
        w["wdown"].data_ptr(), w["ln_next"].data_ptr(), w["wqkv"].data_ptr() if nxt else None,
        w["qn"].data_ptr() if nxt else None, w["kn"].data_ptr() if nxt else None, res.data_ptr(), xn.data_ptr(),
        h.data_ptr(), q.data_ptr(), pool.data_ptr(), st["cos"].data_ptr(), st["sin"].data_ptr(),
        st["cos"].shape[0], st["pos"].data_ptr(), st["bt"].data_ptr(), 4, B, H, Hq, Hkv, D, I, L, 1, st["P"], 16,
        1e-6, ws.data_ptr(), ws.numel(), bar.data_ptr(), s), "decoder_layer_tail")
    return res, xn, h, q, pool


def _close(a, b, what):
    d = (a.float() - b.float()).abs()
    scale = b.float().abs().max().clamp_min(1e-6)
    assert float(d.max()) <= 0.02 * float(scale) + 1e-3, (what, float(d.max()), float(scale))
    assert float(d.mean()) <= 2e-3 * float(b.float().abs().mean()) + 1e-4, (what, float(d.mean()))


@pytest.mark.parametrize("B,with_next", [(64, True), (37, True), (64, False), (1, True)])
def test_fused_layer_matches_unfused_kernels(B, with_next):
    N.device_status(clear=True)
    w, st, c = _setup(B)
    ref = _unfused(w, st, c, with_next)
    got = _fused(w, st, c, with_next)
    for name, a, b in zip(("residual", "xn", "h", "q"), got[:4], ref[:4]):
        if name == "q" and not with_next:
            continue
        _close(a, b, name)
    # the same KV slots written (and nothing else)
    changed_got = (got[4] != st["pool"]).flatten(4).any(-1)
    changed_ref = (ref[4] != st["pool"]).flatten(4).any(-1)
    assert torch.equal(changed_got, changed_ref)
    if with_next:
        _close(got[4], ref[4], "kv")
    assert N.device_status(clear=True) == 0


def test_fused_layer_is_deterministic_and_reusable():
    """Back-to-back launches on one barrier area and workspace: identical results each time (the
    grid barrier re-arms itself, the split-K sums run in a fixed order)."""
    w, st, c = _setup(64, seed=3)
    lib = N.lib()
    ws = torch.zeros(lib.mvb_decoder_layer_workspace_bytes(64, 4096, 4096, 12288, 6144, 0), dtype=torch.uint8,
                     device=DEV)
    bar = torch.zeros(256, dtype=torch.uint8, device=DEV)
    first = _fused(w, st, c, True, bar, ws)
    for _ in range(5):
        again = _fused(w, st, c, True, bar, ws)
        for a, b in zip(first, again):
            assert torch.equal(a, b)
    assert N.device_status(clear=True) == 0


def test_engine_step_with_fused_layers_matches_per_kernel_step():
    """``DecodeEngine(fused_layers=True)`` (one persistent launch per layer after attention) against
    the per-kernel step on the same prefilled KV state: greedy decoding, teacher-forced on the
    per-kernel step's tokens, logits equal to bf16 rounding at every step and the tokens equal
    wherever the top-2 margin is not a near tie."""
    from llm_pytorch_inference_b200.configs import get_config
    from llm_pytorch_inference_b200.engine import DecodeEngine
    from llm_pytorch_inference_b200.weights import canonical_state_dict

    cfg = get_config("qwen3-tiny")
    sd = canonical_state_dict(cfg, 0, torch.bfloat16, device=DEV)
    order = list(range(96))
    random.Random(5).shuffle(order)
    g = torch.Generator().manual_seed(2)
    prompts = {s: torch.randint(0, cfg["vocab_size"], (n,), generator=g).tolist()
               for s, n in enumerate([9, 40, 17, 63, 33, 5, 28, 50])}
    engines = [DecodeEngine(cfg, sd, max_batch=8, max_model_len=160, num_blocks=96, device=DEV,
                            free_order=list(order), fused_layers=f) for f in (False, True)]
    assert not engines[0].runner.fused and engines[1].runner.fused
    firsts = [e.prefill(prompts) for e in engines]
    assert firsts[0] == firsts[1]
    for e in engines:
        e.set_sampling(0.0, -1, 1.0)
    for step in range(6):
        toks = [e.step() for e in engines]
        la, lb = (e.runner.logits[:8].float() for e in engines)
        _close(lb, la, f"logits step {step}")
        top2 = la.topk(2, dim=-1).values
        sure = (top2[:, 0] - top2[:, 1]) > 0.05
        for r in range(8):
            if bool(sure[r]):
                assert toks[1][r] == toks[0][r], (step, r)
        engines[1].force_last_tokens(toks[0])
    assert N.device_status(clear=True) == 0
