"""Sparse MoE (Qwen3-MoE) decode on the GPU, through the C ABI, against the oracle (the
reference's ``Qwen3MoeSparseMoe.forward`` restated, pinned to fixtures the reference made).

* routing: top-k ids exact, weights to fp32 rounding, dispatch order consistent;
* grouped expert GEMMs: against per-expert fp32 matmuls (bf16 tolerance);
* combine: bit-exact against the reference's expert-ordered bf16 accumulation;
* the whole decode step of a 2-layer MoE model, teacher-forced, within the noise-aware bars of
  the dense decode tests.
"""
import pytest
import torch

from llm_pytorch_inference_b200 import _native as N
from oracle import model as om

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _route(logits, K, norm=1):
    B, E = logits.shape
    outs = {n: torch.zeros(*s, dtype=dt, device=DEV) for n, s, dt in (
        ("ids", (B, K), torch.int32), ("w", (B, K), torch.float32), ("pair_row", (B, K), torch.int32),
        ("row_token", (B * K,), torch.int32), ("off", (E + 1,), torch.int32), ("active", (E + 1,), torch.int32))}
    N.check(N.lib().mvb_moe_route(logits.data_ptr(), B, E, K, norm, outs["ids"].data_ptr(), outs["w"].data_ptr(),
                                  outs["pair_row"].data_ptr(), outs["row_token"].data_ptr(), outs["off"].data_ptr(),
                                  outs["active"].data_ptr(), N.stream_handle()), "moe_route")
    torch.cuda.synchronize()
    return outs


@pytest.mark.parametrize("B,E,K", [(32, 128, 8), (5, 16, 4), (64, 128, 8), (256, 64, 2)])
def test_route_matches_oracle_and_dispatch_is_consistent(B, E, K):
    g = torch.Generator().manual_seed(B * E + K)
    logits = (torch.randn(B, E, generator=g) * 2).to(torch.bfloat16)
    r = _route(logits.to(DEV), K)
    topw, topi = om.moe_route(logits, K, True)
    assert torch.equal(r["ids"].cpu().long(), topi)
    torch.testing.assert_close(r["w"].cpu(), topw, rtol=2e-6, atol=1e-7)
    ids, off, act = r["ids"].cpu(), r["off"].cpu(), r["active"].cpu()
    counts = torch.bincount(ids.flatten().long(), minlength=E)
    assert torch.equal(off[1:] - off[:-1], counts.int()) and int(off[0]) == 0
    assert act[1:1 + int(act[0])].tolist() == [e for e in range(E) if counts[e] > 0]
    pr, rt = r["pair_row"].cpu(), r["row_token"].cpu()
    assert sorted(pr.flatten().tolist()) == list(range(B * K))
    for b in range(B):
        for k in range(K):
            assert int(rt[pr[b, k]]) == b
            e = int(ids[b, k])
            assert off[e] <= pr[b, k] < off[e + 1]
    for e in range(E):                                # rows of an expert in ascending token order
        toks = rt[off[e]:off[e + 1]].tolist()
        assert toks == sorted(toks)


@pytest.mark.parametrize("B,E,K,H,I", [(32, 128, 8, 2048, 768), (5, 16, 4, 512, 128), (64, 32, 4, 256, 192),
                                       (128, 8, 2, 256, 128),     # 128-row tiles (up to 128 rows per expert)
                                       (256, 16, 4, 512, 128)])   # 256-row tiles: a prefill chunk's expert groups
def test_grouped_expert_gemms_match_fp32(B, E, K, H, I):
    g = torch.Generator().manual_seed(E + H + I)
    logits = torch.randn(B, E, generator=g).to(torch.bfloat16)
    r = _route(logits.to(DEV), K)
    x = (torch.randn(B, H, generator=g) / H ** 0.5).to(torch.bfloat16).to(DEV)
    wgu = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    wdn = (torch.randn(E, H, I, generator=g) * 0.05).to(torch.bfloat16).to(DEV)
    lib, st, n = N.lib(), N.stream_handle(), B * K
    xs = torch.zeros(n, H, dtype=torch.bfloat16, device=DEV)
    hs = torch.full((n, I), float("nan"), dtype=torch.bfloat16, device=DEV)
    ys = torch.full((n, H), float("nan"), dtype=torch.bfloat16, device=DEV)
    N.check(lib.mvb_moe_gather(xs.data_ptr(), x.data_ptr(), H, r["row_token"].data_ptr(), n, st), "gather")
    N.check(lib.mvb_moe_gemm_bf16(hs.data_ptr(), I, xs.data_ptr(), H, wgu.data_ptr(), 2 * I, H, E, n, B,
                                  N.EPI_SWIGLU, r["off"].data_ptr(), r["active"].data_ptr(), st), "gate_up")
    N.check(lib.mvb_moe_gemm_bf16(ys.data_ptr(), H, hs.data_ptr(), I, wdn.data_ptr(), H, I, E, n, B, N.EPI_STORE,
                                  r["off"].data_ptr(), r["active"].data_ptr(), st), "down")
    torch.cuda.synchronize()
    assert N.device_status(clear=True) == 0
    rt, off = r["row_token"].cpu(), r["off"].cpu()
    assert torch.equal(xs.cpu(), x.cpu()[rt.long()])
    for e in range(E):
        a, b = int(off[e]), int(off[e + 1])
        if a == b:
            continue
        xe = xs[a:b].float()
        gu = (xe @ wgu[e].float().T).to(torch.bfloat16).float()
        h = torch.nn.functional.silu(gu[:, :I]).to(torch.bfloat16).float() * gu[:, I:]
        torch.testing.assert_close(hs[a:b].float(), h, rtol=2e-2, atol=2e-2)
        y = hs[a:b].float() @ wdn[e].float().T
        torch.testing.assert_close(ys[a:b].float(), y, rtol=2e-2, atol=2e-2)


def test_combine_is_bit_exact_against_reference_accumulation():
    B, E, K, H = 9, 16, 4, 512
    g = torch.Generator().manual_seed(3)
    logits = torch.randn(B, E, generator=g).to(torch.bfloat16)
    r = _route(logits.to(DEV), K)
    y = torch.randn(B * K, H, generator=g).to(torch.bfloat16)
    yd = y.to(DEV)
    out = torch.empty(B, H, dtype=torch.bfloat16, device=DEV)
    N.check(N.lib().mvb_moe_combine(out.data_ptr(), yd.data_ptr(), r["w"].data_ptr(), r["ids"].data_ptr(),
                                    r["pair_row"].data_ptr(), B, K, H, N.stream_handle()), "combine")
    pr = r["pair_row"].cpu().long()
    outs = y[pr]                                                     # [B, K, H]
    ref = om.moe_combine(outs, r["w"].cpu(), r["ids"].cpu(), torch.bfloat16)
    got = out.cpu()
    assert torch.equal(got, ref), int((got != ref).sum())


def test_moe_decode_teacher_forced_matches_oracle():
    from test_decode_gpu import _compare_teacher_forced, _setup

    g = torch.Generator().manual_seed(21)
    lens = [21, 40, 9, 33, 17, 64]
    prompts = [torch.randint(0, 4096, (n,), generator=g).tolist() for n in lens]
    cfg, oracle, alt, eng = _setup("qwen3-moe-tiny", prompts, 256)
    _compare_teacher_forced(oracle, alt, eng, 10)
    assert N.device_status(clear=True) == 0


@pytest.mark.parametrize("first,count", [(0, 32), (32, 32), (96, 32), (64, 16)])
def test_expert_range_gemms_equal_the_full_grouped_gemm_on_their_rows(first, count):
    """Expert parallelism: with only experts first .. first+count-1 in the weight tensor, the
    grouped GEMMs compute exactly the full grouped GEMM's rows of those experts and leave every
    other dispatched row untouched."""
    B, E, K, H, I = 32, 128, 8, 2048, 768
    g = torch.Generator().manual_seed(first + count)
    r = _route(torch.randn(B, E, generator=g).to(torch.bfloat16).to(DEV), K)
    x = (torch.randn(B * K, H, generator=g) / H ** 0.5).to(torch.bfloat16).to(DEV)
    wgu = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    lib, st, n = N.lib(), N.stream_handle(), B * K
    full = torch.zeros(n, I, dtype=torch.bfloat16, device=DEV)
    part = torch.full((n, I), 7.0, dtype=torch.bfloat16, device=DEV)
    N.check(lib.mvb_moe_gemm_bf16(full.data_ptr(), I, x.data_ptr(), H, wgu.data_ptr(), 2 * I, H, E, n, B,
                                  N.EPI_SWIGLU, r["off"].data_ptr(), r["active"].data_ptr(), st), "full")
    local = wgu[first:first + count].contiguous()
    N.check(lib.mvb_moe_gemm_bf16_experts(part.data_ptr(), I, x.data_ptr(), H, local.data_ptr(), 2 * I, H, E, first,
                                          count, n, B, N.EPI_SWIGLU, r["off"].data_ptr(), r["active"].data_ptr(), st),
            "experts")
    torch.cuda.synchronize()
    assert N.device_status(clear=True) == 0
    off = r["off"].cpu()
    a, b = int(off[first]), int(off[first + count])
    assert torch.equal(part[a:b], full[a:b])
    assert bool((part[:a] == 7.0).all()) and bool((part[b:] == 7.0).all())


def test_tp_moe_combine_pushes_each_ranks_partial():
    """mvb_tp_moe_combine on one rank: the combined rows (all experts local) land in the receive
    area's layout bit-exact against the reference accumulation; with half the experts, the
    partial is the reference accumulation over those experts' slots only."""
    from llm_pytorch_inference_b200 import tensor_parallel as tpm

    B, E, K, H = 16, 16, 4, 512
    g = torch.Generator().manual_seed(9)
    r = _route(torch.randn(B, E, generator=g).to(torch.bfloat16).to(DEV), K)
    y = torch.randn(B * K, H, generator=g).to(torch.bfloat16)
    yd = y.to(DEV)
    lib = N.lib()
    recv_bytes = lib.mvb_tp_recv_bytes(B, H, 64, 1, 0)
    assert recv_bytes == B * H * 4
    heap = tpm.SymmetricHeap(lib.mvb_tp_signal_bytes() + recv_bytes + 4096, 0, 1)
    try:
        off = (lib.mvb_tp_signal_bytes() + 255) // 256 * 256
        recv = heap.tensor(off, (H // 128, B, 128), torch.float32, DEV)   # [tile][row][128] for one rank
        pr = r["pair_row"].cpu().long()
        for first, count in ((0, E), (8, 8)):
            N.check(lib.mvb_tp_begin_step(heap.comm, N.stream_handle()), "begin")
            N.check(lib.mvb_tp_moe_combine(heap.comm, yd.data_ptr(), r["w"].data_ptr(), r["ids"].data_ptr(),
                                           r["pair_row"].data_ptr(), B, K, H, first, count, off, 5,
                                           N.stream_handle()), "tp_moe_combine")
            N.check(lib.mvb_tp_wait(heap.comm, 5, N.stream_handle()), "wait")
            torch.cuda.synchronize()
            got = recv.permute(1, 0, 2).reshape(B, H).cpu()
            ids, w = r["ids"].cpu(), r["w"].cpu().clone()
            mine = (ids >= first) & (ids < first + count)
            w[~mine] = 0.0          # a zero weight adds exactly nothing to the bf16 chain
            want = om.moe_combine(y[pr], w, ids, torch.bfloat16).float()
            assert torch.equal(got, want), (first, count)
        assert N.device_status(clear=True) == 0
    finally:
        torch.cuda.synchronize()
        heap.close()
