"""Gemma decode on the GPU, through the C ABI, against the oracle.

The oracle's Gemma path is pinned to the reference's own Gemma 3 model
(``models/gemma3_model.py``; tests/golden/decode_gemma3_tiny.pt) and, for the Gemma-2 features
the reference lacks (soft-capping, sliding-window layers), to transformers' Gemma-2
(tests/golden/gemma2_tiny_hf_f32.pt).  Here:

* the GeGLU finalize of split-K partials, the post-norm + residual add + RMSNorm kernel and the
  logit soft-capping kernel against plain PyTorch / unfused compositions;
* whole decode steps of a 2-layer Gemma 3 model and a 4-layer Gemma-2 model (head dim 256,
  prompts longer than the 32-token window), teacher-forced, within the noise-aware bars of the
  dense decode tests (tests/test_decode_gpu.py).
"""
import math

import pytest
import torch
import torch.nn.functional as F

from llm_pytorch_inference_b200 import _native as N
from llm_pytorch_inference_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ulps(a, b):
    """|a - b| in units of the bf16 spacing at |a|."""
    a, b = a.float(), b.float()
    ulp = torch.ldexp(torch.ones_like(a), torch.frexp(a.abs().clamp_min(1e-30))[1] - 8)
    return (a - b).abs() / ulp


def _partials(x, w, ws, epilogue=N.EPI_PARTIALS):
    N.check(N.lib().mvb_gemm_bf16(None, 0, x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), x.shape[0],
                                  w.shape[0], w.shape[1], epilogue, None, 0, ws.data_ptr(), ws.numel(),
                                  N.stream_handle()), "gemm partials")


@pytest.mark.parametrize("m,inter,k", [(16, 14336, 3584), (5, 1024, 512)])
def test_geglu_from_split_k_partials(m, inter, k):
    """GEMM(SWIGLU_PARTIALS) + mvb_gated_gemm(GELU_TANH) against bf16(bf16(gelu_tanh(g)) * u) of the
    bf16 gate/up projections (models/gemma3_model.py:104-105).  The plain GEMM tiles gate and up
    differently from the paired tiling, so a projection may differ by one bf16 step (other fp32
    summation order); GELU's tail magnifies that relatively, so the bar is 2 bf16 steps or 1e-3 of
    the output's scale."""
    g = torch.Generator(device=DEV).manual_seed(inter + m)
    x = (torch.randn(m, k, device=DEV, generator=g) / math.sqrt(k)).to(torch.bfloat16)
    w = torch.randn(2 * inter, k, device=DEV, generator=g).to(torch.bfloat16)
    gu = ops.linear(x, w)
    want = (F.gelu(gu[:, :inter], approximate="tanh") * gu[:, inter:]).to(torch.bfloat16)
    ws = torch.zeros(N.lib().mvb_gemm_workspace_bytes(m, 2 * inter, k, 0), dtype=torch.uint8, device=DEV)
    _partials(x, w, ws, N.EPI_SWIGLU_PARTIALS)
    got = torch.empty(m, inter, dtype=torch.bfloat16, device=DEV)
    N.check(N.lib().mvb_gated_gemm(got.data_ptr(), got.stride(0), ws.data_ptr(), m, inter, k, N.ACT_GELU_TANH,
                                   N.stream_handle()), "gated_gemm")
    torch.testing.assert_close(got.float(), want.float(), rtol=2 ** -7, atol=1e-3 * float(want.abs().max()))
    assert float((_ulps(want, got) > 0).float().mean()) < 1e-2


@pytest.mark.parametrize("m,n,k", [(16, 3584, 4096), (16, 3584, 14336), (7, 512, 1024)])
def test_post_norm_add_rmsnorm_from_partials(m, n, k):
    """GEMM(PARTIALS) + mvb_fused_norm_add_rmsnorm_gemm against the unfused chain (GEMM store,
    RMSNorm(1 + w_post), residual add, RMSNorm(1 + w)) of gemma3_model.py:274-281.  The sums of
    squares use different reduction trees, so values may move by a bf16 step or two."""
    g = torch.Generator(device=DEV).manual_seed(n + k + m)
    x = (torch.randn(m, k, device=DEV, generator=g) / math.sqrt(k)).to(torch.bfloat16)
    w = torch.randn(n, k, device=DEV, generator=g).to(torch.bfloat16)
    pw = (0.2 * torch.randn(n, device=DEV, generator=g)).to(torch.bfloat16)
    ln = (0.2 * torch.randn(n, device=DEV, generator=g)).to(torch.bfloat16)
    res0 = (4 * torch.randn(m, n, device=DEV, generator=g)).to(torch.bfloat16)
    y = ops.linear(x, w)

    def norm(t, wt):   # Gemma RMSNorm (gemma3_model.py:21-25)
        var = t.float().pow(2).mean(-1, keepdim=True)
        return ((t * torch.rsqrt(var + 1e-6)) * (1.0 + wt.float())).to(torch.bfloat16)

    z_want = norm(y, pw)
    res_want = res0 + z_want
    xn_want = norm(res_want, ln)
    ws = torch.zeros(N.lib().mvb_gemm_workspace_bytes(m, n, k, 0), dtype=torch.uint8, device=DEV)
    _partials(x, w, ws)
    res, xn = res0.clone(), torch.empty_like(res0)
    N.check(N.lib().mvb_fused_norm_add_rmsnorm_gemm(xn.data_ptr(), res.data_ptr(), ws.data_ptr(), m, n, k,
                                                    pw.data_ptr(), ln.data_ptr(), 1e-6, 1, N.stream_handle()),
            "norm add norm")
    # one bf16 step of the post-normed z may carry into the sum (also where res0 + z cancels)
    def step(t):
        t = t.float()
        return torch.ldexp(torch.ones_like(t), torch.frexp(t.abs().clamp_min(1e-30))[1] - 8)

    assert bool(((res.float() - res_want.float()).abs() <= step(z_want) + step(res_want)).all())
    assert float((_ulps(res_want, res) > 0).float().mean()) < 1e-2
    assert float((_ulps(xn_want, xn) > 0).float().mean()) < 2e-2
    torch.testing.assert_close(xn.float(), xn_want.float(), rtol=2 ** -6, atol=2 ** -6)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_final_logit_softcap(dtype):
    g = torch.Generator(device=DEV).manual_seed(3)
    x = (torch.randn(16, 256000, device=DEV, generator=g) * 40).to(dtype)
    want = torch.tanh(x / 30.0) * 30.0
    got = x.clone()
    N.check(N.lib().mvb_softcap(got.data_ptr(), got.numel(), 30.0, N.dtype_code(got), N.stream_handle()), "softcap")
    if dtype == torch.bfloat16:
        assert float(_ulps(want, got).max()) <= 1.0
    else:
        torch.testing.assert_close(got, want, rtol=1e-6, atol=1e-5)
    assert float(got.abs().max()) <= 30.0


@pytest.mark.parametrize("arch,lens,jitter", [
    ("gemma3-tiny", [37, 50, 16, 64, 5], 1),     # the reference's Gemma 3 (QK-norm, local/global theta)
    ("gemma2-tiny", [40, 51, 9, 70, 33], 1),     # Gemma-2: softcaps, 32-token sliding window
])
def test_gemma_decode_teacher_forced_matches_oracle(arch, lens, jitter):
    from test_decode_gpu import _compare_teacher_forced, _setup

    g = torch.Generator().manual_seed(31)
    prompts = [torch.randint(0, 4096, (n,), generator=g).tolist() for n in lens]
    cfg, oracle, alt, eng = _setup(arch, prompts, 256, norm_jitter=jitter)
    _compare_teacher_forced(oracle, alt, eng, 12)
    assert N.device_status(clear=True) == 0
