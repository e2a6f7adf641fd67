"""Kernel-level parity on the GPU: each sm_100a kernel against the oracle (the reference's
algorithm restated on the CPU) or a plain fp32 PyTorch reference, at small sizes."""
import math
import random

import numpy as np
import pytest
import torch

from llm_pytorch_inference_b200 import _native as N
from llm_pytorch_inference_b200 import ops
from oracle import model as om
from oracle import sampling as osamp

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def golden(golden_dir):
    return torch.load(golden_dir / "ops_golden.pt")


@pytest.fixture(autouse=True)
def _status_clean():
    N.device_status(clear=True)
    yield
    assert N.device_status(clear=True) == 0, "a kernel reported a device-side error"


def bf16_ulps(a: torch.Tensor, b: torch.Tensor) -> int:
    """Max distance in bf16 units in the last place between two bf16 tensors."""
    ia = a.contiguous().view(torch.int16).to(torch.int32)
    ib = b.contiguous().view(torch.int16).to(torch.int32)
    ia = torch.where(ia < 0, -(ia & 0x7FFF), ia)
    ib = torch.where(ib < 0, -(ib & 0x7FFF), ib)
    return int((ia - ib).abs().max())


# ------------------------------------------------------------------------ norms
@pytest.mark.parametrize("tag", ["bf16", "f32"])
def test_rmsnorm_ops_semantics_match_reference_fallback(golden, tag):
    x, w, res = golden[f"rms_x_{tag}"], golden[f"rms_w_{tag}"], golden[f"rms_res_{tag}"]
    out = ops.rmsnorm(x.to(DEV), w.to(DEV)).cpu()
    ref = golden[f"rmsnorm_{tag}"]
    if tag == "bf16":
        assert bf16_ulps(out, ref) <= 1
    else:
        torch.testing.assert_close(out, ref, rtol=1e-6, atol=1e-6)
    out = ops.rmsnorm_plus_one(x.to(DEV), w.to(DEV)).cpu()
    torch.testing.assert_close(out.float(), golden[f"rmsnorm_p1_{tag}"].float(), rtol=1e-2, atol=2e-2)
    r = res.to(DEV).clone()
    y, r2 = ops.fused_add_rmsnorm(r, x.to(DEV), w.to(DEV))
    assert r2.data_ptr() == r.data_ptr()  # residual updated in place (rmsnorm_kernel.cu:187-204)
    assert torch.equal(r.cpu(), golden[f"fadd_r_{tag}"])
    torch.testing.assert_close(y.cpu().float(), golden[f"fadd_y_{tag}"].float(), rtol=1e-2, atol=2e-2)


def test_rmsnorm_model_semantics_match_oracle():
    torch.manual_seed(0)
    x = torch.randn(64, 4096).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(4096)).to(torch.bfloat16)
    out = torch.empty(64, 4096, dtype=torch.bfloat16, device=DEV)
    xd, wd = x.to(DEV), w.to(DEV)
    N.check(N.lib().mvb_rmsnorm(out.data_ptr(), 4096, xd.data_ptr(), 4096, wd.data_ptr(), 64, 4096, 1e-6, 0,
                                N.NORM_MODEL, N.BF16, N.stream_handle()), "rmsnorm")
    assert bf16_ulps(out.cpu(), om.rms_norm(x, w, 1e-6)) <= 1


@pytest.mark.parametrize("rows,hidden", [(1000, 4096), (300, 512), (777, 3584), (2049, 2048)])
def test_norms_over_many_rows_match_the_row_kernels(rows, hidden):
    """More than 256 rows (a prefill) take the warp-per-row kernels: the per-element rounding of the
    CTA-per-row kernels that decode batches use (run here 256 rows at a time), the fp32 sum of
    squares in another order (at most 1 bf16 ulp apart), the residual sum bit-exact; strided input
    rows, in place."""
    bf = torch.bfloat16
    g = torch.Generator(device=DEV).manual_seed(rows + hidden)
    x = torch.randn(rows, hidden + 64, device=DEV, generator=g).to(bf)   # row stride hidden + 64
    w = (1 + 0.1 * torch.randn(hidden, device=DEV, generator=g)).to(bf)
    lib, st = N.lib(), N.stream_handle()

    def norm(out, inp, n, plus_one, sem):
        N.check(lib.mvb_rmsnorm(out.data_ptr(), out.stride(0), inp.data_ptr(), inp.stride(0), w.data_ptr(), n,
                                hidden, 1e-6, plus_one, sem, N.BF16, st), "rmsnorm")

    for plus_one, sem in [(0, N.NORM_MODEL), (1, N.NORM_MODEL), (0, N.NORM_OPS), (1, N.NORM_OPS)]:
        out = torch.empty(rows, hidden, dtype=bf, device=DEV)
        norm(out, x, rows, plus_one, sem)
        ref = torch.empty_like(out)
        for r0 in range(0, rows, 256):
            norm(ref[r0:], x[r0:], min(256, rows - r0), plus_one, sem)
        assert bf16_ulps(out.cpu(), ref.cpu()) <= 1, (plus_one, sem)
    z = x[:, :hidden].contiguous()
    zz = z.clone()
    norm(zz, zz, rows, 0, N.NORM_MODEL)                      # in place
    out = torch.empty_like(z)
    norm(out, z, rows, 0, N.NORM_MODEL)
    assert torch.equal(zz, out)
    res = torch.randn(rows, hidden, device=DEV, generator=g).to(bf)
    r_a, r_b = res.clone(), res.clone()
    y_a, y_b = torch.empty_like(z), torch.empty_like(z)
    N.check(lib.mvb_fused_add_rmsnorm(y_a.data_ptr(), r_a.data_ptr(), z.data_ptr(), w.data_ptr(), rows, hidden, 1e-6,
                                      0, N.NORM_MODEL, N.BF16, st), "fused_add_rmsnorm")
    for r0 in range(0, rows, 256):
        N.check(lib.mvb_fused_add_rmsnorm(y_b[r0:].data_ptr(), r_b[r0:].data_ptr(), z[r0:].data_ptr(), w.data_ptr(),
                                          min(256, rows - r0), hidden, 1e-6, 0, N.NORM_MODEL, N.BF16, st),
                "fused_add_rmsnorm")
    assert torch.equal(r_a, r_b)
    assert torch.equal(r_a, (res.float() + z.float()).to(bf))
    assert bf16_ulps(y_a.cpu(), y_b.cpu()) <= 1


# ------------------------------------------------------------------ elementwise
def test_rope_op_matches_reference(golden):
    q, k = golden["rope_q"], golden["rope_k"]
    cos, sin = om.rope_tables(128, 1e6, int(golden["rope_table_len"]), torch.bfloat16)
    pos = golden["rope_positions"]
    c, s = cos[pos].unsqueeze(1), sin[pos].unsqueeze(1)
    qe, ke = ops.apply_rotary_pos_emb(q.to(DEV), k.to(DEV), c.to(DEV), s.to(DEV))
    assert torch.equal(qe.cpu(), golden["rope_q_out"])
    assert torch.equal(ke.cpu(), golden["rope_k_out"])


def test_rope_tables_are_built_where_the_reference_builds_them():
    """The reference builds its cos/sin cache on the device of the positions (``model.py:74-80``),
    and a bf16 position ramp rounds differently on the CPU and on the GPU past position 4112.  The
    decode path's tables equal the oracle's built on the same GPU, at every position up to 9000."""
    from llm_pytorch_inference_b200.runner import rope_tables

    for theta in (1e6, 5e5):
        cos, sin = rope_tables(128, theta, 9000, torch.bfloat16, DEV)
        ocos, osin = om.rope_tables(128, theta, 9000, torch.bfloat16, DEV)
        assert torch.equal(cos, ocos) and torch.equal(sin, osin)


def test_activations_embedding_softmax(golden):
    ax, ay = golden["act_x"].to(DEV), golden["act_y"].to(DEV)
    for fn, key in ((ops.silu, "silu"), (ops.gelu, "gelu")):
        assert bf16_ulps(fn(ax).cpu(), golden[key]) <= 1
    assert bf16_ulps(ops.swiglu(ax, ay).cpu(), golden["swiglu"]) <= 1
    assert bf16_ulps(ops.geglu(ax, ay).cpu(), golden["geglu"]) <= 1
    e = ops.embedding(golden["emb_ids"].to(DEV), golden["emb_w"].to(DEV), 1.0).cpu()
    assert torch.equal(e, golden["emb_out"])
    e = ops.embedding(golden["emb_ids"].to(DEV), golden["emb_w"].to(DEV), 2.5).cpu()
    assert torch.equal(e, golden["emb_out_scaled"])
    sm = ops.softmax(golden["softmax_x"].to(DEV)).cpu()
    torch.testing.assert_close(sm, golden["softmax_out"], rtol=1e-5, atol=1e-7)


def test_embedding_bad_id_is_reported_not_faulted():
    w = torch.randn(10, 64, device=DEV).to(torch.bfloat16)
    out = ops.embedding(torch.tensor([3, 11], device=DEV), w)
    assert torch.equal(out[0], w[3]) and torch.count_nonzero(out[1]) == 0
    assert N.device_status(clear=True) & N.DEV_BAD_TOKEN


def test_fused_mlp_module_matches_reference(golden):
    mlp = ops.FusedMLP(256, 384, "silu").to(DEV, torch.bfloat16)
    with torch.no_grad():
        mlp.gate_up_proj.weight.copy_(golden["mlp_gate_up_w"])
        mlp.down_proj.weight.copy_(golden["mlp_down_w"])
    out = mlp(golden["mlp_x"].to(DEV)).cpu()
    torch.testing.assert_close(out.float(), golden["mlp_out"].float(), rtol=2e-2, atol=2e-2)
    gu = golden["mlp_x"].float() @ golden["mlp_gate_up_w"].float().T
    h = ops.fused_mlp_forward(gu.to(torch.bfloat16).to(DEV), 384, 0).cpu()
    g, u = gu.to(torch.bfloat16).chunk(2, -1)
    assert bf16_ulps(h, torch.nn.functional.silu(g) * u) <= 1


# ------------------------------------------------------------------------- GEMM
@pytest.mark.parametrize("m,n,k", [(64, 4096, 4096), (64, 6144, 4096), (1, 512, 512), (37, 1000, 128),
                                   (128, 2048, 1024), (256, 256, 8192), (64, 151936, 256)])
def test_gemm_store_matches_fp32(m, n, k):
    g = torch.Generator(device=DEV).manual_seed(m * 7 + n + k)
    x = (torch.randn(m, k, device=DEV, generator=g) / math.sqrt(k)).to(torch.bfloat16)
    w = torch.randn(n, k, device=DEV, generator=g).to(torch.bfloat16)
    y = ops.linear(x, w)
    ref = x.float() @ w.float().T
    torch.testing.assert_close(y.float(), ref, rtol=1e-2, atol=1e-2)
    assert torch.equal(ops.linear(x, w), y)  # deterministic split-K merge


@pytest.mark.parametrize("m,n,k", [(257, 1024, 512), (700, 4096, 4096), (2049, 6144, 4096), (4096, 512, 12288),
                                   (300, 384, 256)])
def test_gemm_row_tiles_for_prefill(m, n, k):
    """More than 256 rows (a prefill's tokens): row tiles of 256, ragged last tile; the three
    epilogues a prefill uses (store, SwiGLU, residual add).  An even number of weight tiles takes
    the 256 x 256 tile kernel; n = 384 (3 weight tiles, 3 SwiGLU pairs) the 128 x 256 one."""
    g = torch.Generator(device=DEV).manual_seed(m + n + k)
    x = (torch.randn(m, k, device=DEV, generator=g) / math.sqrt(k)).to(torch.bfloat16)
    w = torch.randn(n, k, device=DEV, generator=g).to(torch.bfloat16)
    y = ops.linear(x, w)
    ref = x.float() @ w.float().T
    torch.testing.assert_close(y.float(), ref, rtol=1e-2, atol=1e-2)
    assert torch.equal(ops.linear(x, w), y)
    h = ops.linear(x, w, N.EPI_SWIGLU)
    gu = ref.to(torch.bfloat16)
    sw = torch.nn.functional.silu(gu[:, :n // 2].float()).to(torch.bfloat16).float() * gu[:, n // 2:].float()
    torch.testing.assert_close(h.float(), sw, rtol=2e-2, atol=2e-2)
    aux = torch.randn(m, n, device=DEV, generator=g).to(torch.bfloat16)
    r = ops.linear(x, w, N.EPI_RESADD, aux=aux)
    torch.testing.assert_close(r.float(), aux.float() + gu.float(), rtol=1e-2, atol=2e-2)
    assert N.device_status(clear=True) == 0


def test_gemm_shapes_sharing_one_workspace():
    # the decode step's five GEMM shapes back to back on one buffer, twice, as the runner does
    from llm_pytorch_inference_b200 import _native
    shapes = [(6144, 4096), (4096, 4096), (2 * 12288, 4096), (4096, 12288), (151936, 4096)]
    need = max(_native.lib().mvb_gemm_workspace_bytes(64, n, k, 0) for n, k in shapes)
    ws = torch.zeros(need, dtype=torch.uint8, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(8)
    xs = {k: (torch.randn(64, k, device=DEV, generator=g) / math.sqrt(k)).to(torch.bfloat16) for _, k in shapes}
    ws_ = {s: torch.randn(*s, device=DEV, generator=g).to(torch.bfloat16) for s in shapes}
    for _ in range(2):
        for n, k in shapes:
            y = ops.linear(xs[k], ws_[(n, k)], workspace=ws)
            torch.testing.assert_close(y.float(), xs[k].float() @ ws_[(n, k)].float().T, rtol=1e-2, atol=1e-2)


def test_gemm_swiglu_and_resadd_epilogues():
    g = torch.Generator(device=DEV).manual_seed(3)
    m, inter, k = 64, 1536, 2048
    x = (torch.randn(m, k, device=DEV, generator=g) / math.sqrt(k)).to(torch.bfloat16)
    w = torch.randn(2 * inter, k, device=DEV, generator=g).to(torch.bfloat16)
    h = ops.linear(x, w, N.EPI_SWIGLU)
    gu = (x.float() @ w.float().T).to(torch.bfloat16)
    gate, up = gu[:, :inter], gu[:, inter:]
    ref = (torch.nn.functional.silu(gate.float()).to(torch.bfloat16).float() * up.float())
    torch.testing.assert_close(h.float(), ref, rtol=2e-2, atol=2e-2)
    aux = torch.randn(m, 1024, device=DEV, generator=g).to(torch.bfloat16)
    w2 = torch.randn(1024, k, device=DEV, generator=g).to(torch.bfloat16)
    y = ops.linear(x, w2, N.EPI_RESADD, aux=aux)
    ref = aux.float() + (x.float() @ w2.float().T).to(torch.bfloat16).float()
    torch.testing.assert_close(y.float(), ref, rtol=1e-2, atol=2e-2)


def _gemm_partials(x, w, ws, epilogue=N.EPI_PARTIALS):
    N.check(N.lib().mvb_gemm_bf16(None, 0, x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), x.shape[0],
                                  w.shape[0], w.shape[1], epilogue, None, 0, ws.data_ptr(), ws.numel(),
                                  N.stream_handle()), "gemm partials")


@pytest.mark.parametrize("m,inter,k", [(64, 12288, 4096), (64, 3072, 1024), (5, 1536, 2048), (200, 256, 512),
                                        (128, 14336, 4096), (128, 12288, 4096), (256, 12288, 4096)])
def test_swiglu_from_split_k_partials_bit_exact(m, inter, k):
    """GEMM(MVB_EPI_SWIGLU_PARTIALS) + mvb_swiglu_gemm == GEMM(MVB_EPI_SWIGLU): same contributor-order
    sums, same rounding sequence.  Runs twice on one workspace (the finalize leaves nothing behind)."""
    g = torch.Generator(device=DEV).manual_seed(inter + k + m)
    x = (torch.randn(m, k, device=DEV, generator=g) / math.sqrt(k)).to(torch.bfloat16)
    w = torch.randn(2 * inter, k, device=DEV, generator=g).to(torch.bfloat16)
    want = ops.linear(x, w, N.EPI_SWIGLU)
    ws = torch.zeros(N.lib().mvb_gemm_workspace_bytes(m, 2 * inter, k, 0), dtype=torch.uint8, device=DEV)
    for _ in range(2):
        got = torch.full((m, inter + 8), float("nan"), dtype=torch.bfloat16, device=DEV)
        _gemm_partials(x, w, ws, N.EPI_SWIGLU_PARTIALS)
        N.check(N.lib().mvb_swiglu_gemm(got.data_ptr(), got.stride(0), ws.data_ptr(), m, inter, k,
                                        N.stream_handle()), "swiglu_gemm")
        assert torch.equal(got[:, :inter], want)
        assert bool(got[:, inter:].isnan().all())   # nothing written past inter


@pytest.mark.parametrize("m,n,k", [(64, 4096, 4096), (64, 4096, 12288), (13, 1024, 512), (128, 4096, 14336),
                                   (128, 4096, 4096), (256, 4096, 4096)])
def test_split_k_partials_feed_fused_add_rmsnorm_bit_exactly(m, n, k):
    """GEMM(MVB_EPI_PARTIALS) + mvb_fused_add_rmsnorm_gemm == GEMM(STORE) + fused_add_rmsnorm (model
    semantics): the consumer sums the same partials in the same order, so the updated residual is
    bit-identical.  The normalised output may differ by one bf16 rounding step where the two
    kernels' fp32 sums of squares (different reduction trees) straddle a rounding boundary."""
    g = torch.Generator(device=DEV).manual_seed(n + k)
    x = (torch.randn(m, k, device=DEV, generator=g) / math.sqrt(k)).to(torch.bfloat16)
    w = torch.randn(n, k, device=DEV, generator=g).to(torch.bfloat16)
    ln = (1 + 0.1 * torch.randn(n, device=DEV, generator=g)).to(torch.bfloat16)
    res0 = torch.randn(m, n, device=DEV, generator=g).to(torch.bfloat16)
    y = ops.linear(x, w)
    res_a, xn_a = res0.clone(), torch.empty_like(res0)
    N.check(N.lib().mvb_fused_add_rmsnorm(xn_a.data_ptr(), res_a.data_ptr(), y.data_ptr(), ln.data_ptr(), m, n, 1e-6,
                                          0, N.NORM_MODEL, N.BF16, N.stream_handle()), "fadd")
    ws = torch.zeros(N.lib().mvb_gemm_workspace_bytes(m, n, k, 0), dtype=torch.uint8, device=DEV)
    _gemm_partials(x, w, ws)
    res_b, xn_b = res0.clone(), torch.empty_like(res0)
    N.check(N.lib().mvb_fused_add_rmsnorm_gemm(xn_b.data_ptr(), res_b.data_ptr(), ws.data_ptr(), m, n, k,
                                               ln.data_ptr(), 1e-6, 0, N.stream_handle()), "fadd gemm")
    assert torch.equal(res_a, res_b)
    a, b = xn_a.float(), xn_b.float()
    ulp = torch.ldexp(torch.ones_like(a), torch.frexp(a.abs().clamp_min(1e-30))[1] - 8)  # bf16 spacing at |a|
    assert bool(((a - b).abs() <= ulp).all())
    assert (a != b).float().mean().item() < 0.01


# ------------------------------------------------- QK-norm + RoPE + paged KV write
def _pool(L, P, nkv, D, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(L, 2, P + 1, 16, nkv, D, generator=g).to(torch.bfloat16)


def test_qk_norm_rope_kv_write_indexing_is_bit_exact():
    B, Hq, Hkv, D, L, P, layer = 6, 8, 4, 128, 3, 40, 1
    rng = random.Random(0)
    order = list(range(P))
    rng.shuffle(order)
    lens = [1, 15, 16, 17, 100, 33]       # positions cross block boundaries
    bts, it = [], iter(order)
    for n in lens:
        bts.append([next(it) for _ in range((n + 15) // 16)])
    mb = max(len(b) for b in bts)
    bt = torch.full((B, mb), P, dtype=torch.int32)
    for i, b in enumerate(bts):
        bt[i, :len(b)] = torch.tensor(b)
    pos = torch.tensor([n - 1 for n in lens], dtype=torch.int32)
    g = torch.Generator().manual_seed(1)
    qkv = torch.randn(B, (Hq + 2 * Hkv) * D, generator=g).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    cos, sin = om.rope_tables(D, 1e6, 256, torch.bfloat16)
    pool = _pool(L, P, Hkv, D, 2)
    pool_d = pool.to(DEV)
    q = ops.qk_norm_rope_kv_write(qkv.to(DEV), pool_d, layer, pos.to(DEV), bt.to(DEV), cos.to(DEV), sin.to(DEV),
                                  Hq, Hkv, qn.to(DEV), kn.to(DEV), 1e-6)
    # oracle: model.py:170-184 then _write_kv_cache (model.py:226-243)
    qo = qkv[:, :Hq * D].view(B, 1, Hq, D)
    ko = qkv[:, Hq * D:(Hq + Hkv) * D].view(B, 1, Hkv, D)
    vo = qkv[:, (Hq + Hkv) * D:].view(B, 1, Hkv, D).transpose(1, 2)
    qo = om.rms_norm(qo, qn, 1e-6).transpose(1, 2)
    ko = om.rms_norm(ko, kn, 1e-6).transpose(1, 2)
    c, s = cos[pos.long()].unsqueeze(1).unsqueeze(1), sin[pos.long()].unsqueeze(1).unsqueeze(1)
    qo, ko = om.apply_rope(qo, c, s), om.apply_rope(ko, c, s)
    expect = pool.clone()
    om.OracleDecoder.write_kv(expect, ko, vo, bts, pos.tolist(), layer)
    got = pool_d.cpu()
    changed_got = (got != pool).flatten(4).any(-1)
    changed_exp = (expect != pool).flatten(4).any(-1)
    assert torch.equal(changed_got, changed_exp)          # exactly the same slots written
    assert bf16_ulps(got, expect) <= 1
    assert bf16_ulps(q.cpu(), qo[:, :, 0]) <= 1


@pytest.mark.parametrize("B,qk_norm", [(64, True), (128, True), (128, False), (256, False)])
def test_qk_norm_rope_kv_write_from_split_k_partials_bit_exact(B, qk_norm):
    Hq, Hkv, D, L, H = 32, 8, 128, 2, 4096
    P = 5 * B
    g = torch.Generator(device=DEV).manual_seed(5)
    x = (torch.randn(B, H, device=DEV, generator=g) / math.sqrt(H)).to(torch.bfloat16)
    wqkv = torch.randn((Hq + 2 * Hkv) * D, H, device=DEV, generator=g).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(D, device=DEV, generator=g)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(D, device=DEV, generator=g)).to(torch.bfloat16)
    cos, sin = om.rope_tables(D, 1e6, 256, torch.bfloat16)
    cos, sin = cos.to(DEV), sin.to(DEV)
    pos = torch.randint(0, 64, (B,), device=DEV, dtype=torch.int32)
    bt = torch.randperm(P, device=DEV)[:B * 4].to(torch.int32).view(B, 4)
    if not qk_norm:   # Llama-family: no per-head norm
        qn = kn = None
    pool_a = torch.zeros(L, 2, P + 1, 16, Hkv, D, dtype=torch.bfloat16, device=DEV)
    pool_b = pool_a.clone()
    qkv = ops.linear(x, wqkv)
    q_a = ops.qk_norm_rope_kv_write(qkv, pool_a, 1, pos, bt, cos, sin, Hq, Hkv, qn, kn, 1e-6)
    ws = torch.zeros(N.lib().mvb_gemm_workspace_bytes(B, wqkv.shape[0], H, 0), dtype=torch.uint8, device=DEV)
    _gemm_partials(x, wqkv, ws)
    q_b = torch.empty_like(q_a)
    N.check(N.lib().mvb_qk_norm_rope_kv_write_gemm(
        q_b.data_ptr(), pool_b.data_ptr(), ws.data_ptr(), H, N.ptr(qn), N.ptr(kn), cos.data_ptr(),
        sin.data_ptr(), cos.shape[0], pos.data_ptr(), bt.data_ptr(), 4, B, Hq, Hkv, D, L, 1, P + 1, 16, 1e-6, 0,
        N.stream_handle()), "qk gemm")
    assert torch.equal(q_a, q_b) and torch.equal(pool_a, pool_b)


def test_kv_write_bad_block_is_reported_not_faulted():
    B, Hq, Hkv, D, L, P = 2, 4, 2, 128, 1, 8
    pool = torch.zeros(L, 2, P + 1, 16, Hkv, D, dtype=torch.bfloat16, device=DEV)
    bt = torch.tensor([[3], [P + 5]], dtype=torch.int32, device=DEV)   # second row: block id out of range
    pos = torch.tensor([0, 0], dtype=torch.int32, device=DEV)
    qkv = torch.randn(B, (Hq + 2 * Hkv) * D, device=DEV).to(torch.bfloat16)
    cos, sin = om.rope_tables(D, 1e6, 256, torch.bfloat16)
    ops.qk_norm_rope_kv_write(qkv, pool, 0, pos, bt, cos.to(DEV), sin.to(DEV), Hq, Hkv)
    assert N.device_status(clear=True) & N.DEV_BAD_BLOCK
    assert torch.count_nonzero(pool[0, :, 3]) > 0


# ------------------------------------------------------------ paged attention
def _attention_ref(q, pool, layer, bts, ctx, scale, softcap=0.0, window=0):
    """fp32 restatement of _read_kv_cache_batch + SDPA (model.py:191-221); ``softcap`` and
    ``window`` as Gemma-2 applies them (scores soft-capped before the mask; a sliding window
    keeps the newest ``window`` keys)."""
    B, Hq, D = q.shape
    Hkv = pool.shape[4]
    out = torch.empty(B, Hq, D)
    for b in range(B):
        k = torch.cat([pool[layer, 0, blk] for blk in bts[b]], 0)[:ctx[b]].float()   # [ctx, Hkv, D]
        v = torch.cat([pool[layer, 1, blk] for blk in bts[b]], 0)[:ctx[b]].float()
        lo = max(0, ctx[b] - window) if window else 0
        k = k[lo:].repeat_interleave(Hq // Hkv, dim=1)
        v = v[lo:].repeat_interleave(Hq // Hkv, dim=1)
        s = torch.einsum("hd,thd->ht", q[b].float(), k) * scale
        if softcap:
            s = softcap * torch.tanh(s / softcap)
        p = torch.softmax(s, -1)
        out[b] = torch.einsum("ht,thd->hd", p, v)
    return out


@pytest.mark.parametrize("Hq,Hkv,lens", [
    (32, 8, [2049] * 4 + [1, 16, 17, 300]),     # Qwen3-8B heads, mixed lengths incl. 1 token
    (16, 8, [129, 5, 64]),                      # Qwen3-0.6B heads
    (8, 4, [37, 50, 16, 64]),
    (32, 4, [700, 33]),                         # group 8 (Qwen3-30B-A3B heads)
    (4, 1, [513, 2, 31]),                       # one KV head per rank (TP=8 shard)
    # many blocks per CTA with several consumer warps per KV head (tensor-parallel shards):
    (16, 4, [2049] * 12 + [7, 300]),            # TP=2 shard of Qwen3-8B
    (8, 2, [1200] * 16),                        # TP=4 shard
    (4, 1, [2049] * 16),                        # TP=8 shard
    # Llama-3-8B heads, a batch of 128 with contexts drawn from 128-8192 (up to 513 blocks each)
    (32, 8, [128 + (7919 * i) % 8065 for i in range(128)]),
    # one long sequence: every CTA of the launch is a contributor to the same merge
    (32, 8, [40001]),
    (4, 1, [40001]),                            # two CTAs per SM: twice as many contributors
])
def test_paged_attention_matches_fp32_reference(Hq, Hkv, lens):
    D, L, layer = 128, 2, 1
    total_blocks = sum((n + 15) // 16 for n in lens)
    P = total_blocks + 7
    order = list(range(P))
    random.Random(5).shuffle(order)
    it = iter(order)
    bts = [[next(it) for _ in range((n + 15) // 16)] for n in lens]
    mb = max(len(b) for b in bts)
    bt = torch.full((len(lens), mb), P, dtype=torch.int32)
    for i, b in enumerate(bts):
        bt[i, :len(b)] = torch.tensor(b)
    pool = _pool(L, P, Hkv, D, 9)
    g = torch.Generator().manual_seed(4)
    q = torch.randn(len(lens), Hq, D, generator=g).to(torch.bfloat16)
    scale = 1.0 / math.sqrt(D)
    out = ops.paged_attention_decode(q.to(DEV), pool.to(DEV), layer, bt.to(DEV),
                                     torch.tensor(lens, dtype=torch.int32, device=DEV), scale)
    ref = _attention_ref(q, pool, layer, bts, lens, scale)
    torch.testing.assert_close(out.cpu().float(), ref, rtol=2e-2, atol=1e-2)
    out2 = ops.paged_attention_decode(q.to(DEV), pool.to(DEV), layer, bt.to(DEV),
                                      torch.tensor(lens, dtype=torch.int32, device=DEV), scale)
    assert torch.equal(out, out2)  # deterministic split-KV merge


@pytest.mark.parametrize("D,Hq,Hkv,lens,softcap,window", [
    (256, 16, 8, [8193] * 4 + [1, 16, 17, 300], 50.0, 0),     # Gemma-2-9B heads: global layer
    (256, 16, 8, [8193] * 4 + [1, 16, 17, 300], 50.0, 4096),  # ... sliding-window layer
    (256, 16, 8, [4096, 4097, 4111, 4112, 4113], 0.0, 4096),  # window edges around block bounds
    (256, 4, 2, [37, 50, 16, 64], 0.0, 0),                    # Gemma-3 test model heads
    (256, 2, 1, [2049] * 6 + [5], 50.0, 1000),                # one KV head (TP=8 shard), odd window
    (256, 32, 4, [700, 33], 30.0, 0),                         # group 8
    (128, 32, 8, [2049] * 3 + [1, 300], 50.0, 1024),          # head_dim 128 with both options
    (128, 8, 2, [1200] * 4, 0.0, 17),
])
def test_paged_attention_softcap_window_head_dim_256(D, Hq, Hkv, lens, softcap, window):
    L, layer = 2, 1
    total_blocks = sum((n + 15) // 16 for n in lens)
    P = total_blocks + 7
    order = list(range(P))
    random.Random(6).shuffle(order)
    it = iter(order)
    bts = [[next(it) for _ in range((n + 15) // 16)] for n in lens]
    mb = max(len(b) for b in bts)
    bt = torch.full((len(lens), mb), P, dtype=torch.int32)
    for i, b in enumerate(bts):
        bt[i, :len(b)] = torch.tensor(b)
    pool = _pool(L, P, Hkv, D, 10)
    g = torch.Generator().manual_seed(8)
    q = (torch.randn(len(lens), Hq, D, generator=g) * (6 if softcap else 1)).to(torch.bfloat16)  # scores ~ +-20
    scale = 1.0 / math.sqrt(D)
    ctx = torch.tensor(lens, dtype=torch.int32, device=DEV)
    out = ops.paged_attention_decode(q.to(DEV), pool.to(DEV), layer, bt.to(DEV), ctx, scale, softcap=softcap,
                                     window=window)
    assert N.device_status(clear=True) == 0
    ref = _attention_ref(q, pool, layer, bts, lens, scale, softcap, window)
    torch.testing.assert_close(out.cpu().float(), ref, rtol=2e-2, atol=1e-2)
    if softcap or (window and 2 * window <= max(lens)):   # the options change the result
        plain = _attention_ref(q, pool, layer, bts, lens, scale)
        assert (plain - ref).abs().max() > 5e-2
    out2 = ops.paged_attention_decode(q.to(DEV), pool.to(DEV), layer, bt.to(DEV), ctx, scale, softcap=softcap,
                                      window=window)
    assert torch.equal(out, out2)


# --------------------------------------------------------------------- sampling
def test_greedy_matches_torch_argmax(golden):
    logits = golden["samp_logits_bf16"]
    for t in (logits, logits.float()):
        assert torch.equal(ops.greedy_sample(t.to(DEV)).cpu(), golden["greedy"])


def test_sampling_row_layouts_and_ties():
    """The sampler reads a row as 16-byte vectors when the row is 16-byte aligned and element by
    element otherwise, with a ragged tail when the vocabulary is not a multiple of the vector
    width.  An odd vocabulary, column-sliced views (rows at every alignment) and maxima tied far
    apart (the lowest index wins) give the oracle's tokens in every layout."""
    g = torch.Generator().manual_seed(3)
    V = 151937
    base = torch.randn(4, V + 1, generator=g)
    base[0, 100] = base[0, 150001] = 9.0  # tied maxima in vectors far apart
    base[1, V - 1] = 9.0                  # the maximum in the ragged tail of the first view
    base[2, V] = 9.0                      # the last element of the second view
    for dt in (torch.bfloat16, torch.float32):
        xd = base.to(dt).to(DEV)
        for view in (xd[:, :V], xd[:, 1:]):
            host = view.float().cpu()
            assert torch.equal(ops.greedy_sample(view).cpu(), host.argmax(-1))
            for (T, k, p) in ((0.8, 50, 0.95), (1.3, 5, 1.0), (0.0, 50, 0.95)):
                tok = ops.sample(view, T, k, p, 7, 17).cpu()
                for r in range(4):
                    exp, margin = osamp.sample_row(host[r], T, k, p, 7, r, 17)
                    assert int(tok[r]) == exp or margin < 1e-5, (dt, T, k, p, r, int(tok[r]), exp, margin)
    assert N.device_status(clear=True) == 0


def _exact_nucleus_count(row: torch.Tensor, top_p: float) -> tuple[int, torch.Tensor]:
    """Tokens kept by top-p in exact (fp64) arithmetic, and the stable (value desc, index asc) order."""
    sv, si = torch.sort(row.double(), descending=True, stable=True)
    pr = torch.softmax(sv, -1)
    excl = torch.cumsum(pr, -1) - pr
    return int((excl < top_p).sum()), si


@pytest.mark.parametrize("k,p", [(50, 0.95), (50, 1.0), (1, 1.0), (5, 0.5)])
def test_filter_matches_oracle(golden, k, p):
    """Top-k (+ top-p over <= 2048 candidates): the kept set equals the oracle's with the
    lower-index tie rule, and its size equals the reference's own."""
    logits = golden["samp_logits_bf16"].float()
    got = torch.isfinite(ops.top_k_top_p_filter(logits.to(DEV), k, p).cpu())
    exp = torch.isfinite(osamp.top_k_top_p_filter(logits, k, p, stable=True))
    assert torch.equal(got, exp)
    ref_keep = np.unpackbits(golden[f"filter_k{k}_p{int(p * 100)}_kept_bits"].numpy(), axis=-1)[:, :logits.shape[1]]
    assert np.array_equal(got.sum(-1).numpy(), ref_keep.sum(-1))  # same count as the reference itself


def test_full_vocabulary_nucleus_is_exact_within_rounding(golden):
    """Top-p alone over 151936 tokens: the kernel's kept set is a prefix of the (value desc,
    index asc) order whose size matches exact fp64 arithmetic within 2 tokens.  (The reference's
    own fp32 cumsum over 152k terms carries ~2e-5 of mass error, i.e. a few tokens.)"""
    logits = golden["samp_logits_bf16"].float()
    got = torch.isfinite(ops.top_k_top_p_filter(logits.to(DEV), 0, 0.9).cpu())
    ref_keep = np.unpackbits(golden["filter_k0_p90_kept_bits"].numpy(), axis=-1)[:, :logits.shape[1]]
    for r in range(logits.shape[0]):
        n_exact, order = _exact_nucleus_count(logits[r], 0.9)
        n = int(got[r].sum())
        assert abs(n - n_exact) <= 2, (r, n, n_exact)
        assert bool(got[r][order[:n]].all())                      # a prefix of the sorted order
        assert abs(int(ref_keep[r].sum()) - n_exact) <= 16         # the reference is within its own rounding


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_sample_matches_oracle_draw(golden, dt):
    logits = golden["samp_logits_bf16"].float()
    V = logits.shape[1]
    x = logits.to(dt).to(DEV)
    mismatches = 0
    for seed in range(6):
        for (T, k, p) in ((0.8, 50, 0.95), (1.0, -1, 1.0), (0.7, -1, 0.9), (0.0, 50, 0.95), (1.3, 5, 1.0)):
            probs = torch.empty(4, V, device=DEV)
            tok = ops.sample(x, T, k, p, seed, 17, probs_out=probs).cpu()
            for r in range(4):
                exp, margin = osamp.sample_row(logits[r], T, k, p, seed, r, 17)
                if int(tok[r]) != exp:
                    assert margin < 1e-5, (seed, T, k, p, r, int(tok[r]), exp, margin)
                    mismatches += 1
            if T > 0:
                ref = osamp.gpu_semantics_probs(logits.double(), T, k, p)
                got_p = probs.cpu().double()
                both = (got_p > 0) & (ref > 0)
                torch.testing.assert_close(got_p[both], ref[both], rtol=1e-4, atol=1e-7)
                # survivors differ at most at a full-vocabulary top-p cutoff, by negligible mass
                assert float(got_p[~both].sum() + ref[~both].sum()) < 1e-3 * 4
    assert mismatches <= 1


def test_softmax_multinomial_follows_torch_seed(golden):
    logits = golden["samp_logits_bf16"].float().to(DEV)
    torch.manual_seed(123)
    a = ops.softmax_multinomial_sample(logits, 0.8)
    b = ops.softmax_multinomial_sample(logits, 0.8)
    torch.manual_seed(123)
    c = ops.softmax_multinomial_sample(logits, 0.8)
    assert torch.equal(a, c)
    assert 0 <= int(a.min()) and int(a.max()) < logits.shape[1]
    del b


def test_sample_distribution_is_statistically_right():
    V, rows = 8, 4096
    logits = torch.tensor([2.0, 1.0, 0.5, 0.0, -1.0, 0.3, 1.7, -0.2]).repeat(rows, 1).to(DEV)
    tok = ops.sample(logits, 1.0, -1, 1.0, seed=11, offset=0)
    freq = torch.bincount(tok.cpu(), minlength=V).double() / rows
    p = torch.softmax(logits[0].double().cpu(), -1)
    assert float((freq - p).abs().max()) < 0.03
