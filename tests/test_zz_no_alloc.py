"""The allocation-free paged-attention entry point, through the C ABI.

Callers that cannot allocate device memory (a runtime binding the C ABI with no device
allocator of its own, or a server that has committed all of HBM to the KV pool) use
mvb_paged_attention_decode_noalloc, whose split-KV scratch is a fixed area inside the
library.  Its result must match mvb_paged_attention_decode with a caller workspace, on two
calls in a row (the second sees whatever the first left in the shared area), and a shape
beyond the area's limit must be refused with a clear message.
This file is collected last on purpose; it also passes when run alone.
"""
import math
import random

import pytest
import torch

from llm_pytorch_inference_b200 import _native as N

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(Hq, Hkv, lens, seed):
    D, L, layer = 128, 2, 1
    P = sum((n + 15) // 16 for n in lens) + 5
    order = list(range(P))
    random.Random(seed).shuffle(order)
    it = iter(order)
    bts = [[next(it) for _ in range((n + 15) // 16)] for n in lens]
    mb = max(len(b) for b in bts)
    bt = torch.full((len(lens), mb), P, dtype=torch.int32)
    for i, b in enumerate(bts):
        bt[i, :len(b)] = torch.tensor(b)
    g = torch.Generator().manual_seed(seed)
    pool = torch.randn(L, 2, P + 1, 16, Hkv, D, generator=g).to(torch.bfloat16).to(DEV)
    q = torch.randn(len(lens), Hq, D, generator=g).to(torch.bfloat16).to(DEV)
    return dict(q=q, pool=pool, bt=bt.to(DEV), ctx=torch.tensor(lens, dtype=torch.int32, device=DEV),
                Hq=Hq, Hkv=Hkv, D=D, L=L, layer=layer, P=P + 1, scale=1.0 / math.sqrt(D))


def _args(c, out):
    B = c["q"].shape[0]
    return (out.data_ptr(), out.stride(0), c["q"].data_ptr(), c["q"].stride(0), c["pool"].data_ptr(),
            c["bt"].data_ptr(), c["bt"].shape[1], c["ctx"].data_ptr(), B, c["Hq"], c["Hkv"], c["D"], c["L"],
            c["layer"], c["P"], 16, c["scale"])


def _with_workspace(c):
    lib = N.load()
    out = torch.empty_like(c["q"])
    need = lib.mvb_paged_attention_workspace_bytes(c["q"].shape[0], c["Hq"], c["D"], 0)
    ws = torch.zeros(need, dtype=torch.uint8, device=DEV)
    N.check(lib.mvb_paged_attention_decode(*_args(c, out), ws.data_ptr(), ws.numel(), N.stream_handle()),
            "mvb_paged_attention_decode")
    return out


def _no_alloc(c):
    lib = N.load()
    out = torch.empty_like(c["q"])
    N.check(lib.mvb_paged_attention_decode_noalloc(*_args(c, out), N.stream_handle()),
            "mvb_paged_attention_decode_noalloc")
    return out


def test_no_alloc_attention_matches_workspace_version_on_two_calls():
    N.device_status(clear=True)
    # first call: Qwen3-8B heads, long and short contexts (sequences split across many CTAs)
    a = _case(32, 8, [2049, 700, 1, 33, 300, 16, 17, 1200], seed=1)
    got_a = _no_alloc(a)
    ref_a = _with_workspace(a)
    torch.testing.assert_close(got_a.float(), ref_a.float(), rtol=2e-2, atol=1e-2)
    # second call straight after, different shape and batch: the area still holds the first
    # call's partials; 100 sequences need 400 bytes of per-sequence counters, so the counter area
    # (at the tail) is twice the first call's 256 bytes and starts 256 bytes lower
    lens = [129, 5, 64, 4000, 2] + [1 + (37 * i) % 300 for i in range(95)]
    b = _case(16, 8, lens, seed=2)
    got_b = _no_alloc(b)
    ref_b = _with_workspace(b)
    torch.testing.assert_close(got_b.float(), ref_b.float(), rtol=2e-2, atol=1e-2)
    assert N.device_status(clear=True) == 0


def test_no_alloc_attention_refuses_shapes_beyond_its_scratch():
    c = _case(64, 8, [40, 40], seed=3)      # 64 query heads need ~9.7 MB of scratch > 6 MiB
    out = torch.empty_like(c["q"])
    rc = N.load().mvb_paged_attention_decode_noalloc(*_args(c, out), N.stream_handle())
    assert rc == 2
    assert b"built-in area holds" in N.load().mvb_last_error()
