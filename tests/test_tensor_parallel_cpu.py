"""Host side of tensor parallelism, on the CPU with the gloo backend (world size 2).

The GPU path shards the weights with ``tensor_parallel.shard_state_dict`` and lets its kernels
sum the row-parallel outputs across ranks and gather the vocab-parallel logits.  Here two gloo
ranks run one decode step of a small Qwen3-family model in fp32 with exactly those shards,
replacing the kernels' exchanges with ``all_reduce`` / ``all_gather``, and must reproduce the
unsharded step: this pins the slicing (query heads <-> o_proj columns, KV heads <-> GQA groups,
gate/up rows <-> down_proj columns, vocab slices in rank order).  Also checked: every rank
plans the same heap layout, the signal points of one step are distinct, and the replicated FIFO
block allocator hands every rank the same block ids.
"""
import math
import os
import random
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llm_pytorch_inference_b200 import tensor_parallel as tpm
from llm_pytorch_inference_b200.configs import get_config, head_dim, num_kv_heads
from llm_pytorch_inference_b200.kv_cache import KVCacheManager
from llm_pytorch_inference_b200.weights import canonical_state_dict

CFG = dict(num_hidden_layers=2, hidden_size=256, num_attention_heads=8, num_key_value_heads=4,
           intermediate_size=512, vocab_size=1000)


def _rms(x, w, eps):
    return w * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps))


def _step(cfg, sd, x_ids, kcache, vcache, pos, reduce, gather, kv_heads, q_heads):
    """One decode token per row in fp32; kcache/vcache [L, B, T, kv_heads, D] hold positions < pos."""
    H, D, eps = cfg["hidden_size"], head_dim(cfg), cfg["rms_norm_eps"]
    group = q_heads // kv_heads
    B = x_ids.shape[0]
    res = sd["model.embed_tokens.weight"][x_ids]
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}."
        xn = _rms(res, sd[p + "input_layernorm.weight"], eps)
        q = (xn @ sd[p + "self_attn.q_proj.weight"].T).view(B, q_heads, D)
        k = (xn @ sd[p + "self_attn.k_proj.weight"].T).view(B, kv_heads, D)
        v = (xn @ sd[p + "self_attn.v_proj.weight"].T).view(B, kv_heads, D)
        q = _rms(q, sd[p + "self_attn.q_norm.weight"], eps)
        k = _rms(k, sd[p + "self_attn.k_norm.weight"], eps)
        K = torch.cat([kcache[i], k[:, None]], 1)              # [B, T+1, kv, D] (RoPE omitted: slicing test)
        V = torch.cat([vcache[i], v[:, None]], 1)
        Kq = K.repeat_interleave(group, dim=2)                  # GQA: query head h reads KV head h // group
        Vq = V.repeat_interleave(group, dim=2)
        s = torch.einsum("bhd,bthd->bht", q, Kq) / math.sqrt(D)
        o = torch.einsum("bht,bthd->bhd", s.softmax(-1), Vq).reshape(B, q_heads * D)
        res = res + reduce(o @ sd[p + "self_attn.o_proj.weight"].T)
        xn = _rms(res, sd[p + "post_attention_layernorm.weight"], eps)
        h = torch.nn.functional.silu(xn @ sd[p + "mlp.gate_proj.weight"].T) * (xn @ sd[p + "mlp.up_proj.weight"].T)
        res = res + reduce(h @ sd[p + "mlp.down_proj.weight"].T)
    xn = _rms(res, sd["model.norm.weight"], eps)
    return gather(xn @ sd["lm_head.weight"].T)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, results, nkv=4):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = get_config("qwen3-tiny", **dict(CFG, num_key_value_heads=nkv))
        sd = canonical_state_dict(cfg, seed=0, dtype=torch.float32)
        for k in sd:
            if k.endswith("norm.weight"):   # non-trivial norm weights
                sd[k] = 1 + 0.1 * torch.randn(sd[k].shape, generator=torch.Generator().manual_seed(len(k)))
        L, D = cfg["num_hidden_layers"], head_dim(cfg)
        hq, hkv = cfg["num_attention_heads"], num_kv_heads(cfg)
        B, T = 6, 5
        g = torch.Generator().manual_seed(3)
        ids = torch.randint(0, cfg["vocab_size"], (B,), generator=g)
        kc = torch.randn(L, B, T, hkv, D, generator=g)
        vc = torch.randn(L, B, T, hkv, D, generator=g)

        shard = tpm.shard_state_dict(cfg, sd, world, rank)
        kv0, lh = tpm.kv_head_range(cfg, world, rank)   # one replicated head when hkv < world

        def reduce(t):
            t = t.clone()
            dist.all_reduce(t)
            return t

        def gather(t):
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t.contiguous())
            return torch.cat(parts, -1)

        got = _step(cfg, shard, ids, kc[:, :, :, kv0:kv0 + lh], vc[:, :, :, kv0:kv0 + lh],
                    T, reduce, gather, lh, hq // world)
        want = _step(cfg, sd, ids, kc, vc, T, lambda t: t, lambda t: t, hkv, hq)
        err = float((got - want).abs().max())

        # heap plan, signal points, replicated allocator
        layout = tpm.plan_heap(33024, 64, 4096, 151936, 3 << 20, 6 << 20)
        layouts = [None] * world
        dist.all_gather_object(layouts, layout)
        pts = [f(i) for i in range(36) for f in (tpm.point_o_proj, tpm.point_attn_norm, tpm.point_down,
                                                  tpm.point_mlp_norm)] + [tpm.point_logits(36)]
        order = list(range(300))
        random.Random(0).shuffle(order)
        kv = KVCacheManager(300, 16, 2, 2, 128, device="cpu", free_order=order, allocate_pool=False)
        tabs = [kv.allocate(s, 17 + 23 * s) for s in range(8)]
        for _ in range(40):
            for s in range(8):
                kv.append_token(s)
        tabs = [kv.get_block_table(s) for s in range(8)]
        all_tabs = [None] * world
        dist.all_gather_object(all_tabs, tabs)
        results[rank] = {"err": err, "scale": float(want.abs().max()),
                         "layouts_equal": all(x == layouts[0] for x in layouts),
                         "points_distinct": len(set(pts)) == len(pts) and max(pts) < 1024,
                         "tables_equal": all(t == all_tabs[0] for t in all_tabs)}
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("nkv", [4, 1])
def test_sharded_step_reproduces_the_unsharded_step_on_two_gloo_ranks(nkv):
    """nkv = 1: fewer KV heads than ranks, the head is replicated and each rank keeps the query
    heads of its half of the GQA group."""
    world = 2
    with mp.get_context("spawn").Manager() as m:
        results = m.dict()
        mp.spawn(_worker, args=(world, _free_port(), results, nkv), nprocs=world, join=True)
        res = dict(results)
    for r in range(world):
        assert res[r]["err"] <= 1e-4 * max(1.0, res[r]["scale"]), res[r]
        assert res[r]["layouts_equal"] and res[r]["points_distinct"] and res[r]["tables_equal"], res[r]


def test_shard_shapes_and_divisibility():
    cfg = get_config("qwen3-8b", num_hidden_layers=1)
    shapes = {"model.layers.0.self_attn.q_proj.weight": (4096, 4096), "model.layers.0.self_attn.k_proj.weight":
              (1024, 4096), "model.layers.0.self_attn.v_proj.weight": (1024, 4096),
              "model.layers.0.self_attn.o_proj.weight": (4096, 4096), "model.layers.0.mlp.gate_proj.weight":
              (12288, 4096), "model.layers.0.mlp.up_proj.weight": (12288, 4096),
              "model.layers.0.mlp.down_proj.weight": (4096, 12288), "lm_head.weight": (151936, 4096),
              "model.embed_tokens.weight": (151936, 4096)}
    sd = {k: torch.empty(s, dtype=torch.bfloat16, device="meta") for k, s in shapes.items()}
    out = tpm.shard_state_dict(cfg, sd, 8, 3)
    assert out["model.layers.0.self_attn.q_proj.weight"].shape == (512, 4096)
    assert out["model.layers.0.self_attn.k_proj.weight"].shape == (128, 4096)
    assert out["model.layers.0.self_attn.o_proj.weight"].shape == (4096, 512)
    assert out["model.layers.0.mlp.gate_proj.weight"].shape == (1536, 4096)
    assert out["model.layers.0.mlp.down_proj.weight"].shape == (4096, 1536)
    assert out["lm_head.weight"].shape == (18992, 4096)
    assert out["model.embed_tokens.weight"].shape == (151936, 4096)     # replicated
    assert tpm.local_config(cfg, 8)["num_key_value_heads"] == 1
    with pytest.raises(ValueError):
        tpm.check_divisible(cfg, 3)


def test_gemma2_shard_shapes():
    """Gemma-2-9B at TP=2: head dim 256, query heads and o_proj columns split, KV heads split, the
    sandwich norms replicated, vocab-parallel lm_head (tied to the embedding, which stays whole)."""
    from llm_pytorch_inference_b200.weights import weight_shapes

    cfg = get_config("gemma2-9b", num_hidden_layers=1)
    sd = {k: torch.empty(s, dtype=torch.bfloat16, device="meta") for k, s in weight_shapes(cfg).items()}
    out = tpm.shard_state_dict(cfg, sd, 2, 1)
    H, D, V = cfg["hidden_size"], head_dim(cfg), cfg["vocab_size"]
    nq, nkv, inter = cfg["num_attention_heads"], num_kv_heads(cfg), cfg["intermediate_size"]
    p = "model.layers.0."
    assert out[p + "self_attn.q_proj.weight"].shape == (nq // 2 * D, H)
    assert out[p + "self_attn.k_proj.weight"].shape == (nkv // 2 * D, H)
    assert out[p + "self_attn.v_proj.weight"].shape == (nkv // 2 * D, H)
    assert out[p + "self_attn.o_proj.weight"].shape == (H, nq // 2 * D)
    assert out[p + "mlp.gate_proj.weight"].shape == (inter // 2, H)
    assert out[p + "mlp.down_proj.weight"].shape == (H, inter // 2)
    for norm in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                 "post_feedforward_layernorm"):
        assert out[p + norm + ".weight"].shape == (H,)
    assert out["model.embed_tokens.weight"].shape == (V, H)
    assert "lm_head.weight" not in sd and out["lm_head.weight"].shape == (V // 2, H)   # cut from the tied table
    assert tpm.local_config(cfg, 2)["num_key_value_heads"] == nkv // 2


def _moe_block(sd, p, xn, top_k, first, count):
    """The sparse MoE block of layer prefix ``p`` in fp32 over the experts ``first .. first+count-1``
    only (the state dict holds them as local experts 0 .. count-1); routing over all experts."""
    from oracle.model import moe_route

    topw, topi = moe_route(xn @ sd[p + "mlp.gate.weight"].T, top_k)
    out = torch.zeros_like(xn)
    for b in range(xn.shape[0]):
        for k in range(top_k):
            e = int(topi[b, k])
            if not first <= e < first + count:
                continue
            q = f"{p}mlp.experts.{e - first}."
            h = torch.nn.functional.silu(xn[b] @ sd[q + "gate_proj.weight"].T) * (xn[b] @ sd[q + "up_proj.weight"].T)
            out[b] += topw[b, k] * (h @ sd[q + "down_proj.weight"].T)
    return out


def _moe_worker(rank, world, port, results):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = get_config("qwen3-moe-tiny", num_hidden_layers=1)
        sd = canonical_state_dict(cfg, seed=0, dtype=torch.float32)
        xn = torch.randn(8, cfg["hidden_size"], generator=torch.Generator().manual_seed(5))
        E, K = cfg["num_experts"], cfg["num_experts_per_tok"]
        first, count = tpm.expert_range(cfg, world, rank)
        shard = tpm.shard_state_dict(cfg, sd, world, rank)
        p = "model.layers.0."
        same = all(torch.equal(shard[f"{p}mlp.experts.{j}.{w}_proj.weight"], sd[f"{p}mlp.experts.{first + j}.{w}_proj.weight"])
                   for j in range(count) for w in ("gate", "up", "down"))
        extra = any(f"{p}mlp.experts.{j}.gate_proj.weight" in shard for j in range(count, E))
        part = _moe_block(shard, p, xn, K, first, count)   # this rank's experts only
        dist.all_reduce(part)                               # the owners' sum of the pushed partials
        want = _moe_block(sd, p, xn, K, 0, E)
        results[rank] = {"err": float((part - want).abs().max()), "scale": float(want.abs().max()),
                         "same": same, "extra": extra, "router": torch.equal(shard[p + "mlp.gate.weight"],
                                                                              sd[p + "mlp.gate.weight"])}
    finally:
        dist.destroy_process_group()


def test_expert_parallel_moe_block_reproduces_the_unsharded_block_on_two_gloo_ranks():
    """Expert parallelism of the sparse MoE block: each rank keeps the router and its contiguous
    share of the experts (renumbered from 0); the sum over ranks of each rank's experts'
    contributions is the unsharded block (fp32, up to summation order)."""
    world = 2
    with mp.get_context("spawn").Manager() as m:
        results = m.dict()
        mp.spawn(_moe_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        res = dict(results)
    for r in range(world):
        assert res[r]["same"] and not res[r]["extra"] and res[r]["router"], res[r]
        assert res[r]["err"] <= 1e-5 * max(1.0, res[r]["scale"]), res[r]


def test_moe_shard_shapes():
    """Qwen3-30B-A3B-arch experts at TP=4: 32 whole experts per rank (stacked and per-expert keys),
    the router replicated, attention split by heads; a split that cuts experts is refused."""
    from llm_pytorch_inference_b200.weights import stacked_expert_shapes

    cfg = get_config("qwen3-30b-a3b", num_hidden_layers=1)
    sd = {k: torch.empty(s, dtype=torch.bfloat16, device="meta") for k, s in stacked_expert_shapes(cfg).items()}
    out = tpm.shard_state_dict(cfg, sd, 4, 2)
    p = "model.layers.0."
    assert out[p + "mlp.experts.gate_up_proj.weight"].shape == (32, 2 * 768, 2048)
    assert out[p + "mlp.experts.down_proj.weight"].shape == (32, 2048, 768)
    assert out[p + "mlp.gate.weight"].shape == (128, 2048)
    assert out[p + "self_attn.q_proj.weight"].shape == (8 * 128, 2048)
    assert tpm.expert_range(cfg, 4, 2) == (64, 32)
    assert tpm.local_config(cfg, 4)["num_experts"] == 32
    with pytest.raises(ValueError):
        tpm.check_divisible(dict(cfg, num_experts=130), 4)


def test_kv_heads_replicate_when_fewer_than_ranks():
    """Qwen3-30B-A3B-arch at TP=8: 4 KV heads, each on two ranks; rank r keeps query heads
    4r .. 4r+3 and KV head r // 2, whose GQA group (8 query heads) holds them."""
    from llm_pytorch_inference_b200.weights import stacked_expert_shapes

    cfg = get_config("qwen3-30b-a3b", num_hidden_layers=1)
    sd = {k: torch.arange(s[0], dtype=torch.float32).view(-1, *([1] * (len(s) - 1))).expand(s)
          for k, s in stacked_expert_shapes(cfg).items() if "self_attn" in k or k == "lm_head.weight"}
    for r in range(8):
        out = tpm.shard_state_dict(cfg, sd, 8, r)
        k = out["model.layers.0.self_attn.k_proj.weight"]
        assert k.shape == (128, 2048) and int(k[0, 0]) == (r // 2) * 128
        q = out["model.layers.0.self_attn.q_proj.weight"]
        assert q.shape == (512, 2048) and int(q[0, 0]) == r * 512
        assert (r * 4) // 8 == r // 2       # the rank's first query head is in KV head r // 2's group
    assert tpm.local_kv_heads(cfg, 8) == 1 and tpm.kv_head_range(cfg, 8, 5) == (2, 1)
    assert tpm.kv_head_range(cfg, 2, 1) == (2, 2)
    with pytest.raises(ValueError):
        tpm.check_divisible(dict(cfg, num_key_value_heads=3, num_attention_heads=24), 8)
