"""One rank of the tensor-parallel parity run (launched by tests/test_tensor_parallel_gpu.py via
torch.distributed.run, one process per GPU).

Every rank builds the same 2-layer model (Qwen3-8B, or with --arch the Gemma-2-9B or the sparse-MoE
Qwen3-30B-A3B layer dims, experts split over the ranks) and the same batch of sequences on a shuffled block pool, and decodes with the
tensor-parallel engine (with --fused, its one-launch-per-layer-tail step).  Rank 0 also decodes the
same workload on one GPU (TP=1) and compares, step by step under teacher forcing, the full
logits and the greedy tokens; it writes a JSON report to --out.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import random
import sys
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from llm_pytorch_inference_b200 import _native as N  # noqa: E402
from llm_pytorch_inference_b200 import tensor_parallel as tpm  # noqa: E402
from llm_pytorch_inference_b200.configs import get_config, num_kv_heads  # noqa: E402
from llm_pytorch_inference_b200.engine import DecodeEngine  # noqa: E402
from llm_pytorch_inference_b200.tensor_parallel import TensorParallelConfig  # noqa: E402
from llm_pytorch_inference_b200.weights import canonical_state_dict  # noqa: E402


def build(cfg, tp, dev, batch, lens, num_blocks, fused=False, prefill=False):
    """The engine with its sequences' prompts in the KV pool: synthetic K/V (the same on every
    configuration), or with ``prefill`` the engine's own batched prefill of the prompts, whose
    last-token logits are kept in ``eng.last_prefill_logits``."""
    sd = canonical_state_dict(cfg, seed=0, dtype=torch.bfloat16, device=dev)
    order = list(range(num_blocks))
    random.Random(0).shuffle(order)
    eng = DecodeEngine(cfg, sd, max_batch=batch, max_model_len=max(lens) + 64, num_blocks=num_blocks, device=dev,
                       free_order=order, tp=tp, fused_layers=fused)
    del sd
    g = torch.Generator().manual_seed(1)
    if prefill:
        prompts = {s: torch.randint(0, cfg["vocab_size"], (n,), generator=g).tolist() for s, n in enumerate(lens)}
        eng.prefill(prompts)
        eng.set_sampling(0.0, -1, 1.0)
        eng.prepare_first_step()
        return eng
    for s, n in enumerate(lens):
        eng.add_sequence(s, torch.randint(0, cfg["vocab_size"], (n,), generator=g).tolist())
        eng.append_first_token(s, int(torch.randint(0, cfg["vocab_size"], (1,), generator=g)))
    # identical prompt K/V on every configuration: fill the full-head pool on the CPU, slice heads
    T, r = tp.tp_size, tp.rank
    kv0, hkv = tpm.kv_head_range(cfg, T, r)
    gk = torch.Generator().manual_seed(2)
    for s in range(len(lens)):
        for blk in eng.kv.get_block_table(s):
            full = torch.randn(cfg["num_hidden_layers"], 2, 16, num_kv_heads(cfg), eng.kv.head_dim, generator=gk)
            eng.kv.kv_cache[:, :, blk] = full[:, :, :, kv0:kv0 + hkv].to(dev, torch.bfloat16)
    eng.set_sampling(0.0, -1, 1.0)
    eng.prepare_first_step()
    return eng


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--arch", default="qwen3-8b", choices=["qwen3-8b", "gemma2-9b", "qwen3-30b-a3b"])
    ap.add_argument("--fused", action="store_true", help="the tensor-parallel step with one launch per layer tail")
    ap.add_argument("--kv-heads", type=int, default=None,
                    help="override the KV head count (1: fewer KV heads than ranks, each replicated)")
    ap.add_argument("--q-heads", type=int, default=None, help="override the query head count")
    ap.add_argument("--prefill", action="store_true", help="prompts through the batched prefill, compared too")
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    N.set_pdl(True)
    over = {} if args.kv_heads is None else {"num_key_value_heads": args.kv_heads}
    if args.q_heads is not None:
        over["num_attention_heads"] = args.q_heads
    cfg = get_config(args.arch, num_hidden_layers=2, **over)
    batch = 16
    lens = [37 + 29 * i for i in range(batch)]          # ragged contexts, blocks cross boundaries
    num_blocks = 512
    eng = build(cfg, TensorParallelConfig(world, rank), dev, batch, lens, num_blocks, fused=args.fused,
                prefill=args.prefill)
    ref = None
    if rank == 0:
        ref = build(cfg, TensorParallelConfig(1, 0), dev, batch, lens, num_blocks, prefill=args.prefill)
    report = {"steps": [], "tables_equal": True}
    if args.prefill and rank == 0:
        a, b = eng.last_prefill_logits.float(), ref.last_prefill_logits.float()
        d = (a - b).abs()
        top2 = b.topk(2, dim=-1).values
        ta, tb = [eng.output_tokens(s)[0] for s in range(batch)], [ref.output_tokens(s)[0] for s in range(batch)]
        report["prefill"] = {"max_abs": float(d.max()), "mean_abs": float(d.mean()),
                             "bad_token_rows": [i for i in range(batch) if ta[i] != tb[i] and
                                                float(top2[i, 0] - top2[i, 1]) > 2 * float(d[i].max())]}
        obj = [tb]
    else:
        obj = [None]
    if args.prefill:   # both continue from TP=1's first tokens
        dist.broadcast_object_list(obj, src=0)
        eng.force_last_tokens(obj[0])
        if ref is not None:
            ref.force_last_tokens(obj[0])
    for step in range(args.steps):
        moe = bool(cfg.get("num_experts"))
        if moe:   # every layer's routing, to tell a near-tie expert swap from an error
            routes = {id(eng): [], id(ref): []} if ref is not None else {id(eng): []}
            for e_ in ([eng, ref] if ref is not None else [eng]):
                r_ = e_.runner
                r_._moe_mlp_plain = getattr(r_, "_moe_mlp_plain", r_._moe_mlp)

                def hooked(i, r_=r_, key=id(e_)):
                    r_._moe_mlp_plain(i)
                    routes[key].append((r_.topk_ids.clone(), r_.topk_w.clone()))
                r_._moe_mlp = hooked
        toks = eng.step(use_graph=step > 0 and not moe)
        tabs = [eng.kv.get_block_table(s) for s in range(batch)]
        all_tabs = [None] * world
        dist.all_gather_object(all_tabs, tabs)
        report["tables_equal"] &= all(t == all_tabs[0] for t in all_tabs)
        if rank == 0:
            want = ref.step(use_graph=step > 0 and not moe)
            a = eng.runner.logits.float()
            b = ref.runner.logits.float()
            d = (a - b).abs()
            top2 = b[:batch].topk(2, dim=-1).values
            margin = (top2[:, 0] - top2[:, 1]).tolist()
            # a greedy token may only differ where TP=1's own top-2 margin is within the logit noise
            bad = [i for i in range(batch) if toks[i] != want[i] and margin[i] > 2 * float(d[i].max())]
            flips = []
            if moe:   # a row's expert mix differs: another top-k set, or a weight moved by > 0.01
                for (ia, wa), (ib, wb) in zip(routes[id(eng)], routes[id(ref)]):
                    for i in range(batch):
                        ma = dict(zip(ia[i].tolist(), wa[i].tolist()))
                        mb = dict(zip(ib[i].tolist(), wb[i].tolist()))
                        if set(ma) != set(mb) or max(abs(ma[e] - mb[e]) for e in ma) > 1e-2:
                            flips.append(i)
            report["steps"].append({"max_abs": float(d.max()), "mean_abs": float(d.mean()),
                                    "routing_differs_rows": sorted(set(flips)),
                                    "row_max_abs": [round(float(x), 4) for x in d[:batch].amax(-1)],
                                    "row_mean_abs": [float(x) for x in d[:batch].mean(-1)],
                                    "tokens_tp": toks, "tokens_ref": want, "bad_token_rows": bad,
                                    "tables_ref_equal": tabs == [ref.kv.get_block_table(s) for s in range(batch)]})
            forced = want
        else:
            forced = None
        obj = [forced]
        dist.broadcast_object_list(obj, src=0)
        eng.force_last_tokens(obj[0])            # teacher forcing: both continue from TP=1's tokens
        if rank == 0:
            ref.force_last_tokens(obj[0])
    report["device_status"] = N.device_status(clear=True)
    statuses = [None] * world
    dist.all_gather_object(statuses, report["device_status"])
    report["all_status"] = statuses
    dist.barrier()
    eng.runner.close()
    if ref is not None:
        ref.runner.close()
    if rank == 0:
        Path(args.out).write_text(json.dumps(report))
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
