"""Decode throughput of the Qwen3-8B-architecture workload on the B200 decode path.

Workload (one decode step = one new token for each of 64 sequences):
  Qwen3-8B architecture (36 layers, hidden 4096, 32 q / 8 kv heads, head_dim 128,
  SwiGLU 12288, vocab 151936, QK-norm, RoPE theta 1e6), random-init bf16 weights,
  batch 64, prompts of 2048 tokens whose K/V are pre-filled with seeded random values
  in a shuffled paged pool (block 16, pool sized to the 180 GB per-GPU budget),
  sampling T=0.8 / top-k 50 / top-p 0.95.

Reported (one JSON line from rank 0):
  value     tokens/s of the whole job: K graph replays of the full step (forward + sampling),
            the per-step metadata already resident in HBM, CUDA events on the launching stream,
            max over ranks.  Weights (15.1 GB) + KV (~20 GB) per step >> L2 (126 MB).
  e2e       the same through DecodeEngine.run_steps(K): per step one host->device copy of the
            step's metadata from pinned memory and one device->host read of the 64 sampled tokens
            (with no sequence able to finish, each step is launched before the previous step's
            tokens are read back, and the host's bookkeeping overlaps the GPU).
  roofline  the kernel with the largest share of the step, its algorithmic bytes / average
            launch duration (CUDA events, launching stream) against the measured HBM peak.
  cpu_baseline  the oracle (the reference's PyTorch decode path restated on the CPU) on this
            host's cores, on a bounded sample of the same step, extrapolated to 36 layers.

--impl reference runs only that CPU path (rank 0), as the reference arm.
--gpus N (under torchrun): one tensor-parallel group of N GPUs over the same batch-64 workload
(strong scaling: the total work is fixed; value is the group's tokens/s, timed as the max over
ranks).
"""
from __future__ import annotations

import argparse
import json
import os
import random
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "decode tokens/s Qwen3-8B-arch bf16 at TP=1/2/4/8; paged-attn HBM GB/s % peak"
ARCH = "qwen3-8b"
BATCH = 64
PROMPT = 2048
SAMPLING = (0.8, 50, 0.95)


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--layers", type=int, default=None, help="override layer count (debug only; invalid bench)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--pdl", type=int, default=1)
    ap.add_argument("--fused-layers", type=int, default=0,
                    help="1: one persistent launch per layer tail (mvb_decoder_layer_tail / its tensor-parallel form)")
    ap.add_argument("--case", default=None, choices=["kernels", "moe", "gemma2", "llama3", "prefill", "prefill-kernels",
                                                     "reference-gpu"],
                    help="kernels: small profiling case (2 layers of the workload's dims), each kernel kind "
                         "launched a few times; prints per-kernel timings only.  moe: the sparse-MoE decode "
                         "workload (Qwen3-30B-A3B arch, batch 32, prompt 4096, greedy), 1 GPU.  gemma2: the "
                         "Gemma-2-9B-arch decode workload (batch 16, prompt 8192, greedy), 1 GPU.  prefill: "
                         "batched prefill of the headline's 64 x 2048-token prompts (Qwen3-8B arch), 1 GPU.  "
                         "prefill-kernels: small profiling case of the prefill (2 layers at Qwen3-8B dims, "
                         "8 x 2048-token prompts, ~5 GB on the device).  reference-gpu (with --impl reference): "
                         "the secondary baseline, the reference's PyTorch decode step and GPU sampling on cuda:0")
    ap.add_argument("--arch", default=None, choices=["qwen3-8b", "gemma2-9b"],
                    help="--case kernels: the layer dims (qwen3-8b: batch 64, prompt 2048; gemma2-9b: batch 16, "
                         "prompt 8192)")
    return ap.parse_args(argv)


# ------------------------------------------------------------------ distributed
def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# ----------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clock / throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"mvb_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "100"], stdout=self.fh,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.fh.close()
        rows = [r.split(",") for r in self.path.read_text().strip().splitlines() if r.count(",") >= 8]
        self.path.unlink(missing_ok=True)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        mx = max(float(r[2]) for r in rows)
        under = [s for s in sm if s > 0.5 * mx] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip().lower() == "active"})
        return {"sm_mhz": statistics.median(under), "sm_max_mhz": mx, "reasons": reasons, "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows)}


def peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def ncu_traffic() -> dict:
    """DRAM bytes per launch from the committed ncu summaries: lines
    ``traffic <kernel> <dram bytes per launch> <algorithmic bytes per launch of the captured case>``.
    Returns kernel -> (traffic, case algorithmic bytes); the caller scales the traffic to its own
    launch by the units processed (the ratio of algorithmic bytes)."""
    out = {}
    for f in sorted((REPO / "profiles").glob("*.md")):
        for line in f.read_text().splitlines():
            parts = line.strip().strip("`").split()
            if len(parts) == 4 and parts[0] == "traffic":
                try:
                    out[parts[1]] = (float(parts[2]), float(parts[3]))
                except ValueError:
                    pass
    return out


# -------------------------------------------------------------------- CPU oracle
def cpu_baseline(warmup: int = 1, steps: int = 1, layers: int = 36) -> dict:
    """The oracle's decode step (the reference's PyTorch decode path restated, CPU, bf16, all host
    threads) on the headline workload: every one of the 36 Qwen3-8B layers, batch 64, context 2048,
    final norm, lm_head and T/top-k/top-p sampling; ``warmup`` untimed then ``steps`` timed steps.
    Each layer has its own weights and its own KV pages (host memory as on the GPU: ~16 GB of
    weights, ~20 GB of KV).  Set-up draws one layer's weights and one layer's pages from seeded
    N(0, 0.02) / N(0, 1) and copies them into the others: the CPU's arithmetic and memory traffic
    do not depend on the values, and a full draw would take minutes."""
    from llm_pytorch_inference_b200.configs import get_config
    from oracle import sampling as osamp
    from oracle.model import OracleDecoder

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    cfg = get_config(ARCH, num_hidden_layers=layers)
    V, H, I = cfg["vocab_size"], cfg["hidden_size"], cfg["intermediate_size"]
    bf = torch.bfloat16
    t_setup = time.perf_counter()
    src = torch.empty(1 << 22, dtype=bf).normal_(0, 1, generator=g)   # seeded N(0, 1) values to tile

    def filled(shape, std):
        t = torch.empty(shape, dtype=bf)
        flat, n = t.view(-1), src.numel()
        for o in range(0, flat.numel(), n):
            m = min(n, flat.numel() - o)
            flat[o:o + m].copy_(src[:m])
        return t.mul_(std) if std != 1.0 else t

    sd = {"model.embed_tokens.weight": filled((V, H), 0.02), "lm_head.weight": filled((V, H), 0.02),
          "model.norm.weight": torch.ones(H, dtype=bf)}
    shapes = {"self_attn.q_proj.weight": (4096, H), "self_attn.k_proj.weight": (1024, H),
              "self_attn.v_proj.weight": (1024, H), "self_attn.o_proj.weight": (H, 4096),
              "mlp.gate_proj.weight": (I, H), "mlp.up_proj.weight": (I, H), "mlp.down_proj.weight": (H, I)}
    first = {k: filled(shp, 0.02) for k, shp in shapes.items()}
    for i in range(layers):
        p = f"model.layers.{i}."
        for k in shapes:
            sd[p + k] = first[k] if i == 0 else first[k].clone()
        for k in ("self_attn.q_norm.weight", "self_attn.k_norm.weight"):
            sd[p + k] = torch.ones(128, dtype=bf)
        for k in ("input_layernorm.weight", "post_attention_layernorm.weight"):
            sd[p + k] = torch.ones(H, dtype=bf)
    model = OracleDecoder(cfg, sd, bf)
    nblk = (PROMPT + 16) // 16 + 1
    pool = torch.empty(layers, 2, BATCH * nblk, 16, 8, 128, dtype=bf)
    pool[0].copy_(filled(pool.shape[1:], 1.0))
    for i in range(1, layers):
        pool[i].copy_(pool[0])
    bts = [list(range(b * nblk, (b + 1) * nblk)) for b in range(BATCH)]
    ids = torch.randint(0, V, (BATCH, 1), generator=g)
    pos = [PROMPT] * BATCH
    mask = torch.zeros(BATCH, 1, 1, PROMPT + 1, dtype=bf)
    setup_s = time.perf_counter() - t_setup
    samples = []
    for it in range(warmup + steps):
        t0 = time.perf_counter()
        with torch.no_grad(), torch.autocast("cpu", dtype=bf):
            logits = model.forward(ids, torch.tensor(pos).view(BATCH, 1), pool, bts, pos, use_cache=True,
                                   num_cached=pos, attn_mask=mask)[:, -1].float()
        for b in range(BATCH):
            osamp.sample_row(logits[b], *SAMPLING, seed=0, row=b, offset=it)
        if it >= warmup:
            samples.append(time.perf_counter() - t0)
    step_s = statistics.median(samples)
    del model, pool, sd, first
    return {"value": BATCH / step_s, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": (f"{steps} full batch-{BATCH} decode step(s) at context {PROMPT} through all {layers} Qwen3-8B "
                       f"layers + norm + lm_head + T/top-k/top-p sampling (oracle, bf16, CPU) after {warmup} "
                       f"warm-up step(s): {step_s:.2f} s/step (set-up {setup_s:.1f} s)"),
            "step_s": [round(x, 3) for x in samples], "cpu_model": _cpu_model()}


def _cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args, rank: int, world: int) -> None:
    """The reference arm: the reference's decode step on this host's CPU cores (the oracle, its
    PyTorch path restated), full 36-layer steps.  A step takes ~15 s on 16 cores, so the run is
    bounded: one warm-up step and min(steps, 3) timed steps, named in the line."""
    if rank != 0:
        return
    K = max(1, min(args.steps, 3))
    last = cpu_baseline(warmup=1, steps=K)
    v = last["value"]
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": K, "warmup": 1, "ms_per_step": BATCH / v * 1000.0, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{ARCH} decode, batch {BATCH}, prompt {PROMPT}, T/top-k/top-p "
                                   f"{SAMPLING[0]}/{SAMPLING[1]}/{SAMPLING[2]}",
                       "model": ARCH, "layers": 36, "global_batch": BATCH, "seq_len": PROMPT,
                       "parallelism": "cpu"},
            "cpu_baseline": {k: last[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_reference_gpu(args) -> None:
    """Secondary baseline: the reference's own GPU path on this B200, restated by the oracle --
    the PyTorch decode step of models/model.py as engine.py:339-349 runs it (bf16 autocast, cuBLAS
    projections, SDPA over the pages gathered through the block tables) on the headline workload
    (36 layers, batch 64, 2048-token contexts, zero-filled KV pages: the values do not change the
    work), and the reference's GPU sampling (sampler.py:40-48 filter + ops/sampling.py:69-73
    tempered softmax, torch.multinomial draw) against mvb_sample on the same bf16 logits.  The
    reference's CUDA extension needs libtorch's ATen headers and libraries to build, so it is not
    built here; its sampling kernel is the path this replaces."""
    from llm_pytorch_inference_b200 import ops
    from llm_pytorch_inference_b200.configs import get_config
    from llm_pytorch_inference_b200.weights import canonical_state_dict
    from oracle import sampling as osamp
    from oracle.engine import OracleEngine

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = get_config(ARCH)
    sd = canonical_state_dict(cfg, seed=0, dtype=torch.bfloat16, device=dev)
    K = max(1, min(args.steps, 3))
    per_seq = (PROMPT + 1 + 2 + K + 15) // 16 + 1
    blocks = BATCH * per_seq + 8
    order = list(range(blocks))
    random.Random(0).shuffle(order)
    o = OracleEngine(cfg, sd, torch.bfloat16, blocks, 16, order, device=dev)
    g = torch.Generator().manual_seed(1)
    for s in range(BATCH):
        prompt = torch.randint(0, cfg["vocab_size"], (PROMPT,), generator=g).tolist()
        assert o.blocks.allocate(s, PROMPT + 1) is not None
        o.tokens[s] = prompt + [int(torch.randint(0, cfg["vocab_size"], (1,), generator=g))]
        o.prompt_len[s] = PROMPT
    seqs = list(range(BATCH))
    T, top_k, top_p = SAMPLING
    gen = torch.Generator(device=dev).manual_seed(1234)

    def step():
        logits = o.decode(seqs)
        probs = osamp.gpu_semantics_probs(logits, T, top_k, top_p)
        toks = torch.multinomial(probs, 1, generator=gen).view(-1).tolist()
        for s, t in zip(seqs, toks):
            o.append(s, t)
        return logits

    logits = step()   # warm-up
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    for _ in range(K):
        logits = step()
    e1.record()
    torch.cuda.synchronize(dev)
    step_ms = e0.elapsed_time(e1) / K
    wall_ms = (time.perf_counter() - t0) * 1e3 / K

    # sampling alone, on the last step's logits (bf16, as the model emits them)
    lb = logits.to(torch.bfloat16)

    def timed(fn, iters=20):
        fn()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            fn()
        b.record()
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / iters * 1e3

    ref_us = timed(lambda: torch.multinomial(osamp.gpu_semantics_probs(lb.float(), T, top_k, top_p), 1,
                                             generator=gen))
    out = torch.empty(BATCH, dtype=torch.int64, device=dev)
    ours_us = timed(lambda: ops.sample(lb, T, top_k, top_p, 1234, 0, out=out))
    v = BATCH / (step_ms * 1e-3)
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 2), "unit": "tokens/s", "n_gpus": 1,
            "steps": K, "warmup": 1, "ms_per_step": round(step_ms, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{ARCH} decode, batch {BATCH}, prompt {PROMPT}, T/top-k/top-p "
                                   f"{SAMPLING[0]}/{SAMPLING[1]}/{SAMPLING[2]}",
                       "model": ARCH, "layers": cfg["num_hidden_layers"], "global_batch": BATCH, "seq_len": PROMPT,
                       "parallelism": "tp1", "path": "reference PyTorch path (oracle restatement) on cuda:0"},
            "secondary_baseline": {"decode_step_ms": round(step_ms, 3), "decode_step_wall_ms": round(wall_ms, 3),
                                   "sampling_reference_us": round(ref_us, 2), "sampling_mvb_sample_us": round(ours_us, 2),
                                   "sampling_rows": BATCH, "vocab": int(lb.shape[-1])},
            "e2e": {"value": round(BATCH / (wall_ms * 1e-3), 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": BATCH * 8}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------- GPU path
def run_gpu(args, rank: int, world: int, local: int) -> None:
    from llm_pytorch_inference_b200 import _native as N
    from llm_pytorch_inference_b200.configs import get_config
    from llm_pytorch_inference_b200.engine import DecodeEngine
    from llm_pytorch_inference_b200.tensor_parallel import TensorParallelConfig
    from llm_pytorch_inference_b200.weights import canonical_state_dict

    dev = torch.device("cuda", local)
    N.set_pdl(bool(args.pdl))
    overrides = {} if args.layers is None else {"num_hidden_layers": args.layers}
    cfg = get_config(ARCH, **overrides)
    # N GPUs = one tensor-parallel group over the same batch-64 workload (strong scaling): every
    # rank builds the same model and sequences and keeps its shard.
    tp = TensorParallelConfig(world, rank)
    sd = canonical_state_dict(cfg, seed=0, dtype=torch.bfloat16, device=dev)
    W, K = args.warmup, args.steps
    max_len = PROMPT + 1 + W + 2 * K + 16
    free_order_seed = 0
    eng = DecodeEngine(cfg, sd, max_batch=BATCH, max_model_len=max_len, device=dev, tp=tp,
                       fused_layers=bool(args.fused_layers))
    del sd
    order = list(range(eng.kv.num_blocks))
    random.Random(free_order_seed).shuffle(order)
    from collections import deque

    eng.kv.free_blocks = deque(order)
    g = torch.Generator().manual_seed(1)
    for s in range(BATCH):
        eng.add_sequence(s, torch.randint(0, cfg["vocab_size"], (PROMPT,), generator=g).tolist())
        eng.append_first_token(s, int(torch.randint(0, cfg["vocab_size"], (1,), generator=g)))
    eng.prefill_synthetic(seed=rank)   # each rank fills its own KV heads
    eng.set_sampling(*SAMPLING, seed=1234)
    eng.prepare_first_step()
    r = eng.runner
    stream = torch.cuda.current_stream(dev)

    # warm-up through the public API (captures the graph on the first call)
    for _ in range(W):
        eng.step()
    torch.cuda.synchronize(dev)

    # ---- value: K replays with each step's metadata already in HBM
    metas = torch.stack([eng.plan_step(eng.runner.tokens_host[:BATCH].tolist()) for _ in range(K)]).to(dev)
    clocks = ClockSampler(local)
    clocks.start()
    barrier(world)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for k in range(K):
        r.meta.copy_(metas[k], non_blocking=True)
        r.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    dev_ms = max_over_ranks(e0.elapsed_time(e1), world)
    barrier(world)

    # ---- e2e: K steps through DecodeEngine.run_steps() (per step: H2D metadata, replay, D2H tokens)
    torch.cuda.synchronize(dev)
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    eng.run_steps(K)
    e3.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(e2.elapsed_time(e3), world)
    clk = clocks.stop()
    status = N.device_status(clear=True)

    # ---- per-kernel timing for the roofline
    kinds = r.time_kernels(iters=36 if cfg["num_hidden_layers"] >= 36 else cfg["num_hidden_layers"] * 4)
    step_ms = dev_ms / K
    for v in kinds.values():
        v["share"] = v["avg_ms"] * v["launches_per_step"] / step_ms
    top_name, top = max(kinds.items(), key=lambda kv: kv[1]["share"])
    pk = peaks()
    tr = ncu_traffic().get(top_name)
    traffic = None if tr is None else round(tr[0] * top["bytes_per_launch"] / tr[1])
    achieved = top["bytes_per_launch"] / (top["avg_ms"] * 1e-3) / 1e9
    roof = {"kernel": top_name, "bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": round(achieved / pk["hbm_gbs"], 4), "peak_source": pk["source"],
            "traffic": traffic, "algorithmic_bytes_per_launch": top["bytes_per_launch"],
            "avg_launch_ms": round(top["avg_ms"], 5), "share_of_step": round(top["share"], 3)}
    # whole-step roofline: weights + KV read + KV write of one step / step time
    step_bytes = r.algorithmic_step_bytes()
    step_roof = {"bytes_per_step": step_bytes, "achieved_gbs": round(step_bytes / (step_ms * 1e-3) / 1e9, 1),
                 "frac": round(step_bytes / (step_ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4)}

    barrier(world)
    r.close()   # graph, then the symmetric heap (every rank, before the process group goes)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline()
    if rank != 0:
        return
    h2d = r.meta_host.numel() * r.meta_host.element_size()
    value = BATCH * K / (dev_ms * 1e-3)
    e2e = BATCH * K / (e2e_ms * 1e-3)
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(step_ms, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{ARCH} decode, batch {BATCH}, prompt {PROMPT}, T/top-k/top-p "
                               f"{SAMPLING[0]}/{SAMPLING[1]}/{SAMPLING[2]}",
                   "model": ARCH, "layers": cfg["num_hidden_layers"], "global_batch": BATCH,
                   "seq_len": PROMPT, "context_during_timing": [PROMPT + 1 + W, PROMPT + 1 + W + 2 * K],
                   "parallelism": f"tp{world}",
                   "l2": "inputs larger than L2: 15.1 GB weights + ~20 GB KV read per step",
                   "kv_pool_blocks": eng.kv.num_blocks, "pdl": bool(args.pdl),
                   "layer_tail": "one persistent launch" if r.fused else "per-kernel"},
        "roofline": roof, "step_roofline": step_roof,
        "kernels": {k: {"avg_us": round(v["avg_ms"] * 1e3, 2), "per_step": v["launches_per_step"],
                        "share": round(v["share"], 3), "gbs": round(v["gbs"], 1)} for k, v in kinds.items()},
        "cpu_baseline": None if cpu is None else {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": round(e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": BATCH * 8},
        "gpu_launches": r.launches_per_step() * K,
        "clocks": clk, "device_status": status,
    }
    print(json.dumps(line), flush=True)


def run_kernel_case(args) -> None:
    """Profiling case: Qwen3-8B layer dims with 2 layers, batch 64, context 2048 (537 MB of KV per
    layer, above the 126 MB L2), ~4.5 GB on the device; or (``--arch gemma2-9b``) Gemma-2-9B layer
    dims with 2 layers (one sliding-window, one global), batch 16, context 8192 (1.07 GB of KV per
    layer), ~4.5 GB.  One full decode step runs first, then every kernel kind of the step is launched
    1 + 3 times (first launch = warm-up), in the order of DecodeRunner.kernel_kinds()."""
    from llm_pytorch_inference_b200 import _native as N
    from llm_pytorch_inference_b200.configs import get_config
    from llm_pytorch_inference_b200.engine import DecodeEngine
    from llm_pytorch_inference_b200.weights import canonical_state_dict

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    N.set_pdl(bool(args.pdl))
    arch = args.arch or ARCH
    batch, prompt = (BATCH, PROMPT) if arch == ARCH else (16, 8192)
    cfg = get_config(arch, num_hidden_layers=2)
    sd = canonical_state_dict(cfg, seed=0, dtype=torch.bfloat16, device=dev)
    nblk = batch * ((prompt + 2 + 15) // 16) + 64
    eng = DecodeEngine(cfg, sd, max_batch=batch, max_model_len=prompt + 64, num_blocks=nblk, device=dev)
    del sd
    g = torch.Generator().manual_seed(1)
    for s in range(batch):
        eng.add_sequence(s, torch.randint(0, cfg["vocab_size"], (prompt,), generator=g).tolist())
        eng.append_first_token(s, 1)
    eng.prefill_synthetic(seed=0)
    eng.set_sampling(*SAMPLING, seed=1234)
    eng.prepare_first_step()
    eng._grow_blocks()
    eng.runner.upload_metadata()
    eng.runner.forward()          # one real step first, so every buffer holds realistic values
    torch.cuda.synchronize(dev)
    res = eng.runner.time_kernels(iters=3)
    print(json.dumps({k: {"avg_us": round(v["avg_ms"] * 1e3, 2), "gbs": round(v["gbs"], 1),
                          "bytes_per_launch": v["bytes_per_launch"]} for k, v in res.items()}), flush=True)
    assert N.device_status(clear=True) == 0


def run_moe_case(args) -> None:
    """Sparse-MoE decode (Qwen3-30B-A3B architecture: 48 layers, hidden 2048, 32/4 heads, 128
    experts of 768, top-8), batch 32, 4096-token prompts with seeded synthetic K/V, greedy.  Same
    timing rules as the headline line (CUDA events over K graph replays, inputs far above L2).
    Under torchrun with N GPUs: attention split by heads and the experts split whole over the
    ranks (expert parallel), one group over the same batch (strong scaling), max over ranks."""
    from llm_pytorch_inference_b200 import _native as N
    from llm_pytorch_inference_b200.configs import get_config
    from llm_pytorch_inference_b200.engine import DecodeEngine
    from llm_pytorch_inference_b200.tensor_parallel import TensorParallelConfig
    from llm_pytorch_inference_b200.weights import canonical_state_dict

    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    N.set_pdl(bool(args.pdl))
    cfg = get_config("qwen3-30b-a3b")
    B, prompt = 32, 4096
    W, K = args.warmup, args.steps
    sd = canonical_state_dict(cfg, seed=0, dtype=torch.bfloat16, device=dev, stacked_experts=True)
    eng = DecodeEngine(cfg, sd, max_batch=B, max_model_len=prompt + 2 * (W + 2 * K) + 32, device=dev,
                       tp=TensorParallelConfig(world, rank))
    del sd
    order = list(range(eng.kv.num_blocks))
    random.Random(0).shuffle(order)
    from collections import deque

    eng.kv.free_blocks = deque(order)
    g = torch.Generator().manual_seed(1)
    for s in range(B):
        eng.add_sequence(s, torch.randint(0, cfg["vocab_size"], (prompt,), generator=g).tolist())
        eng.append_first_token(s, int(torch.randint(0, cfg["vocab_size"], (1,), generator=g)))
    eng.prefill_synthetic(seed=rank)   # each rank fills its own KV heads
    eng.set_sampling(0.0, -1, 1.0)
    eng.prepare_first_step()
    r = eng.runner
    stream = torch.cuda.current_stream(dev)
    for _ in range(W):
        eng.step()
    torch.cuda.synchronize(dev)
    metas = torch.stack([eng.plan_step(eng.runner.tokens_host[:B].tolist()) for _ in range(K)]).to(dev)
    clocks = ClockSampler(local)
    clocks.start()
    barrier(world)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for k in range(K):
        r.meta.copy_(metas[k], non_blocking=True)
        r.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = max_over_ranks(e0.elapsed_time(e1) / K, world)
    barrier(world)
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    eng.run_steps(K)
    e3.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(e2.elapsed_time(e3) / K, world)
    clk = clocks.stop()
    # algorithmic bytes per GPU: attention/norm/lm_head weights, the rank's experts the step's
    # routing touched in each layer (counted on the device after the last step), K/V of every
    # attended token of the rank's KV heads
    ids = r.active[1:1 + int(r.active[0])].tolist()
    act = sum(1 for e in ids if r.e_first <= e < r.e_first + r.e_local)
    L, H, E, Im = cfg["num_hidden_layers"], cfg["hidden_size"], cfg["num_experts"], cfg["moe_intermediate_size"]
    w = r.w
    dense = sum(t.numel() * 2 for t in [w.final_norm, w.lm_head, *w.wqkv, *w.wo, *w.ln1, *w.ln2, *w.qn, *w.kn,
                                          *w.router])
    expert_bytes = 3 * Im * H * 2
    kv_token = L * r.Hkv * r.D * 2 * 2
    step_bytes = dense + L * act * expert_bytes + int(r.ctx.cpu().sum()) * kv_token
    pk = peaks()
    status = N.device_status(clear=True)
    statuses = [status]
    if world > 1:
        import torch.distributed as dist

        statuses = [None] * world
        dist.all_gather_object(statuses, status)
        r.close()
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {"case": "moe", "metric": "decode tokens/s Qwen3-30B-A3B-arch bf16 batch 32 ctx 4096 greedy",
            "value": round(B / (ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": world, "ms_per_step": round(ms, 4),
            "steps": K, "warmup": W, "e2e": {"value": round(B / (e2e_ms * 1e-3), 1), "unit": "tokens/s"},
            "parallelism": f"tp{world} (attention heads) / ep{world} (experts)" if world > 1 else "1 GPU",
            "active_experts_last_layer_this_gpu": act, "step_bytes_per_gpu": step_bytes,
            "step_roofline": {"achieved_gbs": round(step_bytes / (ms * 1e-3) / 1e9, 1),
                              "frac": round(step_bytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4)},
            "launches_per_step": r.launches_per_step(), "clocks": clk, "device_status": statuses}
    print(json.dumps(line), flush=True)


def run_llama3_case(args) -> None:
    """Llama-3-8B-architecture decode (32 layers, hidden 4096, 32/8 heads, SwiGLU 14336, vocab 128256,
    theta 5e5, no QK-norm), a mixed batch of 128 sequences whose contexts are drawn uniformly from
    128-8192 (seeded), K/V filled with seeded synthetic values in a shuffled pool, greedy.  Same
    timing rules as the headline line; the e2e figure goes through ``DecodeEngine.run_steps()``."""
    from llm_pytorch_inference_b200 import _native as N
    from llm_pytorch_inference_b200.configs import get_config
    from llm_pytorch_inference_b200.engine import DecodeEngine
    from llm_pytorch_inference_b200.weights import canonical_state_dict

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    N.set_pdl(bool(args.pdl))
    cfg = get_config("llama3-8b")
    B = 128
    W, K = args.warmup, args.steps
    g = torch.Generator().manual_seed(42)
    lens = torch.randint(128, 8193, (B,), generator=g).tolist()
    sd = canonical_state_dict(cfg, seed=0, dtype=torch.bfloat16, device=dev)
    eng = DecodeEngine(cfg, sd, max_batch=B, max_model_len=max(lens) + 2 * (W + 2 * K) + 32, device=dev)
    del sd
    order = list(range(eng.kv.num_blocks))
    random.Random(0).shuffle(order)
    from collections import deque

    eng.kv.free_blocks = deque(order)
    for s, n in enumerate(lens):
        eng.add_sequence(s, torch.randint(0, cfg["vocab_size"], (n,), generator=g).tolist())
        eng.append_first_token(s, int(torch.randint(0, cfg["vocab_size"], (1,), generator=g)))
    eng.prefill_synthetic(seed=0)
    eng.set_sampling(0.0, -1, 1.0)
    eng.prepare_first_step()
    r = eng.runner
    stream = torch.cuda.current_stream(dev)
    for _ in range(W):
        eng.step()
    torch.cuda.synchronize(dev)
    metas = torch.stack([eng.plan_step(eng.runner.tokens_host[:B].tolist()) for _ in range(K)]).to(dev)
    clocks = ClockSampler(0)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for k in range(K):
        r.meta.copy_(metas[k], non_blocking=True)
        r.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / K
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    eng.run_steps(K)
    e3.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e2.elapsed_time(e3) / K
    clk = clocks.stop()
    step_bytes = r.algorithmic_step_bytes()
    kinds = r.time_kernels(iters=32)
    top = max(kinds, key=lambda k: kinds[k]["avg_ms"] * kinds[k]["launches_per_step"])
    pk = peaks()
    line = {"case": "llama3", "metric": "decode tokens/s Llama-3-8B-arch bf16 batch 128 ctx U[128,8192] greedy",
            "value": round(B / (ms * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 4), "steps": K,
            "warmup": W, "config": {"workload": "llama3-8b decode, batch 128, contexts U[128,8192] (seeded), greedy",
                                     "layers": cfg["num_hidden_layers"], "mean_context": round(sum(lens) / B, 1),
                                     "parallelism": "tp1"},
            "e2e": {"value": round(B / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": r.meta_host.numel() * 4, "d2h_bytes_per_step": B * 8},
            "step_bytes": step_bytes,
            "step_roofline": {"achieved_gbs": round(step_bytes / (ms * 1e-3) / 1e9, 1),
                              "frac": round(step_bytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4)},
            "roofline": {"kernel": top, "bound": "hbm", "achieved": round(kinds[top]["gbs"], 1), "peak": pk["hbm_gbs"],
                         "unit": "GB/s", "frac": round(kinds[top]["gbs"] / pk["hbm_gbs"], 3),
                         "peak_source": pk["source"]},
            "kernels": {k: {"avg_us": round(v["avg_ms"] * 1e3, 2), "per_step": v["launches_per_step"],
                            "gbs": round(v["gbs"], 1)} for k, v in kinds.items()},
            "launches_per_step": r.launches_per_step(), "clocks": clk,
            "device_status": N.device_status(clear=True)}
    print(json.dumps(line), flush=True)


def run_gemma2_case(args) -> None:
    """Gemma-2-9B-architecture decode (42 layers, hidden 3584, 16/8 heads of 256, GeGLU 14336,
    vocab 256000, alternating 4096-token sliding-window / global layers, soft-capping 50 / 30,
    tied embeddings), batch 16, 8192-token prompts with seeded synthetic K/V, greedy.  Same
    timing rules as the headline line; per-kind kernel times as in the headline's `kernels`.  Under
    torchrun, the N ranks form one tensor-parallel group over the same workload (strong scaling),
    times are maxima over ranks and rank 0 prints."""
    rank, world, local = dist_setup(args.gpus)
    try:
        _gemma2_case(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


def _gemma2_case(args, rank: int, world: int, local: int) -> None:
    from llm_pytorch_inference_b200 import _native as N
    from llm_pytorch_inference_b200.configs import get_config
    from llm_pytorch_inference_b200.engine import DecodeEngine
    from llm_pytorch_inference_b200.tensor_parallel import TensorParallelConfig
    from llm_pytorch_inference_b200.weights import canonical_state_dict

    dev = torch.device("cuda", local)
    N.set_pdl(bool(args.pdl))
    cfg = get_config("gemma2-9b")
    B, prompt = 16, 8192
    W, K = args.warmup, args.steps
    sd = canonical_state_dict(cfg, seed=0, dtype=torch.bfloat16, device=dev)
    eng = DecodeEngine(cfg, sd, max_batch=B, max_model_len=prompt + 2 * (W + 2 * K) + 32, device=dev,
                       tp=TensorParallelConfig(world, rank))
    del sd
    order = list(range(eng.kv.num_blocks))
    random.Random(0).shuffle(order)
    from collections import deque

    eng.kv.free_blocks = deque(order)
    g = torch.Generator().manual_seed(1)
    for s in range(B):
        eng.add_sequence(s, torch.randint(0, cfg["vocab_size"], (prompt,), generator=g).tolist())
        eng.append_first_token(s, int(torch.randint(0, cfg["vocab_size"], (1,), generator=g)))
    eng.prefill_synthetic(seed=rank)   # each rank fills its own KV heads
    eng.set_sampling(0.0, -1, 1.0)
    eng.prepare_first_step()
    r = eng.runner
    stream = torch.cuda.current_stream(dev)
    for _ in range(W):
        eng.step()
    torch.cuda.synchronize(dev)
    metas = torch.stack([eng.plan_step(eng.runner.tokens_host[:B].tolist()) for _ in range(K)]).to(dev)
    clocks = ClockSampler(local)
    clocks.start()
    barrier(world)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for k in range(K):
        r.meta.copy_(metas[k], non_blocking=True)
        r.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = max_over_ranks(e0.elapsed_time(e1), world) / K
    step_bytes = r.algorithmic_step_bytes()
    barrier(world)
    torch.cuda.synchronize(dev)
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    eng.run_steps(K)
    e3.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(e2.elapsed_time(e3), world) / K
    clk = clocks.stop()
    kinds = r.time_kernels(iters=max(8, r.L))
    status = N.device_status(clear=True)
    barrier(world)
    r.close()
    if rank != 0:
        return
    pk = peaks()
    line = {"case": "gemma2", "metric": "decode tokens/s Gemma-2-9B-arch bf16 batch 16 ctx 8192 greedy",
            "n_gpus": world, "parallelism": f"tp{world}",
            "value": round(B / (ms * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 4), "steps": K,
            "warmup": W, "e2e": {"value": round(B / (e2e_ms * 1e-3), 1), "unit": "tokens/s"},
            "step_bytes": step_bytes,
            "step_roofline": {"achieved_gbs": round(step_bytes / (ms * 1e-3) / 1e9, 1),
                              "frac": round(step_bytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4)},
            "kernels": {k: {"avg_us": round(v["avg_ms"] * 1e3, 2), "launches_per_step": v["launches_per_step"],
                            "gbs": round(v["gbs"], 1), "frac": round(v["gbs"] / pk["hbm_gbs"], 4),
                            "share_of_step": round(v["avg_ms"] * v["launches_per_step"] / ms, 4)}
                        for k, v in kinds.items()},
            "launches_per_step": r.launches_per_step(), "clocks": clk, "device_status": status}
    print(json.dumps(line), flush=True)


def run_prefill_case(args) -> None:
    """Batched prefill (``DecodeEngine.prefill``) of the headline workload's prompts: Qwen3-8B
    architecture, 64 sequences of 2048 uniform-random tokens, into a shuffled paged pool.  One
    warm-up prefill of 2 sequences, then the 64-sequence prefill timed with CUDA events (chunks of
    16384 tokens).  GEMM FLOPs are 2 x tokens x the layers' parameters (plus the last tokens' lm_head);
    attention reads each token's prefix once (the decode kernel, one query per token)."""
    from llm_pytorch_inference_b200 import _native as N
    from llm_pytorch_inference_b200.configs import get_config
    from llm_pytorch_inference_b200.engine import DecodeEngine
    from llm_pytorch_inference_b200.weights import canonical_state_dict

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    N.set_pdl(bool(args.pdl))
    cfg = get_config(ARCH)
    B, prompt = BATCH, PROMPT
    sd = canonical_state_dict(cfg, seed=0, dtype=torch.bfloat16, device=dev)
    eng = DecodeEngine(cfg, sd, max_batch=B + 2, max_model_len=prompt + 64, device=dev)
    del sd
    order = list(range(eng.kv.num_blocks))
    random.Random(0).shuffle(order)
    from collections import deque

    eng.kv.free_blocks = deque(order)
    g = torch.Generator().manual_seed(0)
    prompts = {s: torch.randint(0, cfg["vocab_size"], (prompt,), generator=g).tolist() for s in range(B)}
    eng.prefill({B: prompts[0][:300], B + 1: prompts[1][:700]})          # warm-up (modules, buffers)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    clocks = ClockSampler(0)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    eng.prefill(prompts)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    r = eng.runner
    # per-kind device time: the same prefill again (new sequence ids) with events around each launch
    for s in range(B):
        eng.finish(s)
    eng._prefill.timing = {}
    eng.prefill({B + 2 + s: p for s, p in prompts.items()})
    torch.cuda.synchronize(dev)
    kind_ms = {k: round(sum(a.elapsed_time(b) for a, b in v), 1) for k, v in eng._prefill.timing.items()}
    eng._prefill.timing = None
    T = B * prompt
    layer_params = sum(t.numel() for t in [*r.w.wqkv, *r.w.wo, *r.w.wgu, *r.w.wdown])
    gemm_flops = 2 * T * layer_params + 2 * B * r.w.lm_head.numel()
    # tiled causal attention: each (sequence, 16-token tile, KV head) reads K and V of blocks 0..tile
    tiles_blocks = B * sum(qt + 1 for qt in range(prompt // 16))
    attn_bytes = r.L * tiles_blocks * 16 * r.Hkv * r.D * 2 * 2
    attn_flops = r.L * B * sum(i + 1 for i in range(prompt)) * r.Hq * r.D * 4
    pk = peaks()
    line = {"case": "prefill", "metric": "prefill prompt tokens/s Qwen3-8B-arch bf16, 64 x 2048-token prompts",
            "value": round(T / (ms * 1e-3), 1), "unit": "tokens/s", "ms": round(ms, 1), "tokens": T,
            "gemm_tflop": round(gemm_flops / 1e12, 1), "attention_tflop": round(attn_flops / 1e12, 1),
            "attention_bytes_gb": round(attn_bytes / 1e9, 1),
            "gemm_time_at_peak_ms": round(gemm_flops / (pk["bf16_tflops_sustained"] * 1e12) * 1e3, 1),
            "attention_time_at_hbm_peak_ms": round(attn_bytes / (pk["hbm_gbs"] * 1e9) * 1e3, 1),
            "kind_ms": kind_ms,
            "gemm_tflops_achieved": round(gemm_flops / (kind_ms.get("gemm", ms) * 1e-3) / 1e12, 1),
            "peaks": {"bf16_tflops_sustained": pk["bf16_tflops_sustained"], "hbm_gbs": pk["hbm_gbs"]},
            "clocks": clk, "device_status": N.device_status(clear=True)}
    print(json.dumps(line), flush=True)


def run_prefill_kernel_case(args) -> None:
    """Profiling case of the prefill: 2 layers at Qwen3-8B dims, a pool sized to its prompts.  One
    warm-up prefill of a 300-token prompt (2 attention and 9 GEMM launches), then one prefill of 8
    prompts of 2048 tokens (16384 rows: one chunk); prints the per-kind device times of the second."""
    from llm_pytorch_inference_b200 import _native as N
    from llm_pytorch_inference_b200.configs import get_config
    from llm_pytorch_inference_b200.engine import DecodeEngine
    from llm_pytorch_inference_b200.weights import canonical_state_dict

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    N.set_pdl(bool(args.pdl))
    cfg = get_config(ARCH, num_hidden_layers=2)
    B, prompt = 8, PROMPT
    sd = canonical_state_dict(cfg, seed=0, dtype=torch.bfloat16, device=dev)
    nblk = (B + 1) * ((prompt + 16) // 16) + 16
    eng = DecodeEngine(cfg, sd, max_batch=B + 1, max_model_len=prompt + 64, num_blocks=nblk, device=dev)
    del sd
    g = torch.Generator().manual_seed(0)
    eng.prefill({B: torch.randint(0, cfg["vocab_size"], (300,), generator=g).tolist()})   # warm-up
    torch.cuda.synchronize(dev)
    eng._prefill.timing = {}
    eng.prefill({s: torch.randint(0, cfg["vocab_size"], (prompt,), generator=g).tolist() for s in range(B)})
    torch.cuda.synchronize(dev)
    kind_ms = {k: round(sum(a.elapsed_time(b) for a, b in v), 3) for k, v in eng._prefill.timing.items()}
    print(json.dumps({"case": "prefill-kernels", "tokens": B * prompt, "kind_ms": kind_ms,
                      "device_status": N.device_status(clear=True)}), flush=True)


def main(argv=None) -> int:
    args = parse_args(argv)
    if args.case == "kernels":
        run_kernel_case(args)
        return 0
    if args.case == "gemma2":
        run_gemma2_case(args)
        return 0
    if args.case == "prefill":
        run_prefill_case(args)
        return 0
    if args.case == "prefill-kernels":
        run_prefill_kernel_case(args)
        return 0
    if args.case == "llama3":
        run_llama3_case(args)
        return 0
    if args.case == "moe":
        run_moe_case(args)
        return 0
    if args.case == "reference-gpu":
        if args.impl != "reference":
            raise SystemExit("--case reference-gpu times the reference's path: pass --impl reference")
        run_reference_gpu(args)
        return 0
    rank, world, local = (0, 1, 0)
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, rank, world)
        return 0
    rank, world, local = dist_setup(args.gpus)
    try:
        run_gpu(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
