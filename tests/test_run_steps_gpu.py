"""``DecodeEngine.run_steps`` against the same number of ``step()`` calls on an identical engine:
the same tokens, outputs, block tables, free list and finishes in finish order.  Three regimes:
every step after the first launched ahead of the previous step's token read-back (no limits,
greedy); rows that reach their length limits mid-run, sampled at T 0.8 / top-k 50 / top-p 0.95
(a step where a row can finish is read back before the next launch; once rows have finished the
batch has padding rows and is no longer run ahead); and stop ids (a row could stop at any step,
so no step runs ahead)."""
import random

import pytest
import torch

from llm_pytorch_inference_b200 import _native as N
from llm_pytorch_inference_b200.configs import get_config
from llm_pytorch_inference_b200.engine import DecodeEngine
from llm_pytorch_inference_b200.weights import canonical_state_dict

pytestmark = pytest.mark.gpu

LENS = (37, 50, 16, 64, 20, 33, 15, 47)


@pytest.mark.parametrize("limits,stop,temp", [
    (None, (), 0.0),
    ((9, 30, None, 17, 25, None, 12, 40), (), 0.8),
    (None, (7, 11), 0.8),
])
def test_run_steps_matches_step(limits, stop, temp):
    cfg = get_config("qwen3-tiny")
    sd = {k: v.to(torch.bfloat16) for k, v in canonical_state_dict(cfg, 0, torch.float32).items()}
    P = 120
    order = list(range(P))
    random.Random(2).shuffle(order)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg["vocab_size"], (n,), generator=g).tolist() for n in LENS]
    firsts = torch.randint(0, cfg["vocab_size"], (len(LENS),), generator=g).tolist()
    runs, ahead = [], []
    for mode in ("step", "run_steps"):
        eng = DecodeEngine(cfg, sd, max_batch=len(LENS), max_model_len=256, num_blocks=P, device="cuda",
                           free_order=list(order))
        for s, p in enumerate(prompts):
            eng.add_sequence(s, p, max_tokens=None if limits is None else limits[s], stop_token_ids=stop)
            eng.append_first_token(s, firsts[s])
        eng.prefill_synthetic(seed=5)
        eng.set_sampling(temp, 50, 0.95, seed=9)
        eng.prepare_first_step()
        first = eng.step()   # captures the graph: a step runs ahead only on a captured graph
        if mode == "step":
            steps = [eng.step() for _ in range(45)]
        else:
            steps = eng.run_steps(45)
        runs.append(([first] + steps, {s: eng.output_tokens(s) for s in range(len(LENS))},
                     dict(eng.kv.block_tables), list(eng.kv.free_blocks), list(eng.finish_reason.items())))
        ahead.append(eng.steps_run_ahead)
        assert N.device_status(clear=True) == 0
    assert runs[0] == runs[1]
    assert ahead[0] == 0
    if stop:
        assert ahead[1] == 0
    elif limits is None:
        assert ahead[1] == 44            # every step but the first of the call
    else:
        assert 0 < ahead[1] < 44 and runs[1][4], ahead[1]   # some steps ran ahead, some rows finished
