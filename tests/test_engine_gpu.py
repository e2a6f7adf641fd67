"""Continuous batching on the GPU: sequences finish at different steps and new ones join while
others run, through ``DecodeEngine.schedule_step`` (the reference's ``LLMEngine._step``,
``engine.py:241-360``).  After every step the rows left are compacted, and the kernels must still
read each sequence's own blocks: each decoded row's logits are checked against the oracle's
decode of the same sequence from the same KV state, the block tables and the free list against
the oracle's FIFO manager (bit-exact, freed blocks reused), at every step."""
import random

import pytest
import torch
from torch.nn.attention import SDPBackend

from llm_pytorch_inference_b200 import _native as N
from llm_pytorch_inference_b200.configs import get_config
from llm_pytorch_inference_b200.engine import DecodeEngine
from llm_pytorch_inference_b200.weights import canonical_state_dict
from oracle import sampling as osamp
from oracle.engine import OracleEngine

pytestmark = pytest.mark.gpu


def test_sequences_finish_join_and_rows_compact():
    cfg = get_config("qwen3-tiny")
    sd = canonical_state_dict(cfg, 0, torch.float32)
    P = 40                                    # tight: freed blocks come back into use
    order = list(range(P))
    random.Random(4).shuffle(order)
    g = torch.Generator().manual_seed(8)
    lens = [37, 50, 16, 64, 20, 33]
    prompts = [torch.randint(0, cfg["vocab_size"], (n,), generator=g).tolist() for n in lens]
    max_toks = [3, 9, 5, 12, 6, 8]
    joins = {0: [0, 1, 2, 3], 4: [4, 5]}
    oracle = OracleEngine(cfg, sd, torch.bfloat16, P, 16, list(order))
    alt = OracleEngine(cfg, sd, torch.bfloat16, P, 16, list(order), sdpa_backend=SDPBackend.MATH)
    eng = DecodeEngine(cfg, {k: v.to(torch.bfloat16) for k, v in sd.items()}, max_batch=6, max_model_len=128,
                       num_blocks=P, device="cuda", free_order=list(order))
    eng.set_sampling(0.0, -1, 1.0)
    running: list[int] = []
    step = 0
    while step == 0 or running or step in joins:
        new = joins.get(step, [])
        before = list(running)
        # the reference's step: prefill the new sequences first, then decode the running ones
        firsts = {}
        for s in new:
            firsts[s] = int(osamp.greedy(oracle.prefill(s, prompts[s])[None])[0])
            alt.prefill(s, prompts[s])
            oracle.append(s, firsts[s])
            alt.append(s, firsts[s])
        ref = oracle.decode(before) if before else None
        ref_alt = alt.decode(before) if before else None
        got = eng.schedule_step({s: prompts[s] for s in new}, gen_max_tokens={s: max_toks[s] for s in new})
        assert eng.last_step_seqs == before, step
        assert set(got) == set(new) | set(before)
        if before:
            ours = eng.runner.logits[:len(before)].float().cpu()
            d, n = (ours - ref).abs(), (ref_alt - ref).abs()
            assert float(d.max()) <= max(2e-2, 1.5 * float(n.max())), (step, float(d.max()), float(n.max()))
            assert float(d.mean()) <= max(2e-3, 1.25 * float(n.mean())), (step, float(d.mean()))
        # teacher forcing on the oracle's greedy tokens; the oracle frees what finished, in row order
        ref_tok = dict(zip(before, osamp.greedy(ref).tolist())) if before else {}
        for s, t in ref_tok.items():
            oracle.append(s, t)
            alt.append(s, t)
        running = before + new
        for s in list(running):
            if len(oracle.tokens[s]) - oracle.prompt_len[s] >= max_toks[s]:
                oracle.blocks.free(s)
                alt.blocks.free(s)
                running.remove(s)
        assert eng.seqs == running, step
        assert sorted(eng.finished_last) == sorted(s for s in before + new if s not in running)
        eng.force_tokens({**firsts, **ref_tok})
        for s in running:
            assert eng.kv.get_block_table(s) == oracle.blocks.get_block_table(s), (step, s)
        assert list(eng.kv.free_blocks) == list(oracle.blocks.free_blocks), step
        eng.load_prefilled(oracle.kv_pool)     # the next step starts from the reference's KV state
        alt.kv_pool.copy_(oracle.kv_pool)
        step += 1
    assert all(eng.finish_reason[s] == "length" for s in range(6))
    assert eng.kv.num_free_blocks == P
    assert N.device_status(clear=True) == 0
