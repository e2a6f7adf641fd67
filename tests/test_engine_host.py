"""The decode engine's host bookkeeping (``RunningBatch``) against the reference's own engine.

``tests/golden/engine_trace.json`` was recorded by running the reference's ``LLMEngine._step``
(``engine/engine.py:241-360``, ``engine/scheduler.py:27-57``, ``engine/sequence.py:66-80``) on a
shuffled 20-block pool: sequences with different ``max_tokens``, one that stops on a stop id,
two that join while others run, one whose prompt cannot be allocated.  Replaying the same
sequence of steps and tokens through ``RunningBatch.plan_schedule_step`` must give, bit for bit,
the decoded rows and their order, the block tables and slots the decode forward receives, the
free list after every step, the finished set and every sequence's output."""
import json
import random

import numpy as np
import pytest

from llm_pytorch_inference_b200.engine import RunningBatch, SeqSampling
from llm_pytorch_inference_b200.kv_cache import KVCacheManager
from llm_pytorch_inference_b200.runner import meta_layout

B, MB = 8, 64


def _batch(num_blocks, seed):
    order = list(range(num_blocks))
    random.Random(seed).shuffle(order)
    kv = KVCacheManager(num_blocks, 16, 2, 4, 128, device="cpu", free_order=order, allocate_pool=False)
    return kv, RunningBatch(kv, B, MB)


def _rows(snap):
    lay = meta_layout(B, MB)
    bt = snap[lay["bt"]:].reshape(B, MB)
    return (snap[lay["ids"]:lay["ids"] + B], snap[lay["pos"]:lay["pos"] + B], snap[lay["ctx"]:lay["ctx"] + B], bt,
            snap[lay["temp"]:lay["temp"] + B].view(np.float32))


def test_running_batch_replays_the_reference_engine(golden_dir):
    d = json.loads((golden_dir / "engine_trace.json").read_text())
    kv, rb = _batch(d["num_blocks"], d["pool_seed"])
    prompts, max_toks, stop = d["prompts"], d["max_tokens"], {int(k): v for k, v in d["stop"].items()}
    for step, t in enumerate(d["trace"]):
        first = {s: f for s, f in t["prefill"]}
        new = {s: (prompts[s], first[s], max_toks[s], stop.get(s, [])) for s in d["joins"].get(str(step), [])}
        snap = rb.plan_schedule_step(new, {int(k): v for k, v in t["decode_tokens"].items()})
        assert rb.last_step_seqs == t["decode"] if snap is not None else t["decode"] == [], step
        if snap is not None:
            ids, pos, ctx, bt, temp = _rows(snap)
            for row, s in enumerate(t["decode"]):
                tab = t["block_tables"][row]
                assert bt[row, :len(tab)].tolist() == tab, (step, s)
                assert (bt[row, len(tab):] == kv.scratch_block).all()
                assert pos[row] == t["slot_idx"][row] and ctx[row] == t["slot_idx"][row] + 1
            for row in range(len(t["decode"]), B):       # joined-this-step and unused rows are padding
                assert (bt[row] == kv.scratch_block).all() and ctx[row] == 1 and temp[row] == 0.0
        assert list(kv.free_blocks) == t["free_after"], step
        assert sorted(rb.finish_reason) == t["finished_after"], step
    for s, out in d["outputs"].items():
        assert rb.output_tokens(int(s)) == out
    assert rb.finish_reason == {0: "length", 1: "length", 2: "length", 3: "stop", 4: "length", 5: "length",
                                6: "abort"}
    assert not rb.has_unfinished and kv.num_free_blocks == d["num_blocks"]


def test_finish_compacts_rows_and_returns_blocks_to_the_tail():
    kv, rb = _batch(32, 0)
    tables = [list(rb.add_sequence(s, list(range(5 + 20 * s)), sampling=SeqSampling(0.5 * s, s, 0.9)))
              for s in range(4)]
    for s in range(4):
        rb.append_first_token(s, 100 + s)
    rb.start()
    free_before = list(kv.free_blocks)
    rb.finish(1)
    assert list(kv.free_blocks) == free_before + tables[1]
    assert rb.seqs == [0, 2, 3]
    snap = rb.plan_step([7, 8, 9])
    ids, pos, ctx, bt, temp = _rows(snap)
    assert ids[:3].tolist() == [100, 102, 103]
    assert [bt[r, :len(tables[s])].tolist() for r, s in enumerate([0, 2, 3])] == [tables[0], tables[2], tables[3]]
    assert temp[:4].tolist() == [0.0, 1.0, 1.5, 0.0]            # per-sequence sampling moved with its row
    assert (bt[3] == kv.scratch_block).all() and ctx[3] == 1
    assert [rb.output_tokens(s) for s in (0, 2, 3)] == [[100, 7], [102, 8], [103, 9]]
    with pytest.raises(KeyError):
        rb.finish(1)


def test_first_token_can_finish_a_sequence():
    kv, rb = _batch(16, 0)
    rb.add_sequence(0, [1, 2, 3], max_tokens=1)
    rb.add_sequence(1, [4, 5], stop_token_ids=[9])
    rb.add_sequence(2, [6], max_tokens=3)
    assert rb.append_first_token(0, 5) and rb.append_first_token(1, 9)
    assert not rb.append_first_token(2, 9)
    assert rb.seqs == [2] and rb.finish_reason == {0: "length", 1: "stop"}
    assert kv.num_free_blocks == 15


def test_pool_exhaustion_during_growth_drops_the_sequence():
    """``engine.py:299-309``: a sequence that cannot grow finishes and is not decoded."""
    kv, rb = _batch(3, 0)
    rb.add_sequence(0, list(range(15)))            # 16 tokens: 1 block
    rb.add_sequence(1, list(range(31)))            # 32 tokens: 2 blocks, pool now empty
    rb.append_first_token(0, 1)
    rb.append_first_token(1, 1)
    rb.start()
    # row order: sequence 0 needs a second block and finds none, is freed; sequence 1 then grows
    # into the block sequence 0 just returned
    table0 = list(kv.get_block_table(0))
    rb.plan_step([5, 6])
    assert rb.finish_reason == {0: "abort"} and rb.seqs == [1] and rb.last_step_seqs == [1]
    assert kv.get_block_table(1)[-1] == table0[0]


@pytest.mark.parametrize("num_blocks,seed", [(32, 0), (30, 3), (200, 1)])
def test_step_fast_path_equals_the_general_path(num_blocks, seed):
    """The common step's bookkeeping fast path (no held rows, every block growth fits; the row
    mirrors for growth and the finish rules) against the general per-row path on the same steps:
    identical metadata, free list, block tables, outputs and finish reasons in finish order,
    including steps where the pool runs dry and sequences are dropped."""
    runs = []
    for fast in (True, False):
        kv, rb = _batch(num_blocks, seed)
        if not fast:
            rb._grow_fast = lambda: False   # the general path, which also drops the row mirrors
        r2 = random.Random(seed)
        for s in range(B):
            rb.add_sequence(s, [r2.randrange(1000) for _ in range(r2.randrange(5, 60))],
                            max_tokens=None if s % 2 == 0 else r2.choice([20, 45]),
                            stop_token_ids=[7] if s % 3 == 1 else ())
        rb.start()
        snaps = []
        r3 = random.Random(seed + 100)
        for _ in range(150):
            if not rb.seqs:
                break
            toks = [r3.randrange(50) for _ in range(B)]
            snaps.append(rb.plan_step(toks).copy())
        runs.append((snaps, list(kv.free_blocks), dict(kv.block_tables), list(rb.finish_reason.items()),
                     {s: list(t) for s, t in rb.tokens.items()}))
    (sa, fa, ta, ra, oa), (sb, fb, tb, rb_, ob) = runs
    assert len(sa) == len(sb)
    for a, b in zip(sa, sb):
        assert np.array_equal(a, b)
    assert fa == fb and ta == tb and ra == rb_ and oa == ob   # finish order too
    ra = dict(ra)
    if num_blocks < 100:   # the tight pools run dry: some sequences are dropped while growing
        assert "abort" in ra.values(), ra
