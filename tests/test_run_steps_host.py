"""``DecodeEngine.run_steps`` on the host, against ``step()``, with a stand-in for the device.

The stand-in runner keeps what the GPU would see: at every launch it takes the uploaded
metadata, applies the id feed when the launch asks for it (the ids become the previous
launch's sampled tokens, as ``mvb_feed_ids`` does), and "samples" each row's token as a fixed
function of the ids, positions and sampling offset it was given.  A wrong id, position, block
table or offset in any launch therefore changes the tokens that follow.  ``run_steps`` must
give, launch by launch, the same effective metadata as the same number of ``step()`` calls, and
the same tokens, outputs, block tables, free list and finishes (in finish order): with no limits
(every step but the first launched ahead), with length limits (once rows have finished, the
padding rows keep id 0, which a fed launch would overwrite, so such a batch is not run ahead),
with stop ids (no step ahead), and on a pool so tight that sequences are dropped while growing."""
import random

import numpy as np
import pytest
import torch

from llm_pytorch_inference_b200.engine import DecodeEngine, RunningBatch
from llm_pytorch_inference_b200.kv_cache import KVCacheManager
from llm_pytorch_inference_b200.runner import meta_layout

B, MB = 8, 64


class _Device:
    """The launches of a decode step as the GPU would run them (see the module docstring)."""

    def __init__(self, eng: RunningBatch):
        self.eng = eng
        self.lay = meta_layout(B, MB)
        self.graph = object()                   # a captured step: run-ahead is allowed
        self.tokens = np.zeros(B, dtype=np.int64)   # the sampler's output buffer
        self.launches: list[np.ndarray] = []    # effective metadata of every launch
        self.bufs: list[np.ndarray] = []

    def _run(self, feed: bool) -> np.ndarray:
        m = self.eng.meta_np.copy()
        if feed:
            m[:B] = self.tokens.astype(np.int32)
        m[self.lay["feed"]] = 0
        self.launches.append(m)
        ids, pos = m[:B].astype(np.int64), m[self.lay["pos"]:self.lay["pos"] + B].astype(np.int64)
        off = int(m[self.lay["off"]:self.lay["off"] + 2].view(np.int64)[0])
        bt0 = m[self.lay["bt"]:].reshape(B, MB)[:, 0].astype(np.int64)
        self.tokens = (ids * 31 + pos * 7 + bt0 * 5 + off * 3 + np.arange(B)) % 50
        return self.tokens.copy()

    # the synchronous step() path
    def step(self, use_graph: bool = True) -> None:
        self.bufs = [self._run(False)]

    def fetch_tokens(self) -> torch.Tensor:
        return torch.from_numpy(self.bufs[-1])

    # the run-ahead path
    def launch_staged(self, feed: bool) -> int:
        self.bufs.append(self._run(feed))
        return len(self.bufs) - 1

    def tokens_of(self, i: int) -> torch.Tensor:
        return torch.from_numpy(self.bufs[i])


class _Engine(RunningBatch):
    """The engine's host side with the stand-in device; step() and run_steps() are the engine's own."""

    step = DecodeEngine.step
    run_steps = DecodeEngine.run_steps
    _decode = DecodeEngine._decode
    _can_run_ahead = DecodeEngine._can_run_ahead

    def __init__(self, num_blocks: int, seed: int):
        order = list(range(num_blocks))
        random.Random(seed).shuffle(order)
        kv = KVCacheManager(num_blocks, 16, 2, 4, 128, device="cpu", free_order=order, allocate_pool=False)
        super().__init__(kv, B, MB)
        self.runner = _Device(self)
        self.parity = False
        self.steps_run_ahead = 0


def _run(mode: str, num_blocks: int, seed: int, limits: bool, stop: bool, n: int):
    eng = _Engine(num_blocks, seed)
    r = random.Random(seed)
    for s in range(B):
        eng.add_sequence(s, [r.randrange(1000) for _ in range(r.randrange(5, 60))],
                         max_tokens=(None if s % 3 == 0 else r.choice([6, 20, 33])) if limits else None,
                         stop_token_ids=[7, 19] if stop and s % 2 == 1 else ())
        eng.append_first_token(s, r.randrange(50))
    eng.start()
    if mode == "step":
        steps = [eng.step() for _ in range(n)]
    else:
        steps = eng.run_steps(n)
    return dict(steps=steps, launches=eng.runner.launches, outputs={s: eng.output_tokens(s) for s in range(B)},
                tables=dict(eng.kv.block_tables), free=list(eng.kv.free_blocks),
                finished=list(eng.finish_reason.items()), ahead=eng.steps_run_ahead)


@pytest.mark.parametrize("num_blocks,seed,limits,stop", [
    (200, 0, False, False),   # nothing can finish: every step but the first runs ahead
    (200, 1, True, False),    # length limits: the steps where a row can finish are read back first
    (200, 2, False, True),    # stop ids on half the rows: no step runs ahead
    (200, 3, True, True),
    (26, 4, True, False),     # a tight pool: sequences are dropped while growing
])
def test_run_steps_equals_step_by_step(num_blocks, seed, limits, stop):
    n = 60
    a = _run("step", num_blocks, seed, limits, stop, n)
    b = _run("run_steps", num_blocks, seed, limits, stop, n)
    assert len(a["launches"]) == len(b["launches"])
    for i, (x, y) in enumerate(zip(a["launches"], b["launches"])):
        assert np.array_equal(x, y), i
    for k in ("steps", "outputs", "tables", "free", "finished"):
        assert a[k] == b[k], k
    assert a["ahead"] == 0
    if stop:
        assert b["ahead"] == 0
    elif not limits:
        assert b["ahead"] == n - 1
    else:
        assert 0 < b["ahead"] < n - 1 and b["finished"], b["ahead"]
    if num_blocks < 100:
        assert "abort" in dict(b["finished"]).values()
