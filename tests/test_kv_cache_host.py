"""The product's KV-cache manager on the CPU (no pool tensor): block ids bit-exact against the
allocator trace the reference itself produced (``mini_vllm/engine/kv_cache.py:6-81``, fixture
``tests/golden/kv_golden.json``), the scratch block, slots, and the HBM-budget pool sizing."""
import json
from pathlib import Path

import pytest

from llm_pytorch_inference_b200.kv_cache import GB, KVCacheManager, block_bytes, num_blocks_for_budget

GOLDEN = Path(__file__).parent / "golden"


def test_reference_allocator_trace_replays_bit_exactly():
    tr = json.loads((GOLDEN / "kv_golden.json").read_text())["shuffled_pool"]
    kv = KVCacheManager(64, 16, 2, 2, 128, device="cpu", free_order=tr["order"], allocate_pool=False)
    for ev in tr["log"]:
        if ev[0] == "allocate":
            got = kv.allocate(ev[1], ev[2])
            assert got == ev[3], ev
        elif ev[0] == "append":
            assert kv.append_token(ev[1]) == ev[2], ev
            assert kv.get_block_table(ev[1]) == ev[3], ev
        elif ev[0] == "free":
            kv.free(ev[1])
            assert list(kv.free_blocks) == ev[2], ev
    assert list(kv.free_blocks) == tr["free_end"]


def test_scratch_block_is_never_allocated_and_slots_index_the_table():
    kv = KVCacheManager(8, 16, 1, 1, 128, device="cpu", allocate_pool=False)
    assert kv.scratch_block == 8
    assert kv.allocate(0, 8 * 16) == list(range(8))          # the whole pool, in FIFO order
    assert kv.allocate(1, 1) is None                         # exhausted: the scratch block stays out
    assert kv.append_token(0) is False                       # growing past the pool fails
    assert kv.slot(0, 0) == (0, 0) and kv.slot(0, 17) == (1, 1) and kv.slot(0, 127) == (7, 15)
    kv.free(0)
    assert kv.num_free_blocks == 8 and kv.get_block_table(0) == []


def test_growth_takes_a_block_exactly_at_the_boundary():
    kv = KVCacheManager(4, 16, 1, 1, 128, device="cpu", allocate_pool=False, free_order=[3, 1, 0, 2])
    assert kv.allocate(5, 16) == [3]                         # 16 tokens: one full block
    assert kv.append_token(5) and kv.get_block_table(5) == [3, 1]   # token 17 opens block 1
    for _ in range(15):
        assert kv.append_token(5)
    assert kv.get_block_table(5) == [3, 1]                   # 32 tokens still fit two blocks
    assert kv.append_token(5) and kv.get_block_table(5) == [3, 1, 0]


def test_free_order_must_be_a_permutation():
    with pytest.raises(ValueError):
        KVCacheManager(4, 16, 1, 1, 128, device="cpu", allocate_pool=False, free_order=[0, 1, 1, 2])


def test_pool_sizing_from_the_hbm_budget():
    # Qwen3-8B arch: 36 layers, 8 KV heads of 128, bf16, 16-token blocks
    bb = block_bytes(16, 8, 128, 36, 2)
    assert bb == 2 * 16 * 8 * 128 * 36 * 2 == 2_359_296
    w, ws = 16 * GB, 1 * GB
    n = num_blocks_for_budget(16, 8, 128, 36, 2, w, ws)
    assert n == (180 * GB - w - ws - 2 * GB) // bb
    # never more than the device reports free (minus the same workspace and reserve)
    assert num_blocks_for_budget(16, 8, 128, 36, 2, w, ws, device_free_bytes=50 * GB) == (50 * GB - ws - 2 * GB) // bb
    # a budget smaller than the weights still yields one block
    assert num_blocks_for_budget(16, 8, 128, 36, 2, 200 * GB) == 1
