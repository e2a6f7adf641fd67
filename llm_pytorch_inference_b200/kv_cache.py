"""Paged KV-cache manager with the reference's API and tensor layout.

Mirrors ``mini_vllm/engine/kv_cache.py:6-81``: the pool is one tensor
``[num_layers, 2 (K, V), num_blocks, block_size, num_heads, head_dim]``; blocks
come off a FIFO free list (``deque.popleft``) and go back to its tail; a
sequence allocated for ``n`` tokens holds ``ceil(n / block_size)`` blocks and
``append_token`` grows it by one block when the count crosses a block boundary.
Block ids and therefore slot indices are identical to the reference's for the
same call sequence and free-list order.

Additions for the B200 decode path:

* the pool carries ``num_blocks + 1`` blocks; the extra one (id ``num_blocks``)
  is never handed out and absorbs the KV writes of padded batch rows;
* ``num_blocks_for_budget`` sizes the pool from a per-GPU HBM budget (180 GB by
  default) minus resident weights and workspace, instead of the reference's
  ``0.9 * free memory`` rule (``mini_vllm/utils/config.py:29-57``).
"""
from __future__ import annotations

from collections import deque

import torch

GB = 1_000_000_000
DEFAULT_HBM_BUDGET = 180 * GB


def block_bytes(block_size: int, num_heads: int, head_dim: int, num_layers: int, dtype_size: int) -> int:
    """Bytes of one block across all layers, K and V (``config.py:44``)."""
    return 2 * block_size * num_heads * head_dim * num_layers * dtype_size


def num_blocks_for_budget(block_size: int, num_heads: int, head_dim: int, num_layers: int, dtype_size: int,
                          weights_bytes: int, workspace_bytes: int = 0, budget_bytes: int = DEFAULT_HBM_BUDGET,
                          device_free_bytes: int | None = None, reserve_bytes: int = 2 * GB) -> int:
    """Pool size: (budget - weights - workspace - reserve) / block bytes, never more than
    what is actually free on the device (minus the same reserve)."""
    avail = budget_bytes - weights_bytes - workspace_bytes - reserve_bytes
    if device_free_bytes is not None:
        avail = min(avail, device_free_bytes - workspace_bytes - reserve_bytes)
    return max(int(avail // block_bytes(block_size, num_heads, head_dim, num_layers, dtype_size)), 1)


class KVCacheManager:
    def __init__(self, num_blocks: int, block_size: int, num_layers: int, num_heads: int, head_dim: int,
                 device: str | torch.device = "cuda", dtype: torch.dtype = torch.bfloat16,
                 free_order: list[int] | None = None, allocate_pool: bool = True):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_layers = num_layers
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.device = device
        self.scratch_block = num_blocks  # absorbs writes of padded rows; never allocated
        self.kv_cache = (torch.zeros((num_layers, 2, num_blocks + 1, block_size, num_heads, head_dim), dtype=dtype,
                                     device=device) if allocate_pool else None)
        order = list(range(num_blocks)) if free_order is None else list(free_order)
        if sorted(order) != list(range(num_blocks)):
            raise ValueError("free_order must be a permutation of range(num_blocks)")
        self.free_blocks: deque[int] = deque(order)
        self.block_tables: dict[int, list[int]] = {}
        self.seq_num_tokens: dict[int, int] = {}

    def allocate(self, seq_id: int, num_tokens: int) -> list[int] | None:
        """``kv_cache.py:40-51``."""
        need = (num_tokens + self.block_size - 1) // self.block_size
        if len(self.free_blocks) < need:
            return None
        blocks = [self.free_blocks.popleft() for _ in range(need)]
        self.block_tables[seq_id] = blocks
        self.seq_num_tokens[seq_id] = num_tokens
        return blocks

    def free(self, seq_id: int) -> None:
        """``kv_cache.py:53-57``."""
        if seq_id in self.block_tables:
            self.free_blocks.extend(self.block_tables.pop(seq_id))
            self.seq_num_tokens.pop(seq_id, None)

    def append_token(self, seq_id: int) -> bool:
        """``kv_cache.py:59-74``: one more token; a new block when needed."""
        if seq_id not in self.block_tables:
            return False
        n = self.seq_num_tokens[seq_id] + 1
        need = (n + self.block_size - 1) // self.block_size
        if need > len(self.block_tables[seq_id]):
            if not self.free_blocks:
                return False
            self.block_tables[seq_id].append(self.free_blocks.popleft())
        self.seq_num_tokens[seq_id] = n
        return True

    def get_block_table(self, seq_id: int) -> list[int]:
        return self.block_tables.get(seq_id, [])

    @property
    def num_free_blocks(self) -> int:
        return len(self.free_blocks)

    def slot(self, seq_id: int, pos: int) -> tuple[int, int]:
        """(block id, offset) of token ``pos`` of a sequence (``model.py:233-237``)."""
        bt = self.block_tables[seq_id]
        return bt[pos // self.block_size], pos % self.block_size
