"""Oracle restatement of the reference's KV-block manager and engine step (CPU).

* ``BlockManager`` follows ``mini_vllm/engine/kv_cache.py:6-81``: ceil-div block
  counts, FIFO free list (``deque.popleft``), ``append_token`` grows by one block
  when ``(n + bs - 1) // bs`` exceeds the table, ``free`` returns the blocks to
  the tail of the list.
* ``OracleEngine`` follows ``LLMEngine._run_prefill`` (``engine.py:253-295``) and
  ``LLMEngine._run_decode`` (``engine.py:297-360``): per-sequence prefill with
  ``prompt_len + 1`` tokens allocated and causal attention, then one batched
  decode forward per step with ``positions = slot_idx = num_cached = len - 1``
  and a float mask of -inf past each sequence's length.
"""
from __future__ import annotations

from collections import deque

import torch

from .model import OracleDecoder
from . import sampling as osamp


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int, free_order: list[int] | None = None):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.free_blocks: deque[int] = deque(free_order if free_order is not None else range(num_blocks))
        self.block_tables: dict[int, list[int]] = {}
        self.seq_num_tokens: dict[int, int] = {}

    def allocate(self, seq_id: int, num_tokens: int) -> list[int] | None:      # kv_cache.py:40-51
        need = (num_tokens + self.block_size - 1) // self.block_size
        if len(self.free_blocks) < need:
            return None
        blocks = [self.free_blocks.popleft() for _ in range(need)]
        self.block_tables[seq_id] = blocks
        self.seq_num_tokens[seq_id] = num_tokens
        return blocks

    def free(self, seq_id: int) -> None:                                      # kv_cache.py:53-57
        if seq_id in self.block_tables:
            self.free_blocks.extend(self.block_tables.pop(seq_id))
            self.seq_num_tokens.pop(seq_id, None)

    def append_token(self, seq_id: int) -> bool:                             # kv_cache.py:59-74
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

    def get_block_table(self, seq_id: int) -> list[int]:                     # kv_cache.py:76-77
        return self.block_tables.get(seq_id, [])


def slot_of(block_table: list[int], pos: int, block_size: int) -> tuple[int, int]:
    """(block id, offset) a token at ``pos`` is written to (``model.py:233-237``)."""
    return block_table[pos // block_size], pos % block_size


class OracleEngine:
    """Greedy / sampled generation through the reference's step structure."""

    def __init__(self, cfg: dict, state_dict: dict, dtype: torch.dtype, num_blocks: int = 256,
                 block_size: int = 16, free_order: list[int] | None = None, device="cpu",
                 sdpa_backend=None, prefill_last_only: bool = False, capped_rounding: str = "fp32"):
        """``sdpa_backend`` (a ``torch.nn.attention.SDPBackend``) pins PyTorch's attention
        implementation -- the reference leaves the choice to PyTorch, so two backends are two
        equally valid executions of the reference (used to measure its own rounding noise).
        ``capped_rounding`` chooses how Gemma-2's soft-capped attention rounds (``OracleDecoder``):
        "fp32" (one rounding) or "eager" (transformers' eager attention in the model dtype)."""
        self.model = OracleDecoder(cfg, state_dict, dtype, device)
        self.model.capped_rounding = capped_rounding
        self.sdpa_backend = sdpa_backend
        self.prefill_last_only = prefill_last_only
        self.dtype = dtype
        self.device = torch.device(device)
        self.blocks = BlockManager(num_blocks, block_size, free_order)
        nkv = cfg.get("num_key_value_heads", cfg["num_attention_heads"])
        hd = cfg.get("head_dim", cfg["hidden_size"] // cfg["num_attention_heads"])
        self.kv_pool = torch.zeros(cfg["num_hidden_layers"], 2, num_blocks, block_size, nkv, hd,
                                   dtype=dtype, device=self.device)
        self.tokens: dict[int, list[int]] = {}
        self.prompt_len: dict[int, int] = {}

    def _autocast(self):
        import contextlib

        stack = contextlib.ExitStack()
        if self.sdpa_backend is not None:
            from torch.nn.attention import sdpa_kernel

            stack.enter_context(sdpa_kernel([self.sdpa_backend]))
        if self.dtype == torch.float32:
            stack.enter_context(torch.autocast(device_type=self.device.type, enabled=False))
        else:
            stack.enter_context(torch.autocast(device_type=self.device.type, dtype=self.dtype))
        return stack

    def prefill(self, seq_id: int, prompt: list[int]) -> torch.Tensor:
        """``engine.py:253-290``; returns the fp32 logits row of the last prompt token."""
        bt = self.blocks.allocate(seq_id, len(prompt) + 1)
        if bt is None:
            raise RuntimeError(f"KV pool exhausted for sequence {seq_id}")
        self.tokens[seq_id] = list(prompt)
        self.prompt_len[seq_id] = len(prompt)
        ids = torch.tensor([prompt], dtype=torch.long, device=self.device)
        pos = torch.arange(len(prompt), dtype=torch.long, device=self.device)
        with torch.no_grad(), self._autocast():
            logits = self.model.forward(ids, pos, self.kv_pool, bt, 0, use_cache=False,
                                        last_only=self.prefill_last_only)
        return logits[:, -1, :].float()[0]

    def decode_inputs(self, seq_ids: list[int]):
        """Per-step metadata as ``engine.py:299-337`` builds it (after ``append_token``)."""
        for s in seq_ids:
            if not self.blocks.append_token(s):
                raise RuntimeError(f"KV pool exhausted while growing sequence {s}")
        ids = [[self.tokens[s][-1]] for s in seq_ids]
        pos = [[len(self.tokens[s]) - 1] for s in seq_ids]
        bts = [self.blocks.get_block_table(s) for s in seq_ids]
        slot = [len(self.tokens[s]) - 1 for s in seq_ids]
        ncached = list(slot)
        return ids, pos, bts, slot, ncached

    def decode(self, seq_ids: list[int]) -> torch.Tensor:
        """One batched decode forward; returns fp32 logits ``[B, V]`` (``engine.py:297-353``)."""
        ids, pos, bts, slot, ncached = self.decode_inputs(seq_ids)
        max_cached = max(n + 1 for n in ncached)
        mask = torch.zeros(len(seq_ids), 1, 1, max_cached, dtype=self.dtype, device=self.device)
        for i, n in enumerate(ncached):
            if n + 1 < max_cached:
                mask[i, :, :, n + 1:] = float("-inf")
        with torch.no_grad(), self._autocast():
            logits = self.model.forward(torch.tensor(ids, device=self.device), torch.tensor(pos, device=self.device),
                                        self.kv_pool, bts, slot, use_cache=True, num_cached=ncached, attn_mask=mask)
        return logits[:, -1, :].float()

    def append(self, seq_id: int, token: int) -> None:
        self.tokens[seq_id].append(token)

    def generate_greedy(self, prompts: list[list[int]], max_tokens: int) -> tuple[list[list[int]], list[torch.Tensor]]:
        """Greedy generation (temperature 0): prefill each, then batched decode steps."""
        seq_ids = list(range(len(prompts)))
        for s, p in zip(seq_ids, prompts):
            self.append(s, int(osamp.greedy(self.prefill(s, p)[None])[0]))
        step_logits = []
        for _ in range(max_tokens - 1):
            lg = self.decode(seq_ids)
            step_logits.append(lg)
            for s, t in zip(seq_ids, osamp.greedy(lg).tolist()):
                self.append(s, int(t))
        return [self.tokens[s][self.prompt_len[s]:] for s in seq_ids], step_logits
