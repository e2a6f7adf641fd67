"""Batched decode engine: the reference's ``LLMEngine._run_decode`` loop on the B200 path.

``mini_vllm/engine/engine.py:297-360`` does, per step: ``append_token`` on every
sequence's KV blocks, builds ``input_ids`` / ``positions`` / block tables / slot
indices / a padding mask from Python lists (about 130 small host->device copies per
layer), runs the model, then samples each sequence separately with a host sync per
sequence.  Here the same bookkeeping is done on the host into a pinned int32 buffer,
updated incrementally (a block id is written only when a sequence grows a block),
then one host->device copy, one CUDA-graph replay of the whole step (forward +
sampling for all rows) and one device->host copy of the sampled tokens.

Block allocation is the reference's FIFO ``KVCacheManager`` (bit-exact block ids).
Positions follow ``engine.py:316``/``:326``: a sequence of length n decodes its last
token at position n-1, writes K/V to slot n-1 and attends to n tokens.

Prefill (``engine.py:253-295``) is not part of the decode path: ``load_prefilled``
takes a KV state built elsewhere (the oracle, or the reference), and
``prefill_synthetic`` fills the prompt positions with seeded random K/V for
throughput measurements.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _native as N
from .configs import head_dim, num_kv_heads
from .kv_cache import KVCacheManager, num_blocks_for_budget
from .runner import DecodeRunner, DecodeWeights, resolve_device
from .tensor_parallel import TensorParallelConfig, shard_state_dict


class DecodeEngine:
    """``tp``: this process's place in a tensor-parallel group (one engine per GPU, every rank
    driven with the same calls); ``state_dict`` is the full model, sharded here."""

    def __init__(self, cfg: dict, state_dict: dict[str, torch.Tensor], max_batch: int, max_model_len: int,
                 num_blocks: int | None = None, device="cuda", free_order: list[int] | None = None,
                 hbm_budget_bytes: int | None = None, tp: TensorParallelConfig | None = None):
        self.cfg = cfg
        self.dev = resolve_device(device)
        self.tp = tp or TensorParallelConfig()
        T = self.tp.tp_size
        sd = shard_state_dict(cfg, state_dict, T, self.tp.rank) if T > 1 else state_dict
        self.weights = DecodeWeights(cfg, sd, self.dev)
        del sd
        L, nkv, D = cfg["num_hidden_layers"], num_kv_heads(cfg) // T, head_dim(cfg)
        if num_blocks is None:
            free, _ = torch.cuda.mem_get_info(self.dev)
            kw = {} if hbm_budget_bytes is None else {"budget_bytes": hbm_budget_bytes}
            num_blocks = num_blocks_for_budget(16, nkv, D, L, 2, self.weights.nbytes(), 1 << 30,
                                               device_free_bytes=free, **kw)
            if T > 1:   # block ids are replicated: every rank needs the same pool size
                import torch.distributed as dist

                t = torch.tensor([num_blocks], dtype=torch.int64, device=self.dev)
                dist.all_reduce(t, op=dist.ReduceOp.MIN)
                num_blocks = int(t.item())
        self.kv = KVCacheManager(num_blocks, 16, L, nkv, D, device=self.dev, dtype=torch.bfloat16,
                                 free_order=free_order)
        self.runner = DecodeRunner(cfg, self.weights, self.kv, max_batch, max_model_len, self.dev, tp=self.tp)
        self.seqs: list[int] = []                     # active sequence ids, one per batch row
        self.tokens: dict[int, list[int]] = {}
        self.prompt_len: dict[int, int] = {}
        self.step_count = 0
        self._prefill = None
        self.last_prefill_logits = None
        m = self.runner.meta_host.numpy()
        r = self.runner
        self._ids = m[0:r.B]
        self._pos = m[r._o_pos:r._o_pos + r.B]
        self._ctx = m[r._o_ctx:r._o_ctx + r.B]
        self._off = m[r._o_off:r._o_off + 2].view(np.int64)
        self._bt = m[r._o_bt:].reshape(r.B, r.max_blocks)

    # ------------------------------------------------------------------ sequences
    def add_sequence(self, seq_id: int, prompt: list[int]) -> list[int]:
        """Registers a sequence and allocates ``len(prompt) + 1`` tokens of blocks, as the
        reference's prefill does (``engine.py:262``)."""
        if len(self.seqs) >= self.runner.B:
            raise RuntimeError("engine is full")
        bt = self.kv.allocate(seq_id, len(prompt) + 1)
        if bt is None:
            raise RuntimeError(f"KV pool exhausted allocating sequence {seq_id}")
        self.seqs.append(seq_id)
        self.tokens[seq_id] = list(prompt)
        self.prompt_len[seq_id] = len(prompt)
        return bt

    def append_first_token(self, seq_id: int, token: int) -> None:
        """The token the prefill sampled (``engine.py:288-290``)."""
        self.tokens[seq_id].append(int(token))

    def prefill(self, prompts: dict[int, list[int]], temperature: float = 0.0, top_k: int = -1, top_p: float = 1.0,
                seed: int = 0, max_tokens: int = 16384) -> dict[int, int]:
        """``engine.py:253-290`` for a batch of new sequences on the GPU: registers each (blocks for
        ``len(prompt) + 1`` tokens), prefills all of them in one packed token batch
        (``prefill.BatchedPrefill``), samples each first token from its last position's logits and
        appends it.  Returns seq_id -> first token; ``last_prefill_logits`` keeps the logits."""
        from .prefill import BatchedPrefill

        if self._prefill is None or self._prefill.max_tokens < max_tokens:
            self._prefill = BatchedPrefill(self.runner, max_tokens)
        sids = list(prompts)
        tables = [self.add_sequence(s, prompts[s]) for s in sids]
        logits = self._prefill.run([prompts[s] for s in sids], tables)
        n = len(sids)
        lib = N.lib()
        out = torch.zeros(n, dtype=torch.int64, device=self.dev)
        temp = torch.full((n,), float(temperature), dtype=torch.float32, device=self.dev)
        tk = torch.full((n,), int(top_k), dtype=torch.int32, device=self.dev)
        tp = torch.full((n,), float(top_p), dtype=torch.float32, device=self.dev)
        N.check(lib.mvb_sample(out.data_ptr(), None, logits.data_ptr(), n, logits.shape[1], logits.stride(0),
                               temp.data_ptr(), tk.data_ptr(), tp.data_ptr(), int(seed), 0, None, N.BF16,
                               N.stream_handle(self.dev)), "sample")
        first = out.cpu().tolist()
        self.last_prefill_logits = logits
        for s, t in zip(sids, first):
            self.append_first_token(s, t)
        self._refresh_rows()   # ready for the first decode step
        return dict(zip(sids, first))

    def load_prefilled(self, kv_pool: torch.Tensor) -> None:
        """Copies a prefilled pool ``[L, 2, P, 16, Hkv, D]`` (same block ids) into the device pool."""
        P = kv_pool.shape[2]
        self.kv.kv_cache[:, :, :P].copy_(kv_pool.to(self.dev, torch.bfloat16))

    def prefill_synthetic(self, seed: int = 0) -> None:
        """Fills every prompt position of every active sequence with seeded N(0,1) K/V."""
        g = torch.Generator(device=self.dev).manual_seed(seed)
        pool = self.kv.kv_cache
        for s in self.seqs:
            for blk in self.kv.get_block_table(s):
                pool[:, :, blk].normal_(0.0, 1.0, generator=g)

    # ---------------------------------------------------------------------- step
    def _refresh_rows(self) -> None:
        """Full rewrite of the metadata rows (after sequences were added or removed)."""
        self._bt.fill(self.kv.scratch_block)
        self._ids.fill(0)
        self._pos.fill(0)
        self._ctx.fill(1)
        for row, s in enumerate(self.seqs):
            bt = self.kv.get_block_table(s)
            self._bt[row, :len(bt)] = bt
            n = len(self.tokens[s])
            self._ids[row] = self.tokens[s][-1]
            self._pos[row] = n - 1
            self._ctx[row] = n
        self._rows_dirty = False

    def set_sampling(self, temperature=0.0, top_k=-1, top_p=1.0, seed: int = 0) -> None:
        self.runner.set_sampling(temperature, top_k, top_p, seed)

    def start(self) -> None:
        """Call after adding sequences (and before the first step)."""
        self._refresh_rows()

    def _grow_blocks(self) -> None:
        """``engine.py:299-309``: one more token per sequence, a new block when needed."""
        r = self.runner
        for row, s in enumerate(self.seqs):
            nb = len(self.kv.get_block_table(s))
            if not self.kv.append_token(s):
                raise RuntimeError(f"KV pool exhausted while growing sequence {s}")
            bt = self.kv.get_block_table(s)
            if len(bt) > nb:
                if len(bt) > r.max_blocks:
                    raise RuntimeError(f"sequence {s} exceeds max_model_len")
                self._bt[row, nb:len(bt)] = bt[nb:]
        # the sampling offset of this step (fresh Philox uniforms every step)
        self._off[0] = self.step_count

    def _commit(self, out: list[int]) -> None:
        """The sampled tokens become each row's last token; positions advance by one."""
        for row, s in enumerate(self.seqs):
            self.tokens[s].append(int(out[row]))
            self._ids[row] = int(out[row])
        n = len(self.seqs)
        self._pos[:n] += 1
        self._ctx[:n] += 1
        self.step_count += 1

    def step(self, use_graph: bool = True) -> list[int]:
        """One decode step for every active sequence: host bookkeeping, one host->device copy of
        the step's metadata, one graph replay (forward + sampling), one device->host copy of the
        sampled tokens.  Returns the tokens in row order."""
        self._grow_blocks()
        self.runner.step(use_graph)
        out = self.runner.fetch_tokens()[:len(self.seqs)].tolist()
        self._commit(out)
        return out

    def plan_step(self, tokens: list[int]) -> torch.Tensor:
        """Host bookkeeping of one step without running it: returns that step's metadata
        (a copy of the pinned buffer) and commits ``tokens`` as if they had been sampled."""
        self._grow_blocks()
        snap = self.runner.meta_host.clone()
        self._commit(tokens)
        return snap

    def force_last_tokens(self, tokens: list[int]) -> None:
        """Replaces the token each row sampled last (teacher forcing for parity checks)."""
        for row, s in enumerate(self.seqs):
            self.tokens[s][-1] = int(tokens[row])
            self._ids[row] = int(tokens[row])

    def prepare_first_step(self) -> None:
        """Positions of the first decode step: a sequence of n tokens decodes token n-1."""
        self._refresh_rows()

    def output_tokens(self, seq_id: int) -> list[int]:
        return self.tokens[seq_id][self.prompt_len[seq_id]:]
