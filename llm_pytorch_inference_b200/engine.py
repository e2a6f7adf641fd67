"""Batched decode engine: the reference's ``LLMEngine._run_decode`` loop on the B200 path.

``mini_vllm/engine/engine.py:297-360`` does, per step: ``append_token`` on every
sequence's KV blocks, builds ``input_ids`` / ``positions`` / block tables / slot
indices / a padding mask from Python lists (about 130 small host->device copies per
layer), runs the model, then samples each sequence separately with a host sync per
sequence, appends the token and frees every sequence that finished.  Here the same
bookkeeping is done on the host into a pinned int32 buffer, updated incrementally (a
block id is written only when a sequence grows a block), then one host->device copy,
one CUDA-graph replay of the whole step (forward + sampling for all rows) and one
device->host copy of the sampled tokens.

Block allocation is the reference's FIFO ``KVCacheManager`` (bit-exact block ids).
Positions follow ``engine.py:316``/``:326``: a sequence of length n decodes its last
token at position n-1, writes K/V to slot n-1 and attends to n tokens.

Finishing follows ``Sequence.is_finished`` (``engine/sequence.py:66-80``): a sequence is
done once it has ``max_tokens`` output tokens or its last output token is one of its stop
ids.  Finished sequences are freed in row order right after the step that finished them
(``engine.py:288-294``, ``:352-359``), their rows are compacted away, and the freed blocks go
to the tail of the free list exactly as the reference's ``free`` puts them; a sequence whose
``append_token`` finds the pool empty is dropped from the step and freed (``engine.py:299-309``).

The host bookkeeping lives in ``RunningBatch`` (no GPU needed); ``DecodeEngine`` adds the
device weights, the KV pool and the step runner.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _native as N
from .configs import head_dim
from .kv_cache import KVCacheManager, num_blocks_for_budget
from .runner import DecodeRunner, DecodeWeights, meta_layout, resolve_device
from .tensor_parallel import TensorParallelConfig, local_kv_heads, shard_state_dict


@dataclass
class SeqSampling:
    """A sequence's sampling parameters (``SamplingParams``, ``utils/config.py:61-68``):
    T == 0 is greedy; ``top_k`` <= 0 and ``top_p`` >= 1 disable the filters."""
    temperature: float = 0.0
    top_k: int = -1
    top_p: float = 1.0


class RunningBatch:
    """The running decode set and its per-step metadata (host side only).

    ``meta`` is the int32 metadata buffer of ``runner.meta_layout(batch, max_blocks)`` (the
    pinned host mirror of the device buffer in ``DecodeEngine``).  Rows are the running
    sequences in the order they were added (the reference's ``running_seqs`` order,
    ``scheduler.py:36-40``); rows past the running count are padding that writes into the
    pool's scratch block and attends to one token there."""

    def __init__(self, kv: KVCacheManager, batch: int, max_blocks: int, meta: np.ndarray | None = None):
        self.kv = kv
        self.B = batch
        self.max_blocks = max_blocks
        lay = meta_layout(batch, max_blocks)
        self.meta_np = np.zeros(lay["total"], dtype=np.int32) if meta is None else meta
        m, B = self.meta_np, batch
        self._ids = m[0:B]
        self._pos = m[lay["pos"]:lay["pos"] + B]
        self._ctx = m[lay["ctx"]:lay["ctx"] + B]
        self._off = m[lay["off"]:lay["off"] + 2].view(np.int64)
        self._temp = m[lay["temp"]:lay["temp"] + B].view(np.float32)
        self._topk = m[lay["topk"]:lay["topk"] + B]
        self._topp = m[lay["topp"]:lay["topp"] + B].view(np.float32)
        self._bt = m[lay["bt"]:].reshape(B, max_blocks)
        self.seqs: list[int] = []                     # running sequence ids, one per batch row
        self.tokens: dict[int, list[int]] = {}
        self.prompt_len: dict[int, int] = {}
        self.max_tokens: dict[int, int | None] = {}
        self.stop_ids: dict[int, frozenset[int]] = {}
        self.sampling: dict[int, SeqSampling | None] = {}
        self.default_sampling = SeqSampling()
        self.finish_reason: dict[int, str] = {}     # every finished sequence: "length" | "stop" | "abort"
        self.finished_last: list[int] = []           # sequences finished by the last call
        self.last_step_seqs: list[int] = []          # the sequences the last step decoded, in row order
        self.held: set[int] = set()                  # rows that sit out the next decode (joined in it)
        self.step_count = 0
        # Per-row mirrors for the vectorised common step (see _mirrors), valid while the running
        # rows are exactly _mir_seqs; every general path drops them.
        self._mir_seqs: list[int] | None = None
        self._mir_ntok = self._mir_nblk = self._mir_left = None
        self._mir_stop_rows: list[int] = []

    # ------------------------------------------------------------------ sequences
    def add_sequence(self, seq_id: int, prompt: list[int], max_tokens: int | None = None,
                     stop_token_ids=(), sampling: SeqSampling | None = None) -> list[int] | None:
        """Registers a sequence and allocates ``len(prompt) + 1`` tokens of blocks, as the
        reference's prefill does (``engine.py:262``).  If the pool cannot hold it, the sequence
        finishes unstarted (reason "abort") and ``None`` is returned, as ``engine.py:263-268``
        does.  ``max_tokens`` None means no length limit."""
        if seq_id in self.tokens:
            raise ValueError(f"sequence {seq_id} already exists")
        if len(self.seqs) >= self.B:
            raise RuntimeError("engine is full")
        bt = self.kv.allocate(seq_id, len(prompt) + 1)
        self.tokens[seq_id] = list(prompt)
        self.prompt_len[seq_id] = len(prompt)
        self.max_tokens[seq_id] = max_tokens
        self.stop_ids[seq_id] = frozenset(int(t) for t in stop_token_ids)
        self.sampling[seq_id] = sampling
        if bt is None:
            self.finish_reason[seq_id] = "abort"
            return None
        if len(bt) > self.max_blocks:
            self.kv.free(seq_id)
            raise RuntimeError(f"sequence {seq_id} exceeds max_model_len")
        self.seqs.append(seq_id)
        return bt

    def output_len(self, seq_id: int) -> int:
        return len(self.tokens[seq_id]) - self.prompt_len[seq_id]

    def is_finished(self, seq_id: int) -> bool:
        """``Sequence.is_finished`` (``sequence.py:66-72``)."""
        if seq_id in self.finish_reason:
            return True
        n = self.output_len(seq_id)
        mt = self.max_tokens[seq_id]
        if mt is not None and n >= mt:
            return True
        return n > 0 and self.tokens[seq_id][-1] in self.stop_ids[seq_id]

    def _reason(self, seq_id: int) -> str:
        mt = self.max_tokens[seq_id]
        return "length" if mt is not None and self.output_len(seq_id) >= mt else "stop"

    def _release(self, seq_id: int, reason: str) -> None:
        self.kv.free(seq_id)
        self.finish_reason[seq_id] = reason
        self.finished_last.append(seq_id)

    def finish(self, seq_id: int, reason: str = "abort") -> None:
        """Ends a running sequence now: frees its blocks (to the free list's tail) and removes
        its row; the remaining rows keep their order."""
        if seq_id not in self.seqs:
            raise KeyError(f"sequence {seq_id} is not running")
        self.finished_last = []
        self.held.discard(seq_id)
        self._release(seq_id, reason)
        self.seqs.remove(seq_id)
        self._refresh_rows()

    def append_first_token(self, seq_id: int, token: int) -> bool:
        """The token the prefill sampled (``engine.py:288-294``); a sequence that is already
        finished by it is freed at once.  Returns whether it finished."""
        self.tokens[seq_id].append(int(token))
        if self.is_finished(seq_id):
            self._release(seq_id, self._reason(seq_id))
            self.seqs.remove(seq_id)
            return True
        return False

    # ---------------------------------------------------------------------- rows
    def _row_sampling(self, seq_id: int) -> SeqSampling:
        return self.sampling.get(seq_id) or self.default_sampling

    def _refresh_rows(self) -> None:
        """Full rewrite of the metadata rows (after sequences were added or removed)."""
        self._mir_seqs = None
        self._bt.fill(self.kv.scratch_block)
        self._ids.fill(0)
        self._pos.fill(0)
        self._ctx.fill(1)
        self._temp.fill(0.0)
        self._topk.fill(-1)
        self._topp.fill(1.0)
        for row, s in enumerate(self.seqs):
            bt = self.kv.get_block_table(s)
            self._bt[row, :len(bt)] = bt
            n = len(self.tokens[s])
            self._ids[row] = self.tokens[s][-1]
            self._pos[row] = n - 1
            self._ctx[row] = n
            sp = self._row_sampling(s)
            self._temp[row], self._topk[row], self._topp[row] = sp.temperature, sp.top_k, sp.top_p

    def set_default_sampling(self, temperature=0.0, top_k=-1, top_p=1.0) -> None:
        """Sampling of every sequence added without its own parameters."""
        self.default_sampling = SeqSampling(float(temperature), int(top_k), float(top_p))
        self._refresh_rows()

    def start(self) -> None:
        """Call after adding sequences (and before the first step)."""
        self._refresh_rows()

    prepare_first_step = start

    def _grow_blocks(self) -> None:
        """``engine.py:299-309``: one more token per decoded sequence, a new block when needed;
        a sequence the pool cannot grow is freed and leaves the batch before the step runs.
        Held rows (sequences that joined in this step) are written as padding rows."""
        if not self.held and self._grow_fast():
            self.last_step_seqs = list(self.seqs)
            self._off[0] = self.step_count
            return
        self._mir_seqs = None
        dropped = False
        for row, s in enumerate(list(self.seqs)):
            if s in self.held:
                continue
            nb = len(self.kv.get_block_table(s))
            if not self.kv.append_token(s) or len(self.kv.get_block_table(s)) > self.max_blocks:
                self._release(s, "abort")
                dropped = True
                continue
            if not dropped:
                bt = self.kv.get_block_table(s)
                if len(bt) > nb:
                    self._bt[row, nb:len(bt)] = bt[nb:]
        if dropped:
            self.seqs = [s for s in self.seqs if s not in self.finish_reason]
            self._refresh_rows()
        for row, s in enumerate(self.seqs):
            if s in self.held:
                self._bt[row].fill(self.kv.scratch_block)
                self._ids[row], self._pos[row], self._ctx[row], self._temp[row] = 0, 0, 1, 0.0
        self.last_step_seqs = [s for s in self.seqs if s not in self.held]
        # the sampling offset of this step (fresh Philox uniforms every step)
        self._off[0] = self.step_count

    def _mirrors(self) -> None:
        """Builds the per-row mirrors of the running rows unless they are current: tokens and
        blocks held (``KVCacheManager.seq_num_tokens`` / block-table lengths), output tokens left
        before "length", and the rows that have stop ids."""
        if self._mir_seqs is not None and self._mir_seqs == self.seqs:
            return
        seqs, kv = self.seqs, self.kv
        self._mir_ntok = np.array([kv.seq_num_tokens[q] for q in seqs], dtype=np.int64)
        self._mir_nblk = np.array([len(kv.block_tables[q]) for q in seqs], dtype=np.int64)
        big = 1 << 62
        self._mir_left = np.array([big if self.max_tokens[q] is None else self.max_tokens[q] - self.output_len(q)
                                   for q in seqs], dtype=np.int64)
        self._mir_stop_rows = [row for row, q in enumerate(seqs) if self.stop_ids[q]]
        self._mir_seqs = list(seqs)

    def _grow_fast(self) -> bool:
        """The common step (no held rows): ``KVCacheManager.append_token`` for every row in row
        order, vectorised over the row mirrors; only the rows that cross a block boundary take a
        block from the free list (in row order).  Gives up (returns False, nothing changed) when
        some row would need a block beyond the pool or the block table, where the general path
        frees and drops sequences in the reference's order."""
        kv = self.kv
        self._mirrors()
        ntok = self._mir_ntok + 1
        grow = np.flatnonzero(ntok > self._mir_nblk * kv.block_size)
        if grow.size:
            if int(self._mir_nblk[grow].max()) + 1 > self.max_blocks or grow.size > len(kv.free_blocks):
                return False
            free, tables, seqs = kv.free_blocks, kv.block_tables, self.seqs
            for row in grow.tolist():
                bt = tables[seqs[row]]
                bt.append(free.popleft())
                self._bt[row, len(bt) - 1] = bt[-1]
            self._mir_nblk[grow] += 1
        self._mir_ntok = ntok
        kv.seq_num_tokens.update(zip(self.seqs, ntok.tolist()))
        return True

    def _commit(self, out: list[int]) -> None:
        """The sampled tokens (one per row of the step) become each decoded row's last token
        and positions advance by one; then every sequence this step finished is freed in row
        order and its row removed (``engine.py:352-359``)."""
        rows = list(self.seqs)
        n = len(rows)
        fast = not self.held and self._mir_seqs is not None and self._mir_seqs == rows
        if self.held:
            self._mir_seqs = None
            for row, s in enumerate(rows):
                if s in self.held:
                    continue
                self.tokens[s].append(int(out[row]))
                self._ids[row] = int(out[row])
        else:
            toks = [int(t) for t in out[:n]]
            for s, t in zip(rows, toks):
                self.tokens[s].append(t)
            self._ids[:n] = toks
        self._pos[:n] += 1
        self._ctx[:n] += 1
        self.step_count += 1
        if fast:
            # Sequence.is_finished over the row mirrors: the length limit for every row, the stop
            # ids only for the rows that have some.
            self._mir_left -= 1
            fin = set(np.flatnonzero(self._mir_left <= 0).tolist())
            fin.update(row for row in self._mir_stop_rows if toks[row] in self.stop_ids[rows[row]])
            done = [rows[row] for row in sorted(fin)]
        else:
            done = [s for s in rows if s not in self.held and self.is_finished(s)]
        for s in done:
            self._release(s, self._reason(s))
        if done or self.held:
            self.held = set()
            self.seqs = [s for s in rows if s not in self.finish_reason]
            self._refresh_rows()

    def plan_step(self, tokens: list[int]) -> np.ndarray:
        """Host bookkeeping of one step without running it: returns that step's metadata (a
        copy) and commits ``tokens`` (one per row of the step, held rows included) as if they
        had been sampled."""
        self.finished_last = []
        self._grow_blocks()
        snap = self.meta_np.copy()
        rows = len(self.seqs)
        self._commit(list(tokens[:rows]) + [0] * (rows - len(tokens)))
        return snap

    def plan_schedule_step(self, new: dict[int, tuple], tokens: dict[int, int]) -> np.ndarray | None:
        """Host bookkeeping of one reference ``LLMEngine._step`` (``engine.py:241-251``) with
        given tokens: first the new sequences, in order, each allocated, given its first token
        (``new[seq] = (prompt, first_token, max_tokens, stop_token_ids)``) and freed at once if
        that finishes it (``_run_prefill``, ``:253-294``); then one decode step of the sequences
        that were running before them (``_run_decode``), whose sampled tokens are
        ``tokens[seq]``.  Returns the decode step's metadata, or None if nothing was running."""
        self.finished_last = []
        before = [s for s in self.seqs]
        for s, (prompt, first, max_tokens, stop) in new.items():
            if self.add_sequence(s, prompt, max_tokens, stop) is not None:
                self.append_first_token(s, first)
        self.held = {s for s in self.seqs if s not in before}
        if not before:
            self.held = set()
            self._refresh_rows()
            return None
        self._grow_blocks()
        snap = self.meta_np.copy()
        self._commit([tokens.get(s, 0) for s in self.seqs])
        return snap

    def force_last_tokens(self, tokens: list[int]) -> None:
        """Replaces the token each row sampled last (teacher forcing for parity checks)."""
        for row, s in enumerate(self.seqs):
            self.tokens[s][-1] = int(tokens[row])
            self._ids[row] = int(tokens[row])

    def force_tokens(self, tokens: dict[int, int]) -> None:
        """Replaces the last token of the given running sequences (by sequence id)."""
        for row, s in enumerate(self.seqs):
            if s in tokens:
                self.tokens[s][-1] = int(tokens[s])
                self._ids[row] = int(tokens[s])

    def output_tokens(self, seq_id: int) -> list[int]:
        return self.tokens[seq_id][self.prompt_len[seq_id]:]

    @property
    def has_unfinished(self) -> bool:
        return bool(self.seqs)


class DecodeEngine(RunningBatch):
    """``tp``: this process's place in a tensor-parallel group (one engine per GPU, every rank
    driven with the same calls); ``state_dict`` is the full model, sharded here."""

    def __init__(self, cfg: dict, state_dict: dict[str, torch.Tensor], max_batch: int, max_model_len: int,
                 num_blocks: int | None = None, device="cuda", free_order: list[int] | None = None,
                 hbm_budget_bytes: int | None = None, tp: TensorParallelConfig | None = None,
                 fused_layers: bool = False):
        """``fused_layers``: the dense step's layers as one persistent launch each after attention
        (``DecodeRunner``); off by default."""
        self.cfg = cfg
        self.dev = resolve_device(device)
        self.tp = tp or TensorParallelConfig()
        T = self.tp.tp_size
        sd = shard_state_dict(cfg, state_dict, T, self.tp.rank) if T > 1 else state_dict
        self.weights = DecodeWeights(cfg, sd, self.dev)
        del sd
        L, nkv, D = cfg["num_hidden_layers"], local_kv_heads(cfg, T), head_dim(cfg)
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
        kv = KVCacheManager(num_blocks, 16, L, nkv, D, device=self.dev, dtype=torch.bfloat16, free_order=free_order)
        self.runner = DecodeRunner(cfg, self.weights, kv, max_batch, max_model_len, self.dev, tp=self.tp,
                                   fused_layers=fused_layers)
        super().__init__(kv, self.runner.B, self.runner.max_blocks, self.runner.meta_host.numpy())
        self._prefill = None
        self.last_prefill_logits = None
        self.parity = False
        self.parity_generator: torch.Generator | None = None
        self.steps_run_ahead = 0   # steps run_steps launched before reading the previous step's tokens

    def prefill(self, prompts: dict[int, list[int]], temperature: float = 0.0, top_k: int = -1, top_p: float = 1.0,
                seed: int = 0, max_tokens: int = 16384, gen_max_tokens: dict[int, int | None] | None = None,
                stop_token_ids=()) -> dict[int, int]:
        """``engine.py:253-294`` for a batch of new sequences on the GPU: registers each (blocks
        for ``len(prompt) + 1`` tokens), prefills all of them in one packed token batch
        (``prefill.BatchedPrefill``), samples each first token from its last position's logits
        and appends it; a sequence that this first token finishes is freed.  ``max_tokens``
        bounds the packed prompt tokens of one chunk; ``gen_max_tokens`` gives a sequence's
        output limit.  Returns seq_id -> first token; ``last_prefill_logits`` keeps the logits."""
        from .prefill import BatchedPrefill

        self.finished_last = []
        if self._prefill is None or self._prefill.max_tokens < max_tokens:
            self._prefill = BatchedPrefill(self.runner, max_tokens)
        gen_max_tokens = gen_max_tokens or {}
        sids, tables = [], []
        for s in prompts:
            bt = self.add_sequence(s, prompts[s], gen_max_tokens.get(s), stop_token_ids)
            if bt is not None:
                sids.append(s)
                tables.append(bt)
        if not sids:
            return {}
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
        """Fills every prompt position of every running sequence with seeded N(0,1) K/V."""
        g = torch.Generator(device=self.dev).manual_seed(seed)
        pool = self.kv.kv_cache
        for s in self.seqs:
            for blk in self.kv.get_block_table(s):
                pool[:, :, blk].normal_(0.0, 1.0, generator=g)

    # ---------------------------------------------------------------------- step
    def set_sampling(self, temperature=0.0, top_k=-1, top_p=1.0, seed: int = 0, parity: bool = False,
                     generator: torch.Generator | None = None) -> None:
        """Sampling of every sequence added without its own parameters.

        Fast mode (default): the step's sampler kernel draws in-kernel (Philox4x32-10, one
        uniform per row, inverse CDF over the filtered distribution).  ``parity=True``: the
        kernel writes each row's filtered, tempered probabilities and the draw is the
        reference's own -- ``torch.multinomial(probs, 1)`` per row in row order
        (``ops/sampling.py:69-73`` via ``sampler.py:40-48``, ``engine.py:352-354``) on
        ``generator`` (default: torch's default generator of the device, the one the reference
        draws from).  Greedy rows take the kernel's argmax in both modes."""
        self.set_default_sampling(temperature, top_k, top_p)
        if self.runner.seed != int(seed):
            self.runner.seed = int(seed)
            self.runner.graph = None
        self.parity = bool(parity)
        self.parity_generator = generator
        self.runner.set_probs_out(self.parity)

    def _parity_draw(self, n: int) -> list[int]:
        """Row-by-row ``torch.multinomial`` on the kernel's probabilities (rows with T > 0)."""
        r = self.runner
        greedy = r.tokens[:n].tolist()
        out = []
        for row in range(n):
            if self._temp[row] > 0.0:
                t = torch.multinomial(r.probs[row:row + 1], 1, generator=self.parity_generator)
                out.append(int(t.item()))
            else:
                out.append(int(greedy[row]))
        return out

    def _decode(self, use_graph: bool) -> list[int]:
        self._grow_blocks()
        rows = list(self.seqs)
        decoded = set(self.last_step_seqs)
        if not decoded:
            if rows:   # every row joined in this step: nothing to decode, the rows go live
                self.held = set()
                self._refresh_rows()
            return []
        self.runner.step(use_graph)
        if self.parity:
            out = self._parity_draw(len(rows))
        else:
            out = self.runner.fetch_tokens()[:len(rows)].tolist()
        self._commit(out)
        return [out[i] for i, s in enumerate(rows) if s in decoded]

    def step(self, use_graph: bool = True) -> list[int]:
        """One decode step for every running sequence: host bookkeeping, one host->device copy
        of the step's metadata, one graph replay (forward + sampling), one device->host copy of
        the sampled tokens.  Returns the tokens of the decoded sequences (``last_step_seqs``, row
        order); the sequences that finished are in ``finished_last``."""
        self.finished_last = []
        return self._decode(use_graph)

    def run_steps(self, n: int) -> list[list[int]]:
        """``n`` decode steps, each exactly as ``step()`` would take it (same tokens, block
        tables, free list and finishes); returns each step's tokens.  While step k runs, the host
        already launches step k+1 when every row of the batch is a running sequence, none can
        finish at step k (no length limit reached, no stop ids), no row joins and the growth of
        step k+1 fits: step k+1 then takes
        its input ids from step k's sampled tokens on the device (``mvb_feed_ids``), and the
        token read-back and the bookkeeping of step k overlap step k+1 instead of leaving the GPU
        idle.  Otherwise step k's tokens are read and committed first, as ``step()`` does.
        ``finished_last`` lists the sequences that finished in any of the ``n`` steps."""
        finished = []
        out: list[list[int]] = []
        pending = None   # (rows, decoded rows, token buffer) of the step on the device
        for k in range(n):
            self.finished_last = []
            if pending is None:
                if self.parity:   # the reference's host-side draw needs each step's probabilities
                    out.append(self._decode(True))
                    finished += self.finished_last
                    continue
                self._grow_blocks()
                rows = list(self.seqs)
                decoded = set(self.last_step_seqs)
                if not decoded:
                    if rows:
                        self.held = set()
                        self._refresh_rows()
                    out.append([])
                    continue
                pending = (rows, decoded, self.runner.launch_staged(feed=False))
            rows, decoded, buf = pending
            pending = None
            if k + 1 < n and self._can_run_ahead():
                # Step k's position advance and step k+1's growth, without step k's tokens.
                m = len(rows)
                self._pos[:m] += 1
                self._ctx[:m] += 1
                self.step_count += 1
                self._mir_left -= 1
                self._grow_blocks()
                pending = (list(self.seqs), set(self.last_step_seqs), self.runner.launch_staged(feed=True))
                self.steps_run_ahead += 1
                toks = self.runner.tokens_of(buf)[:m].tolist()
                for s, t in zip(rows, toks):
                    self.tokens[s].append(t)
                self._ids[:m] = toks
            else:
                toks = self.runner.tokens_of(buf)[:len(rows)].tolist()
                self._commit(toks)
            out.append([toks[i] for i, s in enumerate(rows) if s in decoded])
            finished += self.finished_last
        self.finished_last = finished
        return out

    def _can_run_ahead(self) -> bool:
        """Whether the next step can be launched before this step's tokens are read: every row
        of the batch is a running sequence (the id feed copies all rows, and a padding row must
        keep its id 0: in a sparse-MoE step its routing would otherwise change how the experts'
        rows are split), the rows are the ones of the row mirrors, none joins, none can finish
        with this step's token (no length limit reached, no stop ids) and the next step's block
        growth takes the fast path."""
        if self.held or self.parity or len(self.seqs) != self.B or self._mir_seqs is None \
                or self._mir_seqs != self.seqs:
            return False
        if self.runner.graph is None:   # a capture replays the step eagerly first: never with fed ids
            return False
        if self._mir_stop_rows or int(self._mir_left.min()) <= 1:
            return False
        ntok = self._mir_ntok + 1
        grow = np.flatnonzero(ntok > self._mir_nblk * self.kv.block_size)
        if grow.size and (int(self._mir_nblk[grow].max()) + 1 > self.max_blocks or grow.size > len(self.kv.free_blocks)):
            return False
        return True

    def schedule_step(self, new_prompts: dict[int, list[int]] | None = None, use_graph: bool = True,
                      gen_max_tokens: dict[int, int | None] | None = None, stop_token_ids=()) -> dict[int, int]:
        """The reference's ``LLMEngine._step`` (``engine.py:241-251``) for continuous batching:
        the new sequences are prefilled first (their blocks allocated before any decode growth)
        and get their first token; then the sequences that were running before them take one
        decode step, the new rows sitting it out.  Returns seq_id -> the token it got.  The new
        prompts are sampled with the engine's default sampling parameters."""
        self.finished_last = []
        before = set(self.seqs)
        sp = self.default_sampling
        got = {}
        if new_prompts:
            got = self.prefill(new_prompts, sp.temperature, sp.top_k, sp.top_p, seed=self.step_count,
                               gen_max_tokens=gen_max_tokens, stop_token_ids=stop_token_ids)
        self.held = {s for s in self.seqs if s not in before}
        if not before:
            self.held = set()
            self._refresh_rows()
            return got
        out = self._decode(use_graph)
        got.update(zip(self.last_step_seqs, out))
        return got

    def plan_step(self, tokens: list[int]) -> torch.Tensor:
        """As ``RunningBatch.plan_step``, the snapshot as an int32 tensor (pinned-buffer layout)."""
        return torch.from_numpy(super().plan_step(tokens))
