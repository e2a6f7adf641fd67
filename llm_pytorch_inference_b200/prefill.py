"""Batched varlen prefill over the paged KV pool, on the decode path's kernels.

Replaces ``LLMEngine._run_prefill`` (``mini_vllm/engine/engine.py:253-295``), which runs the model
once per sequence (``ForCausalLM.forward`` with ``use_cache=False``: causal SDPA over the prompt,
``Attention._write_kv_cache`` for every position, ``models/model.py:154-243``) and samples the first
token from the last position's logits.  Here all prompts of a call are packed into one token batch
(row r = token i of sequence s) and every layer runs once over all of them:

* RMSNorm, the q|k|v GEMM over all rows (tcgen05, row tiles of 256), per-head QK-norm + RoPE and the
  paged KV write of every token (one row per token: its sequence's block table, its position);
* causal attention over the pool the KV write just filled: ``mvb_prefill_attention``, one CTA per
  (sequence, 16-token query tile, KV head) reading the tile's K/V prefix once for its 16 queries
  (head dim 128, up to 4 query heads per KV head); other shapes take the decode kernel with one
  query per token row over its first ``pos + 1`` keys;
* o_proj GEMM with the residual add in its epilogue, RMSNorm, gate_up GEMM with the SwiGLU epilogue,
  down GEMM with the residual add;
* the final RMSNorm and lm_head on each sequence's last row only, then the sampler.

Gemma models (``models/gemma3_model.py:270-283``) take the same pass with their own layer: the
embedding times its scale, (1 + w) norms, the o_proj and down outputs each post-normalised before
the residual add (``mvb_rmsnorm`` in place, then ``mvb_fused_add_rmsnorm`` into the next norm),
GeGLU on the stored gate_up product (``mvb_fused_mlp``), attention with the layer's soft-capping and
window (one query per token row, head dim 256), and the final logits soft-capped.

Sparse-MoE models (``models/qwen3_moe_model.py:39-66``, every layer sparse) replace the MLP with the
decode step's MoE kernels: the router GEMM over all rows, then per 256-row chunk (the routing
kernel's limit) routing + dispatch order, gather, the grouped gate/up (SwiGLU) and down GEMMs over
the active experts and the expert-ordered combine; the residual add is fused with the next layer's
input norm (``mvb_fused_add_rmsnorm``), as in the decode step.

Rows are processed in chunks of whole sequences so the activations stay within a fixed budget
next to the KV pool.
"""
from __future__ import annotations

from contextlib import contextmanager

import torch

from . import _native as N

_ATTN_ROWS = 4096   # query rows per attention launch at head dim 128 (the kernel's limit on sequences)
_MOE_ROWS = 256     # token rows per MoE routing / dispatch launch (mvb_moe_route's limit)


def split_chunks(lens: list[int], max_tokens: int) -> list[tuple[int, int]]:
    """Consecutive runs ``[i, j)`` of whole sequences of at most ``max_tokens`` tokens each, taken
    greedily in order; a prompt longer than the budget raises ``ValueError``."""
    out, i = [], 0
    while i < len(lens):
        j, n = i, 0
        while j < len(lens) and n + lens[j] <= max_tokens:
            n += lens[j]
            j += 1
        if j == i:
            raise ValueError(f"prompt of {lens[i]} tokens exceeds the prefill budget {max_tokens}")
        out.append((i, j))
        i = j
    return out


def pack_chunk_metadata(ids: list[list[int]], tables: list[list[int]], max_blocks: int,
                        scratch_block: int) -> tuple[torch.Tensor, tuple[int, int, int, int, int]]:
    """The host side of one chunk's metadata, one int32 buffer uploaded with one copy:

    ``token ids [T] | positions [T] | context lengths [T] | block table per row [T, max_blocks] |
    sequence start [S] | sequence length [S] | block table per sequence [S, max_blocks] |
    tile sequence [nt] | tile index [nt]``

    Row r is token i of sequence s (prompts packed in order): position i, context i + 1, its
    sequence's block table (unused entries the scratch block).  The attention tiles are the
    (sequence, 16-token query tile) pairs, the tiles with the longest prefixes first (stable
    within an index).  Returns the buffer and (T, S, nt, offset of the sequence part, offset of
    the tile part)."""
    lens = [len(p) for p in ids]
    T, S, mb = sum(lens), len(ids), max_blocks
    tiles = sorted(((s, qt) for s in range(S) for qt in range((lens[s] + 15) // 16)), key=lambda x: -x[1])
    nt = len(tiles)
    o_seq = 3 * T + T * mb
    o_tile = o_seq + 2 * S + S * mb
    host = torch.zeros(o_tile + 2 * nt, dtype=torch.int32)
    tok, pos, ctx = host[:T], host[T:2 * T], host[2 * T:3 * T]
    bt = host[3 * T:o_seq].view(T, mb)
    bt.fill_(scratch_block)
    seq_start, seq_len = host[o_seq:o_seq + S], host[o_seq + S:o_seq + 2 * S]
    seq_bt = host[o_seq + 2 * S:o_tile].view(S, mb)
    seq_bt.fill_(scratch_block)
    row = 0
    for k, (p, t) in enumerate(zip(ids, tables)):
        n = len(p)
        if len(t) > mb:
            raise ValueError(f"sequence needs {len(t)} blocks > max_blocks {mb}")
        tok[row:row + n] = torch.tensor(p, dtype=torch.int32)
        pos[row:row + n] = torch.arange(n, dtype=torch.int32)
        ctx[row:row + n] = torch.arange(1, n + 1, dtype=torch.int32)
        bt[row:row + n, :len(t)] = torch.tensor(t, dtype=torch.int32)
        seq_start[k], seq_len[k] = row, n
        seq_bt[k, :len(t)] = torch.tensor(t, dtype=torch.int32)
        row += n
    host[o_tile:o_tile + nt] = torch.tensor([x[0] for x in tiles], dtype=torch.int32)
    host[o_tile + nt:] = torch.tensor([x[1] for x in tiles], dtype=torch.int32)
    return host, (T, S, nt, o_seq, o_tile)


def _attention_rows(runner) -> int:
    """Query rows per launch of the decode kernel: it takes up to 4096 (row, head group) pairs at
    head dim 128, where one group holds all KV heads, and 1024 at head dim 256 (groups of 2 heads)."""
    if runner.D == 128:
        return _ATTN_ROWS
    groups = runner.Hkv // (2 if runner.Hkv % 2 == 0 else 1)
    return max(1, 1024 // groups)


class BatchedPrefill:
    """Prefill of dense (Qwen3 / Llama-family), Gemma and sparse-MoE models through a
    ``DecodeRunner``'s weights, tables and KV pool, on one GPU or on a tensor-parallel group.

    Tensor parallel (``engine.py:253-295`` with the decode step's Megatron split): each rank runs
    its column-parallel q|k|v (writing its own KV heads into its pool), its heads' attention and
    its gate/up slice; the row-parallel o_proj and down_proj outputs are summed over the ranks
    with an NCCL all-reduce in fp32 (a prefill chunk moves [tokens, hidden] per layer, bandwidth
    work that NCCL's ring / NVLS algorithms do well; the decode step's in-kernel exchanges are
    sized for 64 rows), then residual add + RMSNorm on every rank (Gemma: the post-norm of the
    summed output first); a sparse MoE block runs the rank's experts only and its combined
    partial is summed the same way; the vocab-parallel logits of the last tokens are
    all-gathered, so every rank samples the same first tokens."""

    def __init__(self, runner, max_tokens: int = 16384):
        self.r = runner
        self.tp = runner.tp
        self.max_tokens = max_tokens
        r, dev, bf = runner, runner.dev, torch.bfloat16
        T = max_tokens
        self.h = torch.zeros(T, r.H, dtype=bf, device=dev)           # residual stream
        self.xn = torch.zeros(T, r.H, dtype=bf, device=dev)
        self.qkv = torch.zeros(T, (r.Hq + 2 * r.Hkv) * r.D, dtype=bf, device=dev)
        self.q = torch.zeros(T, r.Hq, r.D, dtype=bf, device=dev)
        self.attn = torch.zeros(T, r.Hq * r.D, dtype=bf, device=dev)
        self.act = torch.zeros(0 if r.moe else T, r.I, dtype=bf, device=dev)
        if r.moe:   # routing / dispatch state of one 256-row chunk; the router logits of all rows
            C, E, K, i32 = _MOE_ROWS, r.E, r.K, torch.int32
            self.router_logits = torch.zeros(T, E, dtype=bf, device=dev)
            self.topk_ids = torch.zeros(C, K, dtype=i32, device=dev)
            self.topk_w = torch.zeros(C, K, dtype=torch.float32, device=dev)
            self.pair_row = torch.zeros(C, K, dtype=i32, device=dev)
            self.row_token = torch.zeros(C * K, dtype=i32, device=dev)
            self.expert_off = torch.zeros(E + 1, dtype=i32, device=dev)
            self.active = torch.zeros(E + 1, dtype=i32, device=dev)
            self.x_sorted = torch.zeros(C * K, r.H, dtype=bf, device=dev)
            self.h_sorted = torch.zeros(C * K, r.Im, dtype=bf, device=dev)
            self.y_sorted = torch.zeros(C * K, r.H, dtype=bf, device=dev)
            self.moe_out = torch.zeros(T, r.H, dtype=bf, device=dev)
        if r.gemma:   # the stored gate_up product (GeGLU is applied after it) and a post-norm buffer
            self.gu = torch.zeros(T, 2 * r.I, dtype=bf, device=dev)
            self.z = torch.zeros(T, r.H, dtype=bf, device=dev)
        if self.tp.enabled:   # a rank's row-parallel partial, and its fp32 copy for the all-reduce
            self.y = torch.zeros(T, r.H, dtype=bf, device=dev)
            self.y32 = torch.zeros(T, r.H, dtype=torch.float32, device=dev)
        self.gemm_ws = None
        self.timing: dict[str, list] | None = None   # kind -> [(start, end) CUDA events] when profiling
        self.attn_rows = _attention_rows(r)
        ws = N.lib().mvb_paged_attention_workspace_bytes(min(T, self.attn_rows), r.Hq, r.D, dev.index)
        self.attn_ws = torch.zeros(ws, dtype=torch.uint8, device=dev)

    def _mark(self, kind: str):
        """Start/stop CUDA-event pair around one launch when ``timing`` is on (else a no-op)."""
        if self.timing is None:
            return None
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        ev[0].record()
        self.timing.setdefault(kind, []).append(ev)
        return ev[1]

    @contextmanager
    def _timed(self, kind: str):
        """CUDA-event pair around the launches in the block when ``timing`` is on."""
        end = self._mark(kind)
        yield
        if end is not None:
            end.record()

    def _gemm(self, y, x, w, epilogue=N.EPI_STORE, aux=None):
        end = self._mark("gemm")
        self._gemm_launch(y, x, w, epilogue, aux)
        if end is not None:
            end.record()

    def _gemm_launch(self, y, x, w, epilogue, aux):
        lib, dev = N.lib(), self.r.dev
        need = lib.mvb_gemm_workspace_bytes(x.shape[0], w.shape[0], w.shape[1], dev.index)
        if self.gemm_ws is None or self.gemm_ws.numel() < need:
            self.gemm_ws = torch.zeros(need + (1 << 20), dtype=torch.uint8, device=dev)
        N.check(lib.mvb_gemm_bf16(y.data_ptr(), y.stride(0), x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0),
                                  x.shape[0], w.shape[0], w.shape[1], epilogue, N.ptr(aux),
                                  0 if aux is None else aux.stride(0), self.gemm_ws.data_ptr(),
                                  self.gemm_ws.numel(), N.stream_handle(dev)), "gemm_bf16")

    def _all_reduce(self, y: torch.Tensor) -> None:
        """Sums the ranks' partials of a row-parallel product in fp32, then rounds to bf16 (the
        reference's linear-layer output dtype)."""
        if not self.tp.enabled or self.tp.tp_size == 1:
            return
        import torch.distributed as dist

        y32 = self.y32[:y.shape[0]]
        y32.copy_(y)
        with self._timed("all_reduce"):
            dist.all_reduce(y32)
        y.copy_(y32)

    def run(self, ids: list[list[int]], tables: list[list[int]]) -> torch.Tensor:
        """Prefills the sequences whose prompts are ``ids`` into the blocks ``tables`` (each holding
        at least ``len(prompt)`` tokens); returns the bf16 logits ``[n, V]`` of each last token."""
        out = [self._chunk(ids[i:j], tables[i:j]) for i, j in split_chunks([len(p) for p in ids], self.max_tokens)]
        return torch.cat(out)

    def _chunk(self, ids: list[list[int]], tables: list[list[int]]) -> torch.Tensor:
        r, lib = self.r, N.lib()
        dev, w, H, D, L = r.dev, r.w, r.H, r.D, r.L
        lens = [len(p) for p in ids]
        mb = r.max_blocks
        host, (T, S, nt, o_seq, o_tile) = pack_chunk_metadata(ids, tables, mb, r.kv.scratch_block)
        meta = host.to(dev, non_blocking=False)
        tok_d, pos_d, ctx_d = meta[:T], meta[T:2 * T], meta[2 * T:3 * T]
        bt_d = meta[3 * T:o_seq].view(T, mb)
        seq_start_d, seq_len_d = meta[o_seq:o_seq + S], meta[o_seq + S:o_seq + 2 * S]
        seq_bt_d = meta[o_seq + 2 * S:o_tile]
        tile_seq_d, tile_idx_d = meta[o_tile:o_tile + nt], meta[o_tile + nt:]
        tiled = D == 128 and (r.Hq // r.Hkv) in (1, 2, 4) and not r.softcap and not any(r.windows)
        st, eps, bf = N.stream_handle(dev), r.eps, N.BF16
        h, xn, qkv, q, attn, act = (t_[:T] for t_ in (self.h, self.xn, self.qkv, self.q, self.attn, self.act))
        kvc = r.kv.kv_cache
        with self._timed("embedding"):
            N.check(lib.mvb_embedding(h.data_ptr(), tok_d.data_ptr(), N.I32, w.embed.data_ptr(), T, H, r.V,
                                      r.embed_scale, bf, st), "embedding")
        g, moe, tpx = r.gemma, r.moe, self.tp.enabled
        for i in range(L):
            if not (g or moe or tpx) or i == 0:   # else the previous layer's add formed this layer's input norm
                with self._timed("norm"):
                    N.check(lib.mvb_rmsnorm(xn.data_ptr(), H, h.data_ptr(), H, w.ln1[i].data_ptr(), T, H, eps,
                                            r.plus_one, N.NORM_MODEL, bf, st), "rmsnorm")
            self._gemm(qkv, xn, w.wqkv[i])
            cos, sin = r.layer_tables[i]
            with self._timed("qk_rope_kv"):
                N.check(lib.mvb_qk_norm_rope_kv_write(
                    q.data_ptr(), kvc.data_ptr(), qkv.data_ptr(), qkv.stride(0),
                    w.qn[i].data_ptr() if w.qk_norm else None, w.kn[i].data_ptr() if w.qk_norm else None,
                    cos.data_ptr(), sin.data_ptr(), cos.shape[0], pos_d.data_ptr(), bt_d.data_ptr(), mb, T, r.Hq,
                    r.Hkv, D, L, i, r.P, r.kv.block_size, eps, r.plus_one, st), "qk_norm_rope_kv_write")
            end = self._mark("attention")
            if tiled:
                N.check(lib.mvb_prefill_attention(
                    attn.data_ptr(), attn.stride(0), q.data_ptr(), r.Hq * D, kvc.data_ptr(), seq_bt_d.data_ptr(), mb,
                    seq_start_d.data_ptr(), seq_len_d.data_ptr(), tile_seq_d.data_ptr(), tile_idx_d.data_ptr(), nt,
                    r.Hq, r.Hkv, D, L, i, r.P, r.kv.block_size, r.scale, st), "prefill_attention")
            for a0 in range(0, 0 if tiled else T, self.attn_rows):
                n = min(self.attn_rows, T - a0)
                N.check(lib.mvb_paged_attention_decode_ex(
                    attn[a0:].data_ptr(), attn.stride(0), q[a0:].data_ptr(), r.Hq * D, kvc.data_ptr(),
                    bt_d[a0:].data_ptr(), mb, ctx_d[a0:].data_ptr(), n, r.Hq, r.Hkv, D, L, i, r.P,
                    r.kv.block_size, r.scale, r.softcap, r.windows[i], self.attn_ws.data_ptr(),
                    self.attn_ws.numel(), st), "paged_attention_decode")
            if end is not None:
                end.record()
            if g:
                self._gemma_mlp_block(i, T, h, xn, attn, act)
                continue
            if tpx:   # row-parallel o_proj / down_proj: this rank's partials, summed over the ranks
                y = self.y[:T]
                self._gemm(y, attn, w.wo[i])
                self._all_reduce(y)
                with self._timed("norm"):
                    N.check(lib.mvb_fused_add_rmsnorm(xn.data_ptr(), h.data_ptr(), y.data_ptr(), w.ln2[i].data_ptr(),
                                                      T, H, eps, r.plus_one, N.NORM_MODEL, bf, st), "fused_add_rmsnorm")
                if moe:   # this rank's experts, their combined partial summed over the ranks
                    self._moe_block(i, T, xn, y)
                    self._all_reduce(y)
                    nw = w.ln1[i + 1] if i + 1 < L else w.final_norm
                    with self._timed("norm"):
                        N.check(lib.mvb_fused_add_rmsnorm(xn.data_ptr(), h.data_ptr(), y.data_ptr(), nw.data_ptr(), T,
                                                          H, eps, r.plus_one, N.NORM_MODEL, bf, st),
                                "fused_add_rmsnorm")
                    continue
                self._gemm(act, xn, w.wgu[i], N.EPI_SWIGLU)
                self._gemm(y, act, w.wdown[i])
                self._all_reduce(y)
                nw = w.ln1[i + 1] if i + 1 < L else w.final_norm
                with self._timed("norm"):
                    N.check(lib.mvb_fused_add_rmsnorm(xn.data_ptr(), h.data_ptr(), y.data_ptr(), nw.data_ptr(), T, H,
                                                      eps, r.plus_one, N.NORM_MODEL, bf, st), "fused_add_rmsnorm")
                continue
            self._gemm(h, attn, w.wo[i], N.EPI_RESADD, aux=h)          # h = h + o_proj(attn)
            with self._timed("norm"):
                N.check(lib.mvb_rmsnorm(xn.data_ptr(), H, h.data_ptr(), H, w.ln2[i].data_ptr(), T, H, eps,
                                        r.plus_one, N.NORM_MODEL, bf, st), "rmsnorm")
            if moe:   # h = h + moe(xn), xn = the next layer's input norm (the final norm after the last)
                out = self.moe_out[:T]
                self._moe_block(i, T, xn, out)
                nw = w.ln1[i + 1] if i + 1 < L else w.final_norm
                with self._timed("norm"):
                    N.check(lib.mvb_fused_add_rmsnorm(xn.data_ptr(), h.data_ptr(), out.data_ptr(), nw.data_ptr(), T,
                                                      H, eps, r.plus_one, N.NORM_MODEL, bf, st), "fused_add_rmsnorm")
                continue
            self._gemm(act, xn, w.wgu[i], N.EPI_SWIGLU)
            self._gemm(h, act, w.wdown[i], N.EPI_RESADD, aux=h)        # h = h + down(swiglu)
        last = torch.tensor([sum(lens[:k + 1]) - 1 for k in range(len(lens))], device=dev)
        if g or moe or tpx:   # xn already holds the final norm of every row
            xl = xn.index_select(0, last).contiguous()
        else:
            hl = h.index_select(0, last).contiguous()
            xl = torch.empty_like(hl)
            N.check(lib.mvb_rmsnorm(xl.data_ptr(), H, hl.data_ptr(), H, w.final_norm.data_ptr(), len(lens), H, eps,
                                    r.plus_one, N.NORM_MODEL, bf, st), "rmsnorm")
        logits = torch.empty(len(lens), r.V, dtype=torch.bfloat16, device=dev)
        if tpx and self.tp.tp_size > 1:   # vocab-parallel lm_head: every rank's columns, gathered in rank order
            import torch.distributed as dist

            part = torch.empty(len(lens), r.Vl, dtype=torch.bfloat16, device=dev)
            self._gemm(part, xl, w.lm_head)
            parts = [torch.empty_like(part) for _ in range(self.tp.tp_size)]
            dist.all_gather(parts, part)
            torch.cat(parts, dim=1, out=logits)
        else:
            self._gemm(logits, xl, w.lm_head)
        if r.final_softcap:
            N.check(lib.mvb_softcap(logits.data_ptr(), logits.numel(), r.final_softcap, bf, st), "softcap")
        return logits

    def _moe_block(self, i, T, xn, out) -> None:
        """The sparse MoE block of layer i on ``xn`` into ``out`` (``qwen3_moe_model.py:39-65``): the
        router GEMM over all T rows, then per chunk of up to 256 rows the decode step's routing,
        gather, grouped SwiGLU and down GEMMs over the chunk's active experts, and combine."""
        r, lib, w = self.r, N.lib(), self.r.w
        H, E, K, st = r.H, r.E, r.K, N.stream_handle(r.dev)
        rl = self.router_logits[:T]
        self._gemm(rl, xn, w.router[i])
        end = self._mark("moe")
        for c0 in range(0, T, _MOE_ROWS):
            n = min(_MOE_ROWS, T - c0)
            N.check(lib.mvb_moe_route(rl[c0:].data_ptr(), n, E, K, r.norm_topk, self.topk_ids.data_ptr(),
                                      self.topk_w.data_ptr(), self.pair_row.data_ptr(), self.row_token.data_ptr(),
                                      self.expert_off.data_ptr(), self.active.data_ptr(), st), "moe_route")
            N.check(lib.mvb_moe_gather(self.x_sorted.data_ptr(), xn[c0:].data_ptr(), H, self.row_token.data_ptr(),
                                       n * K, st), "moe_gather")
            e0, ne = r.e_first, r.e_local   # all experts on one GPU; this rank's under tensor parallelism
            N.check(lib.mvb_moe_gemm_bf16_experts(self.h_sorted.data_ptr(), r.Im, self.x_sorted.data_ptr(), H,
                                                  w.egu[i].data_ptr(), 2 * r.Im, H, E, e0, ne, n * K, n,
                                                  N.EPI_SWIGLU, self.expert_off.data_ptr(), self.active.data_ptr(),
                                                  st), "moe_gemm gate_up")
            N.check(lib.mvb_moe_gemm_bf16_experts(self.y_sorted.data_ptr(), H, self.h_sorted.data_ptr(), r.Im,
                                                  w.edown[i].data_ptr(), H, r.Im, E, e0, ne, n * K, n, N.EPI_STORE,
                                                  self.expert_off.data_ptr(), self.active.data_ptr(), st),
                    "moe_gemm down")
            N.check(lib.mvb_moe_combine_experts(out[c0:].data_ptr(), self.y_sorted.data_ptr(), self.topk_w.data_ptr(),
                                                self.topk_ids.data_ptr(), self.pair_row.data_ptr(), n, K, H, e0, ne,
                                                st), "moe_combine")
        if end is not None:
            end.record()

    def _gemma_mlp_block(self, i, T, h, xn, attn, act) -> None:
        """The rest of Gemma layer i after attention (gemma3_model.py:274-281): o_proj, its post-norm,
        residual add + pre-feed-forward norm, gate_up, GeGLU, down, its post-norm, residual add + the
        next layer's input norm (the final norm after the last layer)."""
        r, lib, w = self.r, N.lib(), self.r.w
        H, eps, bf, st = r.H, r.eps, N.BF16, N.stream_handle(r.dev)
        z, gu = self.z[:T], self.gu[:T]

        def post_add_norm(post_w, next_w):
            # z = RMSNorm(z; post_w) in place, then h += z, xn = RMSNorm(h; next_w)
            N.check(lib.mvb_rmsnorm(z.data_ptr(), H, z.data_ptr(), H, post_w.data_ptr(), T, H, eps, r.plus_one,
                                    N.NORM_MODEL, bf, st), "rmsnorm")
            N.check(lib.mvb_fused_add_rmsnorm(xn.data_ptr(), h.data_ptr(), z.data_ptr(), next_w.data_ptr(), T, H,
                                              eps, r.plus_one, N.NORM_MODEL, bf, st), "fused_add_rmsnorm")

        self._gemm(z, attn, w.wo[i])
        self._all_reduce(z)   # tensor parallel: the ranks' row-parallel partials (no-op on one GPU)
        post_add_norm(w.ln2[i], w.pre_ff[i])
        self._gemm(gu, xn, w.wgu[i])
        N.check(lib.mvb_fused_mlp(act.data_ptr(), gu.data_ptr(), T, r.I, r.act, bf, st), "fused_mlp")
        self._gemm(z, act, w.wdown[i])
        self._all_reduce(z)
        post_add_norm(w.post_ff[i], w.ln1[i + 1] if i + 1 < r.L else w.final_norm)
