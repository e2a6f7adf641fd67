"""Drop-ins for the reference's model classes (``mini_vllm/models/model_cuda.py``) on the sm_100a kernels.

``ForCausalLM`` and ``Attention`` keep the reference's constructor argument (the HF-style config
dict), parameter names (``load_state_dict`` takes the reference model's state dict) and
``forward`` signatures, so ``LLMEngine`` drives them unchanged with its own ``KVCacheManager``
tensor, block tables, slot indices and cached-token counts (``engine.py:253-360``):

* decode (``use_cache=True``, one token per sequence, ``block_tables`` a list per sequence): the
  decode step's kernels -- tcgen05 GEMMs, fused QK-norm/RoPE/KV write, TMA paged attention over the
  pool, fused residual-add + RMSNorm -- on the caller's pool.  The float ``attn_mask`` the reference
  builds (``engine.py:330-337``) only masks keys past each sequence's ``num_cached + 1``; the paged
  kernel reads exactly those keys, so the mask is not read.
* prefill (``use_cache=False``, one sequence, ``block_tables`` a flat list): the batched-prefill
  kernels over the prompt, writing every position's K/V into the pool.  The logits come back for
  the last position only, shape ``[1, 1, V]``, which is the row ``_run_prefill`` reads
  (``logits[:, -1, :]``, ``engine.py:286``).

The KV pool must be the reference's bf16 tensor ``[L, 2, num_blocks, 16, Hkv, D]``
(``kv_cache.py:24-29``) on the model's GPU; the model runs over the paged pool only (no
``kv_cache=None`` path).  Positions must equal the slot indices, as the reference's engine passes
them (``engine.py:316``, ``:326``).
"""
from __future__ import annotations

import math

import torch
from torch import nn

from . import _native as N
from .configs import head_dim as cfg_head_dim
from .runner import DecodeRunner, DecodeWeights


class _PoolView:
    """The attributes of a ``KVCacheManager`` the runner reads, over a caller-owned pool tensor
    that has no scratch block (every row of a call is a real sequence, so none is needed)."""

    def __init__(self, kv_cache: torch.Tensor, num_layers: int):
        self.kv_cache = kv_cache
        self.block_size = kv_cache.shape[3]
        self.num_heads = kv_cache.shape[4]
        self.head_dim = kv_cache.shape[5]
        self.num_layers = num_layers
        self.num_blocks = kv_cache.shape[2]
        self.scratch_block = kv_cache.shape[2]   # never indexed: unused table entries only


def _check_pool(kv_cache, cfg):
    if kv_cache is None:
        raise NotImplementedError("the B200 model runs over the paged KV pool: pass kv_cache")
    N.require_cuda(kv_cache)
    if kv_cache.dtype != torch.bfloat16 or kv_cache.dim() != 6 or kv_cache.shape[3] != 16:
        raise ValueError("kv_cache must be the bf16 pool [L, 2, num_blocks, 16, Hkv, D]")
    if kv_cache.shape[0] != cfg["num_hidden_layers"] or kv_cache.shape[5] != cfg_head_dim(cfg):
        raise ValueError("kv_cache geometry does not match the model")


def _pow2_at_least(n: int, lo: int) -> int:
    m = lo
    while m < n:
        m *= 2
    return m


class ForCausalLM(nn.Module):
    """``ForCausalLM`` (``model_cuda.py:404-415``; ``models/model.py:412-424``)."""

    def __init__(self, config: dict, device: str | torch.device = "cuda"):
        super().__init__()
        self.config = config
        self.device_ = torch.device(device)
        self.weights: DecodeWeights | None = None
        self._runners: dict = {}
        self._prefill = None

    @classmethod
    def from_reference(cls, model: nn.Module, device: str | torch.device = "cuda") -> "ForCausalLM":
        """Wraps the weights of a reference ``ForCausalLM`` (or any model with the same
        state-dict keys and a ``config`` attribute)."""
        m = cls(model.config, device)
        m.load_state_dict(model.state_dict())
        return m

    def load_state_dict(self, state_dict, strict: bool = True, assign: bool = False):
        """Takes the reference model's state dict (HF keys; ``gate_up_proj`` fused or
        ``gate_proj``/``up_proj`` separate; tied ``lm_head`` optional) into the kernels' layout."""
        sd = {k: v for k, v in state_dict.items() if k.endswith(".weight")}
        if strict and "model.embed_tokens.weight" not in sd:
            raise KeyError("state dict has no model.embed_tokens.weight")
        self.weights = DecodeWeights(self.config, sd, self.device_)
        self._runners.clear()
        self._prefill = None
        return nn.modules.module._IncompatibleKeys([], [])

    def _runner(self, kv_cache: torch.Tensor, batch: int, need_blocks: int) -> DecodeRunner:
        mb = _pow2_at_least(need_blocks, 16)
        key = (kv_cache.data_ptr(), tuple(kv_cache.shape), batch, mb)
        r = self._runners.get(key)
        if r is None:
            if len(self._runners) >= 8:    # a few shapes stay resident; the oldest goes
                self._runners.pop(next(iter(self._runners)))
            r = DecodeRunner(self.config, self.weights, _PoolView(kv_cache, self.config["num_hidden_layers"]),
                             batch, mb * 16, kv_cache.device)
            self._runners[key] = r
        return r

    def forward(self, input_ids, positions, kv_cache=None, block_tables=None, slot_idx=None, use_cache=False,
                num_cached_tokens=0, num_cached_tokens_list=None, attn_mask=None):
        """Logits in bf16: ``[B, 1, V]`` for a decode step, ``[1, 1, V]`` (the last prompt
        position) for a prefill."""
        if self.weights is None:
            raise RuntimeError("load_state_dict first")
        _check_pool(kv_cache, self.config)
        if block_tables is None or slot_idx is None:
            raise NotImplementedError("the B200 model runs over the paged KV pool: pass block_tables and slot_idx")
        with torch.cuda.device(kv_cache.device):
            if use_cache:
                return self._decode(input_ids, positions, kv_cache, block_tables, slot_idx, num_cached_tokens,
                                    num_cached_tokens_list)
            return self._prefill_one(input_ids, positions, kv_cache, block_tables, slot_idx)

    def _decode(self, input_ids, positions, kv_cache, block_tables, slot_idx, num_cached, num_cached_list):
        if not isinstance(block_tables[0], list):       # one sequence: model_cuda.py:145-155
            block_tables, slot_idx = [block_tables], [slot_idx]
            num_cached_list = [num_cached]
        B = len(block_tables)
        if input_ids.shape[0] != B or input_ids.numel() != B:
            raise ValueError("decode takes one token per sequence")
        pos = [int(p) for p in positions.reshape(-1).tolist()]
        slots = [int(s) for s in slot_idx]
        if pos != slots:
            raise ValueError("positions must equal slot_idx (engine.py:316, :326)")
        ctx = [int(n) + 1 for n in (num_cached_list if num_cached_list is not None else slots)]
        r = self._runner(kv_cache, B, max(len(t) for t in block_tables))
        r.set_metadata([int(t) for t in input_ids.reshape(-1).tolist()], pos, block_tables, 0, ctx)
        r.upload_metadata()
        r.forward()
        return r.logits[:B].clone().view(B, 1, -1)

    def _prefill_one(self, input_ids, positions, kv_cache, block_tables, slot_idx):
        from .prefill import BatchedPrefill

        if isinstance(block_tables[0], list) or input_ids.shape[0] != 1:
            raise ValueError("prefill takes one sequence (engine.py:253-286)")
        if int(slot_idx) != 0 or int(positions.reshape(-1)[0]) != 0:
            raise ValueError("prefill starts at position 0")
        ids = [int(t) for t in input_ids.reshape(-1).tolist()]
        r = self._runner(kv_cache, 1, len(block_tables))
        budget = _pow2_at_least(len(ids), 256)
        if self._prefill is None or self._prefill.r is not r or self._prefill.max_tokens < budget:
            self._prefill = BatchedPrefill(r, budget)
        return self._prefill.run([ids], [list(block_tables)]).view(1, 1, -1)


class Attention(nn.Module):
    """``Attention`` (``model_cuda.py:76-177``): q/k/v projections, optional per-head QK-norm,
    RoPE with the given cos/sin rows, the paged KV write, attention and o_proj -- one layer on the
    kernels.  Parameters have the reference's names (``q_proj``, ``k_proj``, ``v_proj``, ``o_proj``,
    ``q_norm``, ``k_norm``)."""

    def __init__(self, hidden_size: int, num_heads: int, num_kv_heads: int, head_dim: int,
                 attention_bias: bool = False, o_proj_bias: bool = False, qk_norm: bool = False,
                 rms_norm_eps: float = 1e-6, query_pre_attn_scalar: float | None = None):
        super().__init__()
        if attention_bias or o_proj_bias:
            raise NotImplementedError("projection biases are not on the B200 path")
        self.num_heads, self.num_kv_heads, self.head_dim = num_heads, num_kv_heads, head_dim
        self.q_proj = nn.Linear(hidden_size, num_heads * head_dim, bias=False)
        self.k_proj = nn.Linear(hidden_size, num_kv_heads * head_dim, bias=False)
        self.v_proj = nn.Linear(hidden_size, num_kv_heads * head_dim, bias=False)
        self.o_proj = nn.Linear(num_heads * head_dim, hidden_size, bias=False)
        self.q_norm = _NormWeight(head_dim) if qk_norm else None
        self.k_norm = _NormWeight(head_dim) if qk_norm else None
        self.eps = rms_norm_eps
        self.scale = 1.0 / math.sqrt(query_pre_attn_scalar or head_dim)
        self._wqkv = None

    def _fused_qkv(self) -> torch.Tensor:
        ws = (self.q_proj.weight, self.k_proj.weight, self.v_proj.weight)
        key = tuple((w.data_ptr(), w._version) for w in ws)
        if self._wqkv is None or self._wqkv[0] != key:
            self._wqkv = (key, torch.cat([w.detach().to(torch.bfloat16) for w in ws], 0).contiguous())
        return self._wqkv[1]

    def forward(self, hidden_states, position_cos, position_sin, kv_cache=None, block_tables=None, slot_idx=None,
                layer_idx: int = 0, use_cache: bool = False, num_cached_tokens: int = 0,
                num_cached_tokens_list=None, attn_mask=None):
        """``model_cuda.py:108-177``.  Decode: ``hidden_states`` ``[B, 1, H]``, ``block_tables`` a list
        per sequence, K/V read back for ``num_cached + 1`` tokens.  Prefill: one sequence
        ``[1, S, H]`` at ``slot_idx`` 0, causal attention over its S positions."""
        if kv_cache is None or block_tables is None or slot_idx is None:
            raise NotImplementedError("the B200 attention runs over the paged KV pool")
        N.require_cuda(hidden_states, kv_cache)
        lib, dev = N.lib(), hidden_states.device
        B, S, H = hidden_states.shape
        Hq, Hkv, D = self.num_heads, self.num_kv_heads, self.head_dim
        L, P, bs = kv_cache.shape[0], kv_cache.shape[2], kv_cache.shape[3]
        batched = isinstance(block_tables[0], list)
        tables = block_tables if batched else [list(block_tables)] * B
        starts = list(slot_idx) if batched else [int(slot_idx)] * B
        # one row per token: its sequence's table, its position (= slot, engine.py:316/326)
        pos = [starts[b] + i for b in range(B) for i in range(S)]
        rows = B * S
        mb = max(len(t) for t in tables)
        bt = torch.full((rows, mb), P, dtype=torch.int32)
        for b in range(B):
            bt[b * S:(b + 1) * S, :len(tables[b])] = torch.tensor(tables[b], dtype=torch.int32)
        bt = bt.to(dev)
        pos_d = torch.tensor(pos, dtype=torch.int32, device=dev)
        # cos/sin rows [B, 1, S, D] (or [1, 1, S, D]) scattered to a table indexed by position
        tlen = max(pos) + 1
        cos_t = torch.zeros(tlen, D, dtype=torch.bfloat16, device=dev)
        sin_t = torch.zeros(tlen, D, dtype=torch.bfloat16, device=dev)
        cos_rows = position_cos.to(torch.bfloat16).expand(B, 1, S, D).reshape(rows, D)
        sin_rows = position_sin.to(torch.bfloat16).expand(B, 1, S, D).reshape(rows, D)
        cos_t[pos_d.long()] = cos_rows
        sin_t[pos_d.long()] = sin_rows
        x = hidden_states.to(torch.bfloat16).reshape(rows, H).contiguous()
        wqkv = self._fused_qkv()
        qkv = torch.empty(rows, wqkv.shape[0], dtype=torch.bfloat16, device=dev)
        ws_bytes = lib.mvb_gemm_workspace_bytes(rows, max(wqkv.shape[0], H), max(H, Hq * D), dev.index)
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
        st = N.stream_handle(dev)
        N.check(lib.mvb_gemm_bf16(qkv.data_ptr(), qkv.stride(0), x.data_ptr(), H, wqkv.data_ptr(), H, rows,
                                  wqkv.shape[0], H, N.EPI_STORE, None, 0, ws.data_ptr(), ws_bytes, st), "gemm_bf16")
        q = torch.empty(rows, Hq, D, dtype=torch.bfloat16, device=dev)
        qn = self.q_norm.weight.detach().to(torch.bfloat16).contiguous() if self.q_norm is not None else None
        kn = self.k_norm.weight.detach().to(torch.bfloat16).contiguous() if self.k_norm is not None else None
        N.check(lib.mvb_qk_norm_rope_kv_write(q.data_ptr(), kv_cache.data_ptr(), qkv.data_ptr(), qkv.stride(0),
                                              N.ptr(qn), N.ptr(kn), cos_t.data_ptr(), sin_t.data_ptr(), tlen,
                                              pos_d.data_ptr(), bt.data_ptr(), mb, rows, Hq, Hkv, D, L, layer_idx, P,
                                              bs, self.eps, 0, st), "qk_norm_rope_kv_write")
        # attention: decode reads num_cached + 1 keys per sequence; prefill token i reads i + 1
        if use_cache and batched:
            ctx = [int(n) + 1 for n in (num_cached_tokens_list or starts)]
        elif use_cache:
            ctx = [int(num_cached_tokens) + 1 + i for i in range(S)] * B
        else:
            ctx = [p + 1 for p in pos]
        ctx_d = torch.tensor(ctx, dtype=torch.int32, device=dev)
        out = torch.empty(rows, Hq * D, dtype=torch.bfloat16, device=dev)
        # rows per launch: the kernel takes up to 4096 (row, head group) pairs at head dim 128 (one
        # group of all KV heads) and 1024 at head dim 256 (groups of two heads)
        chunk = 4096 if D == 128 else max(1, 1024 // (Hkv // 2 if Hkv % 2 == 0 else Hkv))
        aws_bytes = lib.mvb_paged_attention_workspace_bytes(min(rows, chunk), Hq, D, dev.index)
        aws = torch.zeros(aws_bytes, dtype=torch.uint8, device=dev)
        for a0 in range(0, rows, chunk):
            n = min(chunk, rows - a0)
            N.check(lib.mvb_paged_attention_decode_ex(
                out[a0:].data_ptr(), out.stride(0), q[a0:].data_ptr(), Hq * D, kv_cache.data_ptr(), bt[a0:].data_ptr(),
                mb, ctx_d[a0:].data_ptr(), n, Hq, Hkv, D, L, layer_idx, P, bs, self.scale, 0.0, 0, aws.data_ptr(),
                aws_bytes, st), "paged_attention_decode")
        wo = self.o_proj.weight.detach().to(torch.bfloat16).contiguous()
        y = torch.empty(rows, H, dtype=torch.bfloat16, device=dev)
        N.check(lib.mvb_gemm_bf16(y.data_ptr(), H, out.data_ptr(), Hq * D, wo.data_ptr(), Hq * D, rows, H, Hq * D,
                                  N.EPI_STORE, None, 0, ws.data_ptr(), ws_bytes, st), "gemm_bf16")
        return y.view(B, S, H)


class _NormWeight(nn.Module):
    """Holds an RMSNorm ``weight`` under the reference's parameter name (``RMSNorm.weight``)."""

    def __init__(self, dim: int):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
