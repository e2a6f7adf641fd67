"""Oracle restatement of the reference's decoder math (pure PyTorch, CPU).

Follows ``mini_vllm/models/model.py`` (the PyTorch-path model the reference runs
with ``MINI_VLLM_BACKEND=pytorch``) operation by operation, in the same dtype and
with the same intermediate roundings, so that the CUDA path can be compared with
it at bf16 tolerance and its KV-cache indexing bit for bit.  Gemma models follow
``mini_vllm/models/gemma3_model.py`` (sandwich (1 + w) norms, GeGLU, sqrt(hidden)
embedding scale, per-layer RoPE theta); the Gemma-2 features the reference does not
have (attention / final logit soft-capping, sliding-window layers) are restated from
Gemma-2's published definition and pinned to the transformers implementation
(``tests/golden/make_gemma2_golden.py``).

Weights come in as an HF-keyed state dict; ``gate_proj``/``up_proj`` stay separate
as in ``model.py:106-117``.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def is_gemma(cfg: dict) -> bool:
    """``loader.py:70``: model_type gemma3_text selects ``Gemma3ForCausalLM``; Gemma-2 shares its
    layer structure (sandwich norms, GeGLU, embedding scale)."""
    return cfg.get("model_type") in ("gemma2", "gemma3_text")


def layer_rope_theta(cfg: dict, i: int) -> float:
    """``gemma3_model.py:307-320``: layer i uses the global ``rope_theta`` when
    ``i % pattern == pattern - 1`` and ``rope_local_base_freq`` otherwise; other models one theta."""
    if cfg.get("model_type") == "gemma3_text":
        pattern = cfg.get("sliding_window_pattern", 6)
        return cfg.get("rope_theta", 1000000.0) if i % pattern == pattern - 1 else cfg.get("rope_local_base_freq",
                                                                                            10000.0)
    return cfg.get("rope_theta", 10000.0)


def layer_window(cfg: dict, i: int) -> int:
    """Gemma-2: even layers attend through a ``sliding_window``, odd layers globally (the
    reference's Gemma 3 applies no window)."""
    if cfg.get("model_type") == "gemma2" and cfg.get("sliding_window"):
        return int(cfg["sliding_window"]) if i % 2 == 0 else 0
    return 0


# ----------------------------------------------------------------- primitives
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, plus_one: bool = False) -> torch.Tensor:
    """RMSNorm as ``model.py:19-25``: variance in fp32, then ``(w * x_hat)`` cast back."""
    orig = x.dtype
    var = x.float().pow(2).mean(-1, keepdim=True)
    xh = x * torch.rsqrt(var + eps)
    if plus_one:
        return (xh * (1.0 + w.float())).to(orig)
    return (w * xh).to(orig)


def ops_rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """The ops-API fallback ``ops/rmsnorm.py:12-20``: ``(w * x)`` rounds to the input dtype first."""
    w = w if w.dtype == x.dtype else w.to(x.dtype)
    var = x.float().pow(2).mean(-1, keepdim=True)
    return (w * x * torch.rsqrt(var + eps)).to(x.dtype)


def ops_rmsnorm_plus_one(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """``ops/rmsnorm.py:23-31``."""
    w = w if w.dtype == x.dtype else w.to(x.dtype)
    var = x.float().pow(2).mean(-1, keepdim=True)
    return ((1.0 + w.float()) * (x * torch.rsqrt(var + eps))).to(x.dtype)


def ops_fused_add_rmsnorm(residual, x, w, eps, plus_one=False):
    """``ops/rmsnorm.py:34-53``: returns ``(out, residual + x)``.

    The plus-one variant associates as ``((1 + w) * r) * rsqrt`` (``:51``), unlike
    the unfused ``rmsnorm_plus_one``.
    """
    r = residual + x
    if not plus_one:
        return ops_rmsnorm(r, w, eps), r
    w = w if w.dtype == x.dtype else w.to(x.dtype)
    var = r.float().pow(2).mean(-1, keepdim=True)
    return ((1.0 + w.float()) * r * torch.rsqrt(var + eps)).to(x.dtype), r


def inv_freq(head_dim: int, theta: float) -> torch.Tensor:
    """``model.py:31``: fp32 inverse frequencies (no rope_scaling for Qwen3/Llama-3 cfgs here)."""
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))


def rope_tables(head_dim: int, theta: float, length: int, dtype: torch.dtype,
                device: str | torch.device = "cpu") -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin cache as ``RotaryEmbedding.forward`` builds it (``model.py:74-81``).

    After ``model.to(dtype)`` (``loader.py:297``) the ``inv_freq`` buffer is in the
    model dtype, and the position ramp is ``arange(..., dtype=inv_freq.dtype)``:
    in bf16 the positions themselves are rounded (2049 -> 2048).  The table rows
    depend only on the position, not on the grown cache length.
    """
    f = inv_freq(head_dim, theta).to(dtype).to(device)
    t = torch.arange(length, device=device, dtype=f.dtype)
    freqs = torch.outer(t, f)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos(), emb.sin()


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """``model.py:94-97``."""
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """``model.py:100-103``: ``x*cos + rotate_half(x)*sin`` in the tensors' dtype."""
    return (x * cos) + (rotate_half(x) * sin)


# ----------------------------------------------------------------------- model
def moe_route(logits: torch.Tensor, top_k: int, norm_topk: bool = True):
    """``qwen3_moe_model.py:45-53``: softmax over the expert logits, top-k, optional
    renormalisation.  The reference's GPU decode runs under CUDA autocast, where softmax computes
    and returns fp32 from the bf16 logits; that is the semantics stated here for every dtype.
    Ties among equal probabilities go to the lower expert index."""
    probs = F.softmax(logits.float(), dim=-1)
    order = torch.sort(probs, dim=-1, descending=True, stable=True)   # equal values: ascending index
    topw, topi = order.values[:, :top_k], order.indices[:, :top_k]
    if norm_topk:
        topw = topw / topw.sum(dim=-1, keepdim=True)
    return topw, topi


def moe_combine(outs: torch.Tensor, topw: torch.Tensor, topi: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """``qwen3_moe_model.py:55-63`` for one token per row: ``outs[b, k]`` is expert ``topi[b, k]``'s
    output for row b; the weighted outputs are added into zeros of ``dtype`` in ascending expert
    order, each addition rounded to ``dtype``."""
    B, K, H = outs.shape
    final = torch.zeros(B, H, dtype=dtype)
    for b in range(B):
        for k in sorted(range(K), key=lambda j: int(topi[b, j])):
            # the reference's weights are an [n, 1] fp32 tensor: the product and the sum are fp32
            final[b] = (final[b].float() + topw[b, k].float() * outs[b, k].float()).to(dtype)
    return final


class OracleDecoder:
    """The reference's ``ForCausalLM`` forward (``model.py:412-424``) over a paged KV pool.

    ``kv_pool`` has the reference layout ``[L, 2, num_blocks, block_size, n_kv, head_dim]``
    (``kv_cache.py:24-29``).
    """

    def __init__(self, cfg: dict, state_dict: dict[str, torch.Tensor], dtype: torch.dtype,
                 device: str | torch.device = "cpu"):
        self.cfg = cfg
        self.dtype = dtype
        self.device = torch.device(device)
        self.L = cfg["num_hidden_layers"]
        self.H = cfg["hidden_size"]
        self.nq = cfg["num_attention_heads"]
        self.nkv = cfg.get("num_key_value_heads", self.nq)
        self.hd = cfg.get("head_dim", self.H // self.nq)
        self.eps = cfg.get("rms_norm_eps", 1e-6)
        self.theta = cfg.get("rope_theta", 10000.0)
        self.qk_norm = cfg.get("_qk_norm", False)
        self.plus_one = cfg.get("_rms_norm_plus_one", False)
        self.scale = cfg.get("query_pre_attn_scalar") or self.hd    # model.py:139
        act = cfg.get("hidden_act", "silu")
        self.act = {"silu": F.silu, "gelu": F.gelu, "gelu_new": lambda t: F.gelu(t, approximate="tanh"),
                    "relu": F.relu}[act]                                  # model.py:85-90
        self.w = {k: v.to(device=self.device, dtype=dtype) for k, v in state_dict.items()}
        if "lm_head.weight" not in self.w:                                # tied (model.py:417-418)
            self.w["lm_head.weight"] = self.w["model.embed_tokens.weight"]
        self.gemma = is_gemma(cfg)
        if self.gemma:
            self.plus_one = True
        self.softcap = float(cfg.get("attn_logit_softcapping") or 0.0)
        self.final_softcap = float(cfg.get("final_logit_softcapping") or 0.0)
        self.thetas = [layer_rope_theta(cfg, i) for i in range(self.L)]
        self.windows = [layer_window(cfg, i) for i in range(self.L)]
        self._tables: dict[float, tuple[torch.Tensor, torch.Tensor, int]] = {}
        # Gemma-2 soft-capped attention: "fp32" computes scores, softmax and p.v in fp32 and rounds
        # once; "eager" rounds as transformers' eager attention does in the model dtype (scores and
        # each soft-capping op in the dtype, fp32 softmax rounded to the dtype, p.v in the dtype).
        # Both are executions of the same definition; their spread measures its rounding noise.
        self.capped_rounding = "fp32"

    # model.py:60-81 (gemma3_model.py:60-81, one cache per theta) -- grow like the reference:
    # max(seq_len, 2*cache_len, 256)
    def rope(self, positions: torch.Tensor, theta: float | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        theta = self.theta if theta is None else theta
        seq_len = int(positions.max().item()) + 1
        cos, sin, n = self._tables.get(theta, (None, None, 0))
        if cos is None or n < seq_len:
            grow_to = max(seq_len, n * 2, 256)
            cos, sin = rope_tables(self.hd, theta, grow_to, self.dtype, self.device)
            self._tables[theta] = (cos, sin, grow_to)
        return cos[:seq_len], sin[:seq_len]

    # model.py:226-243
    @staticmethod
    def write_kv(kv_pool, k, v, block_tables, slot_idx, layer):
        bs = kv_pool.shape[3]
        is_batch = isinstance(block_tables[0], list)
        for i in range(k.shape[2]):
            if is_batch:
                for b in range(k.shape[0]):
                    pos = slot_idx[b] + i
                    blk = block_tables[b][pos // bs]
                    kv_pool[layer, 0, blk, pos % bs] = k[b, :, i]
                    kv_pool[layer, 1, blk, pos % bs] = v[b, :, i]
            else:
                pos = slot_idx + i
                blk = block_tables[pos // bs]
                kv_pool[layer, 0, blk, pos % bs] = k[0, :, i]
                kv_pool[layer, 1, blk, pos % bs] = v[0, :, i]

    # model.py:245-279
    @staticmethod
    def read_kv_batch(kv_pool, block_tables, layer, num_cached):
        max_cached = max(n + 1 for n in num_cached)
        ks, vs = [], []
        for b, bt in enumerate(block_tables):
            k = torch.cat([kv_pool[layer, 0, blk] for blk in bt], 0)[: num_cached[b] + 1]
            v = torch.cat([kv_pool[layer, 1, blk] for blk in bt], 0)[: num_cached[b] + 1]
            if k.shape[0] < max_cached:
                pad = torch.zeros(max_cached - k.shape[0], *k.shape[1:], dtype=k.dtype, device=k.device)
                k, v = torch.cat([k, pad]), torch.cat([v, pad])
            ks.append(k)
            vs.append(v)
        return torch.stack(ks).transpose(1, 2), torch.stack(vs).transpose(1, 2)

    def attention(self, i, x, cos, sin, kv_pool, block_tables, slot_idx, use_cache, num_cached, attn_mask):
        """``Attention.forward`` (``model.py:154-224``)."""
        w, p = self.w, f"model.layers.{i}.self_attn."
        B, S, _ = x.shape
        q = F.linear(x, w[p + "q_proj.weight"], w.get(p + "q_proj.bias")).view(B, S, self.nq, self.hd)
        k = F.linear(x, w[p + "k_proj.weight"], w.get(p + "k_proj.bias")).view(B, S, self.nkv, self.hd)
        v = F.linear(x, w[p + "v_proj.weight"], w.get(p + "v_proj.bias")).view(B, S, self.nkv, self.hd)
        v = v.transpose(1, 2)
        if self.qk_norm:   # Gemma: the (1 + w) form (gemma3_model.py:135-136, :159-160)
            q = rms_norm(q, w[p + "q_norm.weight"], self.eps, self.gemma)
            k = rms_norm(k, w[p + "k_norm.weight"], self.eps, self.gemma)
        q, k = q.transpose(1, 2), k.transpose(1, 2)
        q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
        if kv_pool is not None and block_tables is not None and slot_idx is not None:
            self.write_kv(kv_pool, k, v, block_tables, slot_idx, i)
            if use_cache:
                k, v = self.read_kv_batch(kv_pool, block_tables, i, num_cached)
        g = self.nq // self.nkv
        if g > 1:
            k = k.repeat_interleave(g, dim=1)
            v = v.repeat_interleave(g, dim=1)
        sc = 1.0 / math.sqrt(self.scale)
        if self.softcap or self.windows[i]:
            o = self.capped_attention(q, k, v, sc, self.windows[i], num_cached if use_cache else None)
            o = o.transpose(1, 2).contiguous().view(B, S, -1)
            return F.linear(o, w[p + "o_proj.weight"], w.get(p + "o_proj.bias"))
        if attn_mask is not None:
            o = F.scaled_dot_product_attention(q, k, v, scale=sc, attn_mask=attn_mask)
        elif use_cache:
            o = F.scaled_dot_product_attention(q, k, v, scale=sc)
        else:
            o = F.scaled_dot_product_attention(q, k, v, scale=sc, is_causal=True)
        o = o.transpose(1, 2).contiguous().view(B, S, -1)
        return F.linear(o, w[p + "o_proj.weight"], w.get(p + "o_proj.bias"))

    def capped_attention(self, q, k, v, scale, window, num_cached):
        """Gemma-2 attention: scores ``q k^T * scale`` soft-capped (``cap * tanh(s / cap)``) before
        the mask, then softmax and ``p v``; computed in fp32 and rounded once to the model dtype.
        The mask keeps key j for query position t when j <= t and, in a sliding-window layer,
        t - j < window.  Decode (``num_cached`` given): query b sits at position num_cached[b]
        with keys 0..num_cached[b] valid; prefill: query i at position i (causal)."""
        B, Hq, S, D = q.shape
        T = k.shape[2]
        eager = self.capped_rounding == "eager"
        if eager:
            s = torch.matmul(q, k.transpose(-1, -2)) * scale
            if self.softcap:
                s = torch.tanh(s / self.softcap) * self.softcap
        else:   # fp32 throughout: autocast would otherwise run both products in the model dtype
            with torch.autocast(device_type=q.device.type, enabled=False):
                s = torch.matmul(q.float(), k.float().transpose(-1, -2)) * scale
            if self.softcap:
                s = self.softcap * torch.tanh(s / self.softcap)
        j = torch.arange(T, device=s.device)
        if num_cached is not None:
            t = torch.tensor(num_cached, device=s.device).view(B, 1, 1, 1)     # query positions
        else:
            t = torch.arange(S, device=s.device).view(1, 1, S, 1)
        keep = j.view(1, 1, 1, T) <= t
        if window:
            keep = keep & (t - j.view(1, 1, 1, T) < window)
        s = s.masked_fill(~keep, float("-inf"))
        if eager:
            p = torch.softmax(s, dim=-1, dtype=torch.float32).to(q.dtype)
            return torch.matmul(p, v)
        with torch.autocast(device_type=q.device.type, enabled=False):
            p = torch.softmax(s, dim=-1)
            return torch.matmul(p, v.float()).to(q.dtype)

    def mlp(self, i, x):
        """``MLP.forward`` (``model.py:116-117``): ``down(act(gate(x)) * up(x))``."""
        if self.cfg.get("num_experts"):
            return self.moe(i, x)
        w, p = self.w, f"model.layers.{i}.mlp."
        return F.linear(self.act(F.linear(x, w[p + "gate_proj.weight"])) * F.linear(x, w[p + "up_proj.weight"]),
                        w[p + "down_proj.weight"])

    def route(self, i, flat):
        """Router of ``Qwen3MoeSparseMoe.forward`` (``qwen3_moe_model.py:45-53``) for layer i."""
        logits = F.linear(flat, self.w[f"model.layers.{i}.mlp.gate.weight"])
        return moe_route(logits, self.cfg["num_experts_per_tok"], self.cfg.get("norm_topk_prob", True))

    def moe(self, i, x):
        """``Qwen3MoeSparseMoe.forward`` (``qwen3_moe_model.py:39-65``): each expert's
        ``down(silu(gate(x)) * up(x))`` on its tokens; the weighted outputs are added into a zero
        tensor of the model dtype expert by expert in ascending index (``final += w * out``: the
        product in the routing weights' dtype, each addition rounded to the model dtype)."""
        w, p = self.w, f"model.layers.{i}.mlp."
        B, S, H = x.shape
        flat = x.reshape(-1, H)
        topw, topi = self.route(i, flat)
        final = torch.zeros_like(flat)
        for e in range(self.cfg["num_experts"]):
            mask = topi == e
            if not bool(mask.any()):
                continue
            tok = mask.any(dim=-1).nonzero(as_tuple=True)[0]
            q = f"{p}experts.{e}."
            xe = flat[tok]
            out = F.linear(F.silu(F.linear(xe, w[q + "gate_proj.weight"])) * F.linear(xe, w[q + "up_proj.weight"]),
                           w[q + "down_proj.weight"])
            for k in range(topi.shape[1]):
                km = mask[tok, k]
                if bool(km.any()):
                    rows = tok[km]
                    final[rows] = (final[rows] + topw[rows, k].unsqueeze(-1) * out[km]).to(final.dtype)
        return final.view(B, S, H)

    def forward(self, input_ids, positions, kv_pool=None, block_tables=None, slot_idx=None, use_cache=False,
                num_cached=None, attn_mask=None, return_hidden=False, last_only=False):
        """``ForCausalLM.forward`` -> logits ``[B, S, V]`` in the model dtype (``model.py:369-424``).

        ``last_only`` projects only the last position through the final norm and lm_head
        (rows are independent there; it saves the ``S x V`` prefill projection)."""
        w = self.w
        h = F.embedding(input_ids, w["model.embed_tokens.weight"])
        if self.gemma:   # gemma3_model.py:295-299, :330: times the sqrt(hidden) buffer, which
            # model.to(dtype) (loader.py:297) has cast to the model dtype
            h = h * torch.tensor(math.sqrt(self.H), dtype=torch.float32).to(self.dtype)
        tables = {}
        for theta in dict.fromkeys(self.thetas):
            cos, sin = self.rope(positions, theta)
            cos, sin = cos[positions], sin[positions]
            if cos.dim() == 3:
                cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
            else:
                cos, sin = cos.unsqueeze(0).unsqueeze(0), sin.unsqueeze(0).unsqueeze(0)
            tables[theta] = (cos, sin)
        if self.gemma:
            return self._forward_gemma(h, tables, kv_pool, block_tables, slot_idx, use_cache, num_cached, attn_mask,
                                       return_hidden, last_only)
        cos, sin = tables[self.theta]
        for i in range(self.L):
            p = f"model.layers.{i}."
            r = h
            h = rms_norm(h, w[p + "input_layernorm.weight"], self.eps, self.plus_one)
            h = self.attention(i, h, cos, sin, kv_pool, block_tables, slot_idx, use_cache, num_cached, attn_mask)
            h = r + h
            r = h
            h = rms_norm(h, w[p + "post_attention_layernorm.weight"], self.eps, self.plus_one)
            h = self.mlp(i, h)
            h = r + h
        if last_only:
            h = h[:, -1:]
        h = rms_norm(h, w["model.norm.weight"], self.eps, self.plus_one)
        logits = F.linear(h, w["lm_head.weight"])
        return (logits, h) if return_hidden else logits

    def _forward_gemma(self, h, tables, kv_pool, block_tables, slot_idx, use_cache, num_cached, attn_mask,
                       return_hidden, last_only):
        """``Gemma3DecoderLayer.forward`` (gemma3_model.py:270-283) for every layer, the final norm
        and lm_head (``:345-372``), then Gemma-2's final soft-capping ``cap * tanh(x / cap)`` as
        the three ops ``x / cap``, ``tanh``, ``* cap`` in the logits' dtype."""
        w = self.w
        for i in range(self.L):
            p = f"model.layers.{i}."
            cos, sin = tables[self.thetas[i]]
            r = h
            x = rms_norm(h, w[p + "input_layernorm.weight"], self.eps, True)
            x = self.attention(i, x, cos, sin, kv_pool, block_tables, slot_idx, use_cache, num_cached, attn_mask)
            x = rms_norm(x, w[p + "post_attention_layernorm.weight"], self.eps, True)
            h = r + x
            r = h
            x = rms_norm(h, w[p + "pre_feedforward_layernorm.weight"], self.eps, True)
            x = self.mlp(i, x)
            x = rms_norm(x, w[p + "post_feedforward_layernorm.weight"], self.eps, True)
            h = r + x
        if last_only:
            h = h[:, -1:]
        h = rms_norm(h, w["model.norm.weight"], self.eps, True)
        logits = F.linear(h, w["lm_head.weight"])
        if self.final_softcap:
            logits = torch.tanh(logits / self.final_softcap) * self.final_softcap
        return (logits, h) if return_hidden else logits
