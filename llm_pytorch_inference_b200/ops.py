"""Drop-in mirror of the reference's ``mini_vllm.ops`` API on the sm_100a kernels.

Same function / class names, argument meaning and return conventions as
``mini_vllm/ops/__init__.py:1-51``; every call goes through the C ABI of
``libmvb200.so``.  There is no CPU path: a CPU tensor raises ``RuntimeError``
(the reference would fall back to PyTorch, ``mini_vllm/ops/_utils.py:70-78``).

Numerics match the reference's PyTorch expressions (see the per-function notes);
the one deliberate difference is ``apply_rotary_pos_emb``, which broadcasts cos/sin
per sequence for K as well as Q (the reference's CUDA branch expands cos to Q's
shape and indexes it with K's rows, ``mini_vllm/ops/rope.py:59-70``).
"""
from __future__ import annotations

import threading

import torch
import torch.nn as nn
from torch.nn.parameter import Parameter

from . import _native as N

__all__ = [
    "rmsnorm", "rmsnorm_plus_one", "fused_add_rmsnorm", "fused_add_rmsnorm_plus_one", "RMSNorm",
    "precompute_freqs_cis", "rotate_half", "apply_rotary_pos_emb", "silu", "gelu", "swiglu", "geglu",
    "greedy_sample", "top_k_top_p_filter", "softmax_multinomial_sample", "embedding", "Embedding", "softmax",
    "FusedMLP", "linear", "paged_attention_decode", "qk_norm_rope_kv_write", "sample",
]


def _st(t: torch.Tensor) -> int:
    return N.stream_handle(t.device)


def _w(weight: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    w = weight if weight.dtype == like.dtype else weight.to(like.dtype)
    return w.contiguous()


# ----------------------------------------------------------------------- RMSNorm
def _rms(x, weight, eps, plus_one, semantics):
    N.require_cuda(x, weight)
    w = _w(weight, x)
    xc = x.contiguous()
    out = torch.empty_like(xc)
    H = xc.shape[-1]
    rows = xc.numel() // H if H else 0
    with torch.cuda.device(xc.device):
        N.check(N.lib().mvb_rmsnorm(out.data_ptr(), H, xc.data_ptr(), H, w.data_ptr(), rows, H, float(eps),
                                    int(plus_one), semantics, N.dtype_code(xc), _st(xc)), "rmsnorm")
    return out


def rmsnorm(input: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """``ops/rmsnorm.py:12-20``: ``(w * x * rsqrt(mean(x^2) + eps))`` in the input dtype."""
    return _rms(input, weight, eps, False, N.NORM_OPS)


def rmsnorm_plus_one(input: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """``ops/rmsnorm.py:23-31``: ``(1 + w) * x * rsqrt(...)``."""
    return _rms(input, weight, eps, True, N.NORM_OPS)


def _fused(residual, input, weight, eps, plus_one):
    N.require_cuda(residual, input, weight)
    if not residual.is_contiguous() or not input.is_contiguous():
        raise RuntimeError("fused_add_rmsnorm: residual and input must be contiguous")
    if residual.shape != input.shape or residual.dtype != input.dtype:
        raise RuntimeError("fused_add_rmsnorm: residual and input must match in shape and dtype")
    w = _w(weight, input)
    out = torch.empty_like(input)
    H = input.shape[-1]
    with torch.cuda.device(input.device):
        N.check(N.lib().mvb_fused_add_rmsnorm(out.data_ptr(), residual.data_ptr(), input.data_ptr(), w.data_ptr(),
                                              input.numel() // H, H, float(eps), int(plus_one), N.NORM_OPS,
                                              N.dtype_code(input), _st(input)), "fused_add_rmsnorm")
    return out, residual


def fused_add_rmsnorm(residual: torch.Tensor, input: torch.Tensor, weight: torch.Tensor,
                      eps: float = 1e-6) -> tuple[torch.Tensor, torch.Tensor]:
    """``ops/rmsnorm.py:34-42``: ``residual += input`` (in place), returns ``(norm(residual), residual)``."""
    return _fused(residual, input, weight, eps, False)


def fused_add_rmsnorm_plus_one(residual: torch.Tensor, input: torch.Tensor, weight: torch.Tensor,
                               eps: float = 1e-6) -> tuple[torch.Tensor, torch.Tensor]:
    """``ops/rmsnorm.py:45-53``."""
    return _fused(residual, input, weight, eps, True)


class RMSNorm(nn.Module):
    """``ops/rmsnorm.py:60-76``: weight init ones (or zeros for the (1+w) form)."""

    def __init__(self, hidden_size: int, eps: float = 1e-6, plus_one: bool = False):
        super().__init__()
        self.weight = Parameter(torch.zeros(hidden_size) if plus_one else torch.ones(hidden_size))
        self.eps = eps
        self.plus_one = plus_one

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return rmsnorm_plus_one(x, self.weight, self.eps) if self.plus_one else rmsnorm(x, self.weight, self.eps)


# --------------------------------------------------------------------------- RoPE
def precompute_freqs_cis(dim: int, seq_len: int, theta: float = 10000.0, device="cpu",
                         dtype: torch.dtype = torch.float32) -> tuple[torch.Tensor, torch.Tensor]:
    """Table construction as ``ops/rope.py:15-37`` (host-side set-up, not a decode kernel)."""
    freqs = 1.0 / (theta ** (torch.arange(0, dim, 2, device=device, dtype=dtype) / dim))
    t = torch.arange(seq_len, device=device, dtype=dtype)
    emb = torch.cat((torch.outer(t, freqs),) * 2, dim=-1)
    return emb.cos(), emb.sin()


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """``ops/rope.py:40-44`` (tensor utility)."""
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    D = x.shape[-1]
    c = cos.expand_as(x).reshape(-1, D).contiguous().to(x.dtype)
    s = sin.expand_as(x).reshape(-1, D).contiguous().to(x.dtype)
    xf = x.reshape(-1, D).contiguous()
    out = torch.empty_like(xf)
    with torch.cuda.device(x.device):
        N.check(N.lib().mvb_rotary_pos_emb(out.data_ptr(), xf.data_ptr(), c.data_ptr(), s.data_ptr(), xf.shape[0], D,
                                           N.dtype_code(xf), _st(xf)), "rotary_pos_emb")
    return out.reshape(x.shape)


def apply_rotary_pos_emb(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor,
                         sin: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """``ops/rope.py:47-77``: ``x*cos + rotate_half(x)*sin`` for q ``[B,Hq,S,D]`` and k ``[B,Hkv,S,D]``
    with cos/sin broadcastable ``[B,1,S,D]``; each product and the sum round to the dtype."""
    N.require_cuda(q, k, cos, sin)
    return _rope(q, cos, sin), _rope(k, cos, sin)


# -------------------------------------------------------------------- activations
def _act(x, act):
    N.require_cuda(x)
    xc = x.contiguous()
    out = torch.empty_like(xc)
    with torch.cuda.device(xc.device):
        N.check(N.lib().mvb_activation(out.data_ptr(), xc.data_ptr(), xc.numel(), act, N.dtype_code(xc), _st(xc)),
                "activation")
    return out


def _gated(g, u, act):
    N.require_cuda(g, u)
    if g.shape != u.shape:
        raise RuntimeError("gate and up must have the same shape")
    gc, uc = g.contiguous(), u.contiguous().to(g.dtype)
    out = torch.empty_like(gc)
    with torch.cuda.device(gc.device):
        N.check(N.lib().mvb_gated_activation(out.data_ptr(), gc.data_ptr(), uc.data_ptr(), gc.numel(), act,
                                             N.dtype_code(gc), _st(gc)), "gated_activation")
    return out


def silu(input: torch.Tensor) -> torch.Tensor:
    """``ops/activation.py:10-19``."""
    return _act(input, N.ACT_SILU)


def gelu(input: torch.Tensor) -> torch.Tensor:
    """``ops/activation.py:22-31`` (tanh approximation)."""
    return _act(input, N.ACT_GELU_TANH)


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``ops/activation.py:34-48``: ``silu(gate) * up``."""
    return _gated(gate, up, N.ACT_SILU)


def geglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``ops/activation.py:51-66``: ``gelu(gate) * up``."""
    return _gated(gate, up, N.ACT_GELU_TANH)


# ------------------------------------------------------------------------ sampling
def greedy_sample(logits: torch.Tensor) -> torch.Tensor:
    """``ops/sampling.py:10-21``: row argmax (lowest index among ties), int64 ``[B]``."""
    N.require_cuda(logits)
    x = logits.contiguous()
    V = x.shape[-1]
    rows = x.numel() // V
    out = torch.empty(rows, dtype=torch.int64, device=x.device)
    with torch.cuda.device(x.device):
        N.check(N.lib().mvb_greedy_sample(out.data_ptr(), x.data_ptr(), rows, V, V, N.dtype_code(x), _st(x)),
                "greedy_sample")
    return out


def top_k_top_p_filter(logits: torch.Tensor, top_k: int = 0, top_p: float = 1.0) -> torch.Tensor:
    """``ops/sampling.py:24-50``: filtered copy, non-survivors ``-inf`` (untempered logits).
    Among logits tied at the top-p cutoff the lower indices survive."""
    N.require_cuda(logits)
    x = logits.clone().contiguous()
    V = x.shape[-1]
    with torch.cuda.device(x.device):
        N.check(N.lib().mvb_top_k_top_p_filter(x.data_ptr(), x.numel() // V, V, int(top_k), float(top_p),
                                               N.dtype_code(x), _st(x)), "top_k_top_p_filter")
    return x


_rng_lock = threading.Lock()
_rng_fallback = [0]


def _next_seed_offset(device: torch.device, rows: int) -> tuple[int, int]:
    """(seed, offset) from torch's default CUDA generator, advanced like a draw of ``rows`` values."""
    gen = torch.cuda.default_generators[device.index if device.index is not None else torch.cuda.current_device()]
    seed = int(gen.initial_seed())
    with _rng_lock:
        if hasattr(gen, "get_offset"):
            off = int(gen.get_offset())
            gen.set_offset(off + 4 * ((rows + 3) // 4 + 1))
        else:
            off = _rng_fallback[0]
            _rng_fallback[0] += 1
    return seed, off


def softmax_multinomial_sample(logits: torch.Tensor, temperature: float = 1.0) -> torch.Tensor:
    """``ops/sampling.py:53-73``: ``softmax(logits / T)`` and one draw per row (int64 ``[B]``).
    The draw is a Philox4x32-10 inverse CDF seeded from torch's CUDA generator state."""
    N.require_cuda(logits)
    x = logits.contiguous()
    V = x.shape[-1]
    rows = x.numel() // V
    out = torch.empty(rows, dtype=torch.int64, device=x.device)
    seed, off = _next_seed_offset(x.device, rows)
    with torch.cuda.device(x.device):
        N.check(N.lib().mvb_softmax_multinomial_sample(out.data_ptr(), x.data_ptr(), rows, V, float(temperature),
                                                       seed, off, N.dtype_code(x), _st(x)),
                "softmax_multinomial_sample")
    return out


def sample(logits: torch.Tensor, temperature: torch.Tensor | float, top_k: torch.Tensor | int,
           top_p: torch.Tensor | float, seed: int, offset: int, probs_out: torch.Tensor | None = None,
           out: torch.Tensor | None = None, offset_dev: torch.Tensor | None = None) -> torch.Tensor:
    """Fused per-row sampler (greedy if T == 0, else top-k, top-p, /T, softmax, Philox draw).
    Per-row parameters may be CUDA tensors (fp32 / int32 / fp32 of length B) or scalars."""
    N.require_cuda(logits)
    x = logits if logits.stride(-1) == 1 else logits.contiguous()
    V = x.shape[-1]
    rows = x.numel() // V
    dev = x.device

    def vec(v, dt):
        if isinstance(v, torch.Tensor):
            return v.to(device=dev, dtype=dt).contiguous()
        return torch.full((rows,), v, dtype=dt, device=dev)

    t, k, p = vec(temperature, torch.float32), vec(top_k, torch.int32), vec(top_p, torch.float32)
    if out is None:
        out = torch.empty(rows, dtype=torch.int64, device=dev)
    with torch.cuda.device(dev):
        N.check(N.lib().mvb_sample(out.data_ptr(), N.ptr(probs_out), x.data_ptr(), rows, V, x.stride(-2) if x.dim() > 1
                                   else V, t.data_ptr(), k.data_ptr(), p.data_ptr(), int(seed), int(offset),
                                   N.ptr(offset_dev), N.dtype_code(x), _st(x)), "sample")
    return out


# ------------------------------------------------------------- embedding / softmax
def embedding(input_ids: torch.Tensor, weight: torch.Tensor, scale: float = 1.0) -> torch.Tensor:
    """``ops/embedding.py:11-35``: ``W[ids] * scale``; output shape ``ids.shape + [H]``."""
    N.require_cuda(input_ids, weight)
    ids = input_ids.reshape(-1).contiguous()
    if ids.dtype not in (torch.int32, torch.int64):
        ids = ids.to(torch.int64)
    w = weight.contiguous()
    V, H = w.shape
    out = torch.empty(ids.numel(), H, dtype=w.dtype, device=w.device)
    with torch.cuda.device(w.device):
        N.check(N.lib().mvb_embedding(out.data_ptr(), ids.data_ptr(), N.dtype_code(ids), w.data_ptr(), ids.numel(), H,
                                      V, float(scale), N.dtype_code(w), _st(w)), "embedding")
    return out.reshape(*input_ids.shape, H) if input_ids.dim() > 1 else out


class Embedding(nn.Module):
    """``ops/embedding.py:38-50``."""

    def __init__(self, num_embeddings: int, embedding_dim: int, scale: float = 1.0):
        super().__init__()
        self.weight = Parameter(torch.empty(num_embeddings, embedding_dim))
        self.scale = scale
        nn.init.normal_(self.weight, mean=0.0, std=0.02)

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        return embedding(input_ids, self.weight, self.scale)


def softmax(input: torch.Tensor, dim: int = -1) -> torch.Tensor:
    """``ops/softmax.py:5-25``: last-dim softmax in fp32, one rounding to the input dtype."""
    if dim != -1 and dim != input.dim() - 1:
        raise RuntimeError("softmax: only the last dimension is implemented by the kernel")
    N.require_cuda(input)
    x = input.contiguous()
    out = torch.empty_like(x)
    n = x.shape[-1]
    with torch.cuda.device(x.device):
        N.check(N.lib().mvb_softmax(out.data_ptr(), x.data_ptr(), x.numel() // n, n, N.dtype_code(x), _st(x)),
                "softmax")
    return out


# ----------------------------------------------------------------------- GEMM / MLP
class _Workspaces:
    """Zero-initialised scratch per device for the stream-K GEMM and split-KV attention.
    The kernels leave their counters at zero, so a buffer is reusable call after call
    on one stream (concurrent calls on different streams need separate buffers)."""

    def __init__(self):
        self._buf: dict[tuple[int, str], torch.Tensor] = {}
        self._lock = threading.Lock()

    def get(self, device: torch.device, kind: str, nbytes: int) -> torch.Tensor:
        key = (device.index if device.index is not None else torch.cuda.current_device(), kind)
        with self._lock:
            b = self._buf.get(key)
            if b is None or b.numel() < nbytes:
                b = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
                self._buf[key] = b
            return b


WORKSPACES = _Workspaces()


def linear(x: torch.Tensor, weight: torch.Tensor, epilogue: int = N.EPI_STORE, aux: torch.Tensor | None = None,
           out: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """``y = x @ weight.T`` (bf16, tcgen05).  ``epilogue``: EPI_STORE, EPI_SWIGLU (weight =
    cat([gate, up]); y = silu(gate) * up) or EPI_RESADD (y = aux + x @ W.T)."""
    N.require_cuda(x, weight)
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise RuntimeError("linear: the tcgen05 GEMM takes bf16 operands")
    K = x.shape[-1]
    xf = x.reshape(-1, K)
    if xf.stride(-1) != 1:
        xf = xf.contiguous()
    w = weight if weight.stride(-1) == 1 else weight.contiguous()
    Nn = w.shape[0]
    M = xf.shape[0]
    cols = Nn // 2 if epilogue == N.EPI_SWIGLU else Nn
    if out is None:
        out = torch.empty(M, cols, dtype=torch.bfloat16, device=x.device)
    auxf = None if aux is None else aux.reshape(-1, cols)
    dev = x.device
    with torch.cuda.device(dev):
        # + a fixed 1 MiB counter reserve: shapes sharing the cached buffer keep their partials
        # clear of every other shape's counters (up to 256K output tiles)
        need = N.lib().mvb_gemm_workspace_bytes(M, Nn, K, dev.index if dev.index is not None else 0) + (1 << 20)
        ws = workspace if workspace is not None else WORKSPACES.get(dev, "gemm", need)
        N.check(N.lib().mvb_gemm_bf16(out.data_ptr(), out.stride(0), xf.data_ptr(), xf.stride(0), w.data_ptr(),
                                      w.stride(0), M, Nn, K, epilogue, None if auxf is None else auxf.data_ptr(),
                                      0 if auxf is None else auxf.stride(0), ws.data_ptr(), ws.numel(), _st(x)),
                "gemm_bf16")
    return out.reshape(*x.shape[:-1], cols)


_ACT_CODE = {"silu": 0, "gelu": 1, "gelu_new": 1}   # ops/mlp.py:9-13


class FusedMLP(nn.Module):
    """``ops/mlp.py:46-84``: gate_up GEMM -> act(gate) * up -> down GEMM.

    For SiLU the activation runs in the gate_up GEMM's epilogue (one kernel); GELU uses
    the standalone fused_mlp kernel between the two GEMMs."""

    def __init__(self, hidden_size: int, intermediate_size: int, hidden_act: str = "silu"):
        super().__init__()
        self.gate_up_proj = nn.Linear(hidden_size, 2 * intermediate_size, bias=False)
        self.down_proj = nn.Linear(intermediate_size, hidden_size, bias=False)
        self.intermediate_size = intermediate_size
        self.hidden_act = hidden_act
        if hidden_act not in _ACT_CODE:
            raise ValueError(f"unsupported activation {hidden_act!r}")
        self._act_code = _ACT_CODE[hidden_act]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self._act_code == 0:
            h = linear(x, self.gate_up_proj.weight, N.EPI_SWIGLU)
        else:
            gu = linear(x, self.gate_up_proj.weight)
            h = fused_mlp_forward(gu, self.intermediate_size, self._act_code)
        return linear(h, self.down_proj.weight)


def fused_mlp_forward(gate_up: torch.Tensor, intermediate_size: int, activation: int) -> torch.Tensor:
    """``fused_mlp_forward`` (``mlp_kernel.cu:61-93``): ``act(gate_up[..., :I]) * gate_up[..., I:]``."""
    N.require_cuda(gate_up)
    g = gate_up.contiguous()
    rows = g.numel() // (2 * intermediate_size)
    out = torch.empty(*g.shape[:-1], intermediate_size, dtype=g.dtype, device=g.device)
    with torch.cuda.device(g.device):
        N.check(N.lib().mvb_fused_mlp(out.data_ptr(), g.data_ptr(), rows, intermediate_size, int(activation),
                                      N.dtype_code(g), _st(g)), "fused_mlp")
    return out


# ------------------------------------------------- paged decode attention / KV write
def qk_norm_rope_kv_write(qkv: torch.Tensor, kv_cache: torch.Tensor, layer: int, positions: torch.Tensor,
                          block_tables: torch.Tensor, cos_table: torch.Tensor, sin_table: torch.Tensor,
                          num_q_heads: int, num_kv_heads: int, q_norm_w: torch.Tensor | None = None,
                          k_norm_w: torch.Tensor | None = None, eps: float = 1e-6,
                          q_out: torch.Tensor | None = None, plus_one: bool = False) -> torch.Tensor:
    """Per-head QK-norm + RoPE of one new token per sequence and its K/V written into
    ``kv_cache[layer, 0|1, block_tables[b][pos // bs], pos % bs]``; returns q ``[B, Hq, D]``.
    ``plus_one`` selects Gemma's ``(1 + w)`` norm scale."""
    N.require_cuda(qkv, kv_cache, positions, block_tables, cos_table, sin_table)
    L, _, P, bs, nkv, D = kv_cache.shape
    B = qkv.shape[0]
    if q_out is None:
        q_out = torch.empty(B, num_q_heads, D, dtype=torch.bfloat16, device=qkv.device)
    with torch.cuda.device(qkv.device):
        N.check(N.lib().mvb_qk_norm_rope_kv_write(
            q_out.data_ptr(), kv_cache.data_ptr(), qkv.data_ptr(), qkv.stride(0), N.ptr(q_norm_w), N.ptr(k_norm_w),
            cos_table.data_ptr(), sin_table.data_ptr(), cos_table.shape[0], positions.data_ptr(),
            block_tables.data_ptr(), block_tables.shape[1], B, num_q_heads, num_kv_heads, D, L, layer, P, bs,
            float(eps), int(plus_one), _st(qkv)), "qk_norm_rope_kv_write")
    return q_out


def paged_attention_decode(q: torch.Tensor, kv_cache: torch.Tensor, layer: int, block_tables: torch.Tensor,
                           ctx_lens: torch.Tensor, scale: float, out: torch.Tensor | None = None,
                           workspace: torch.Tensor | None = None, softcap: float = 0.0,
                           window: int = 0) -> torch.Tensor:
    """Decode attention of q ``[B, Hq, D]`` over each sequence's first ``ctx_lens[b]`` cached
    tokens of ``layer`` (read through ``block_tables``); returns ``[B, Hq, D]``.  ``softcap`` > 0
    soft-caps the scaled scores (``softcap * tanh(s / softcap)``); ``window`` > 0 keeps only the
    newest ``window`` keys of each sequence."""
    N.require_cuda(q, kv_cache, block_tables, ctx_lens)
    L, _, P, bs, nkv, D = kv_cache.shape
    B, Hq, _ = q.shape
    if out is None:
        out = torch.empty_like(q)
    dev = q.device
    with torch.cuda.device(dev):
        need = N.lib().mvb_paged_attention_workspace_bytes(B, Hq, D, dev.index if dev.index is not None else 0) + (1 << 16)
        ws = workspace if workspace is not None else WORKSPACES.get(dev, "attention", need)
        N.check(N.lib().mvb_paged_attention_decode_ex(
            out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0), kv_cache.data_ptr(), block_tables.data_ptr(),
            block_tables.shape[1], ctx_lens.data_ptr(), B, Hq, nkv, D, L, layer, P, bs, float(scale), float(softcap),
            int(window), ws.data_ptr(), ws.numel(), _st(q)), "paged_attention_decode")
    return out
