"""Oracle restatement of the reference's sampling semantics (CPU, fp32/fp64).

Two reference semantics exist (both restated here):

* logits on a CUDA tensor -- ``Sampler._sample_with_temperature`` hands them to
  ``mini_vllm.ops.sampling`` (``sampler.py:40-48``), whose PyTorch fallbacks are:
  top-k then top-p on the *untempered* logits (``ops/sampling.py:26-50``), then
  ``/T`` and softmax (``ops/sampling.py:60-73``).  This is the semantics of the
  GPU decode path and of ``top_k_top_p_filter`` / ``softmax_multinomial_sample``.
* logits on a CPU tensor -- ``sampler.py:50-69``: ``/T`` first, then top-k, top-p.

The reference draws with ``torch.multinomial``.  The CUDA path's own draw is an
inverse CDF over the filtered distribution in vocabulary order, driven by one
Philox4x32-10 uniform per row; ``philox4x32_10`` and ``inverse_cdf`` below are its
CPU statement (Philox: Salmon et al., "Parallel random numbers: as easy as 1, 2,
3", SC'11 -- the published round function and constants).
"""
from __future__ import annotations

import numpy as np
import torch

NEG_INF = float("-inf")


def greedy(logits: torch.Tensor) -> torch.Tensor:
    """``ops/sampling.py:19-21``: argmax, first index on ties, int64."""
    return logits.argmax(dim=-1).to(torch.int64)


def top_k_top_p_filter(logits: torch.Tensor, top_k: int = 0, top_p: float = 1.0,
                       stable: bool = False) -> torch.Tensor:
    """``ops/sampling.py:26-50`` (PyTorch branch).  Ties at the k-th value are kept.

    Top-p sorts descending.  The reference's ``torch.sort`` leaves the order of
    equal logits unspecified, so when the cutoff falls inside a group of tied
    (bf16-rounded) logits, *which* of them survive is implementation-defined; the
    number kept and their values are not.  ``stable=False`` reproduces the
    reference call exactly; ``stable=True`` puts the lower index first among
    ties, the rule the CUDA kernel implements.
    """
    x = logits.clone()
    if top_k > 0:
        kth = torch.topk(x, min(top_k, x.shape[-1]))[0][..., -1, None]
        x[x < kth] = NEG_INF
    if top_p < 1.0:
        sx, si = torch.sort(x, descending=True, stable=stable) if stable else torch.sort(x, descending=True)
        sm = torch.softmax(sx, dim=-1)
        remove = torch.cumsum(sm, dim=-1) - sm >= top_p
        sx[remove] = NEG_INF
        x = sx.scatter(-1, si, sx)
    return x


def tempered_probs(logits: torch.Tensor, temperature: float) -> torch.Tensor:
    """``ops/sampling.py:69-72``: divide by T (unless T is 0 or 1), then softmax."""
    if temperature > 0 and temperature != 1.0:
        logits = logits / temperature
    return torch.softmax(logits, dim=-1)


def gpu_semantics_probs(logits: torch.Tensor, temperature: float, top_k: int, top_p: float,
                        stable: bool = True) -> torch.Tensor:
    """``sampler.py:40-48`` on a CUDA tensor: filter (if enabled), then tempered softmax."""
    if top_k > 0 or top_p < 1.0:
        logits = top_k_top_p_filter(logits, top_k, top_p, stable=stable)
    return tempered_probs(logits, temperature)


def cpu_semantics_logits(logits: torch.Tensor, temperature: float, top_k: int, top_p: float) -> torch.Tensor:
    """``sampler.py:50-69`` on a CPU tensor: ``/T`` first, then top-k (``:71-76``), top-p (``:78-88``)."""
    x = logits / temperature
    if top_k > 0:
        kth = torch.topk(x, top_k)[0][..., -1, None]
        x = x.clone()
        x[x < kth] = NEG_INF
    if top_p < 1.0:
        sx, si = torch.sort(x, descending=True)
        cp = torch.cumsum(torch.softmax(sx, dim=-1), dim=-1)
        rm = cp - torch.softmax(sx, dim=-1) >= top_p
        sx = sx.clone()
        sx[rm] = NEG_INF
        x = sx.scatter(-1, si, sx)
    return x


# ------------------------------------------------------------------ Philox draw
_M0, _M1 = 0xD2511F53, 0xCD9E8D57
_W0, _W1 = 0x9E3779B9, 0xBB67AE85
_MASK = 0xFFFFFFFF


def philox4x32_10(ctr: tuple[int, int, int, int], key: tuple[int, int]) -> tuple[int, int, int, int]:
    """Philox4x32 with 10 rounds (Random123 round function and Weyl key schedule)."""
    c0, c1, c2, c3 = (int(c) & _MASK for c in ctr)
    k0, k1 = (int(k) & _MASK for k in key)
    for r in range(10):
        if r:
            k0, k1 = (k0 + _W0) & _MASK, (k1 + _W1) & _MASK
        p0, p1 = _M0 * c0, _M1 * c2
        hi0, lo0 = p0 >> 32, p0 & _MASK
        hi1, lo1 = p1 >> 32, p1 & _MASK
        c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
    return c0, c1, c2, c3


SAMPLE_TAG = 0x53414D50  # fourth counter word of every sampling draw


def uniform(seed: int, row: int, offset: int) -> float:
    """The uniform in [0, 1) the kernel draws for ``row`` at ``offset`` (24-bit resolution)."""
    w = philox4x32_10((row, offset & _MASK, (offset >> 32) & _MASK, SAMPLE_TAG), (seed & _MASK, (seed >> 32) & _MASK))
    return (w[0] >> 8) * (1.0 / 16777216.0)


def inverse_cdf(weights: np.ndarray, u: float) -> tuple[int, float]:
    """First index (vocabulary order) whose running sum of ``weights`` exceeds ``u * total``.

    Returns the index and the relative distance of ``u * total`` to the nearest
    bucket edge, so a comparison can tell a real mismatch from a float tie.
    """
    w = np.asarray(weights, dtype=np.float64)
    cdf = np.cumsum(w)
    total = cdf[-1]
    target = u * total
    idx = int(np.searchsorted(cdf, target, side="right"))
    nz = np.nonzero(w)[0]
    if idx >= len(w):
        idx = int(nz[-1])
    edges = np.abs(cdf[nz] - target)
    return idx, float(edges.min() / total) if len(edges) else 1.0


def sample_row(logits_row: torch.Tensor, temperature: float, top_k: int, top_p: float,
               seed: int, row: int, offset: int) -> tuple[int, float]:
    """The CUDA path's sampled token for one fp32 logits row (GPU semantics + Philox draw)."""
    if temperature == 0.0:
        return int(greedy(logits_row[None])[0]), 1.0
    probs = gpu_semantics_probs(logits_row.double()[None], temperature, top_k, top_p)[0]
    return inverse_cdf(probs.numpy(), uniform(seed, row, offset))
