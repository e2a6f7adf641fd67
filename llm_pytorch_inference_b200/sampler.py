"""Drop-in for the reference's ``Sampler`` (``mini_vllm/engine/sampler.py:6-69``) on the sm_100a kernels.

``Sampler.sample(logits, SamplingParams) -> list[int]`` keeps the reference's signature and the
semantics its engine gets on CUDA tensors (``sampler.py:40-48`` with the ``mini_vllm.ops``
fallbacks, ``ops/sampling.py:10-73``):

* ``temperature == 0``: argmax, the lowest index among equal maxima (``mvb_greedy_sample``);
* otherwise: top-k (ties at the k-th value kept), then top-p on the *untempered* logits, then
  ``/ T`` and softmax -- one fused kernel (``mvb_sample``) writes these probabilities -- and the
  draw.

The draw has two modes.  ``"reference"`` (default) is the reference's own draw,
``torch.multinomial(probs, 1)`` on torch's generator, so given the same logits and generator
state the tokens are the reference's.  ``"fast"`` keeps the draw in the kernel: one
Philox4x32-10 uniform per row (seed and offset taken from torch's CUDA generator) and an inverse
CDF over the filtered distribution in vocabulary order, with no host round trip.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import _native as N
from . import ops


@dataclass
class SamplingParams:
    """The fields of the reference's ``SamplingParams`` (``utils/config.py:61-68``)."""
    temperature: float = 1.0
    top_k: int = -1
    top_p: float = 1.0
    max_tokens: int = 512
    stop: list[str] = field(default_factory=list)
    presence_penalty: float = 0.0
    eos_token_id: int | list[int] = 2


class Sampler:
    def __init__(self, mode: str = "reference", generator: torch.Generator | None = None):
        if mode not in ("reference", "fast"):
            raise ValueError(f"unknown sampling mode {mode!r}")
        self.mode = mode
        self.generator = generator

    def sample(self, logits: torch.Tensor, sampling_params) -> list[int]:
        """``sampler.py:21-31``: one token per row of ``logits`` ``[batch, vocab]`` (a CUDA tensor,
        fp32 / bf16 / fp16)."""
        N.require_cuda(logits)
        if sampling_params.temperature == 0.0:
            return ops.greedy_sample(logits).tolist()
        x = logits if logits.dim() == 2 else logits.reshape(-1, logits.shape[-1])
        rows, V = x.shape
        T, k, p = float(sampling_params.temperature), int(sampling_params.top_k), float(sampling_params.top_p)
        if not T > 0.0:   # ops/sampling.py:69: a negative temperature samples at T = 1
            T = 1.0
        if self.mode == "fast":
            seed, off = ops._next_seed_offset(x.device, rows)
            return ops.sample(x, T, k, p, seed, off).tolist()
        probs = torch.empty(rows, V, dtype=torch.float32, device=x.device)
        ops.sample(x, T, k, p, 0, 0, probs_out=probs)
        return torch.multinomial(probs, num_samples=1, generator=self.generator).squeeze(-1).tolist()
