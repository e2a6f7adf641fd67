"""Tensor parallelism for the decode path: one process per GPU, NVLink peer memory.

The reference ships only a stub (``mini_vllm/distributed/tensor_parallel.py:14-35``:
``TensorParallelConfig``, ``init_distributed`` and an engine that raises for
``tp_size > 1``).  This module keeps those names and supplies the Megatron-style split of
the decode step:

* q/k/v: column-parallel by heads (rank r owns query heads ``[r*Hq/N, (r+1)*Hq/N)`` and KV
  heads ``[r*Hkv/N, (r+1)*Hkv/N)``); the KV pool of a rank holds only its KV heads, while
  block tables and slots are replicated (the same FIFO allocator runs on every rank, so the
  indexing is bit-identical on each).
* o_proj, down_proj: row-parallel (the input columns of the rank's heads / intermediate
  features); their outputs are summed across ranks by the kernels themselves (push of fp32
  split-K partials to the owner of each batch row, residual + RMSNorm there, all-gather of
  the normalised rows), replacing the NCCL all-reduce.
* gate/up: column-parallel (``I/N`` features of each); lm_head: vocab-parallel
  (``V/N`` rows), all-gathered into every rank's logits so every rank samples the same tokens.
* embedding and norms: replicated.

Host plumbing (rendezvous, the IPC-handle exchange) uses ``torch.distributed``; the device
side is the ``mvb_tp_*`` C ABI.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import torch

from .configs import head_dim, num_kv_heads


@dataclass
class TensorParallelConfig:
    """``mini_vllm/distributed/tensor_parallel.py:14-20``: size and this process's rank.
    ``exchange`` runs the tensor-parallel kernels even for one rank (self-push, self-gather),
    which must reproduce the single-GPU step bit for bit."""
    tp_size: int = 1
    rank: int = 0
    exchange: bool = False

    @property
    def enabled(self) -> bool:
        return self.tp_size > 1 or self.exchange


def init_distributed(backend: str = "nccl", timeout_s: float = 60.0) -> TensorParallelConfig:
    """Joins the process group described by the torchrun environment (RANK, WORLD_SIZE,
    MASTER_ADDR, MASTER_PORT) and returns this process's ``TensorParallelConfig``
    (``tensor_parallel.py:23-35``).  A single process without that environment gets TP=1."""
    import datetime

    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        return TensorParallelConfig(1, 0)
    if not dist.is_initialized():
        kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group(backend, **kw)
    return TensorParallelConfig(dist.get_world_size(), dist.get_rank())


# ------------------------------------------------------------------------ weights
def check_divisible(cfg: dict, tp_size: int) -> None:
    """The split needs whole heads, whole intermediate slices (whole experts for a sparse MoE
    model) and whole vocab slices per rank."""
    hq, hkv, inter, vocab = (cfg["num_attention_heads"], num_kv_heads(cfg), cfg["intermediate_size"],
                             cfg["vocab_size"])
    checks = [("num_attention_heads", hq), ("vocab_size", vocab)]
    if hkv >= tp_size or tp_size % hkv:   # fewer KV heads than ranks: each is replicated on tp_size / hkv ranks
        checks.append(("num_key_value_heads", hkv))
    checks.append(("num_experts", cfg["num_experts"]) if cfg.get("num_experts") else ("intermediate_size", inter))
    for name, v in checks:
        if v % tp_size:
            raise ValueError(f"{name}={v} is not divisible by tp_size={tp_size}")


def local_kv_heads(cfg: dict, tp_size: int) -> int:
    """KV heads a rank holds: its share, or one replicated head when there are fewer KV heads than
    ranks (the query heads of a rank always sit in one GQA group then)."""
    return max(num_kv_heads(cfg) // tp_size, 1)


def kv_head_range(cfg: dict, tp_size: int, rank: int) -> tuple[int, int]:
    """The first KV head of rank ``rank`` and how many: heads [r n, (r + 1) n) when they split, else
    the one head whose GQA group holds the rank's query heads (head r / (tp_size / n_kv))."""
    hkv = num_kv_heads(cfg)
    if hkv >= tp_size:
        per = hkv // tp_size
        return rank * per, per
    return rank // (tp_size // hkv), 1


def expert_range(cfg: dict, tp_size: int, rank: int) -> tuple[int, int]:
    """Expert parallelism of a sparse MoE block: rank r holds experts [r E / T, (r + 1) E / T)."""
    per = cfg["num_experts"] // tp_size
    return rank * per, per


def shard_state_dict(cfg: dict, sd: dict[str, torch.Tensor], tp_size: int, rank: int) -> dict[str, torch.Tensor]:
    """Rank ``rank``'s part of a HuggingFace-keyed state dict (tensors are views or copies of
    ``sd``'s, on the same device).  Norm weights, the embedding and q_norm/k_norm (per head
    dimension) are replicated; a sparse MoE block's router is replicated and its experts are
    split whole over the ranks (``expert_range``)."""
    check_divisible(cfg, tp_size)
    if tp_size == 1:
        return dict(sd)
    D = head_dim(cfg)
    hq = cfg["num_attention_heads"] // tp_size
    kv0, hkv = kv_head_range(cfg, tp_size, rank)
    inter = cfg["intermediate_size"] // tp_size
    vocab = cfg["vocab_size"] // tp_size
    out: dict[str, torch.Tensor] = {}

    def rows(t, n):
        return t[rank * n:(rank + 1) * n].contiguous()

    def cols(t, n):
        return t[:, rank * n:(rank + 1) * n].contiguous()

    first, per = expert_range(cfg, tp_size, rank) if cfg.get("num_experts") else (0, 0)
    for k, t in sd.items():
        if ".mlp.experts." in k:   # expert parallel: this rank's experts, renumbered from 0
            head, tail = k.split(".mlp.experts.")
            if tail in ("gate_up_proj.weight", "down_proj.weight"):   # stacked [E, ...]
                out[k] = t[first:first + per].contiguous()
            else:
                j, rest = tail.split(".", 1)
                if first <= int(j) < first + per:
                    out[f"{head}.mlp.experts.{int(j) - first}.{rest}"] = t
            continue
        if k.endswith("self_attn.q_proj.weight"):
            out[k] = rows(t, hq * D)
        elif k.endswith("self_attn.k_proj.weight") or k.endswith("self_attn.v_proj.weight"):
            out[k] = t[kv0 * D:(kv0 + hkv) * D].contiguous()
        elif k.endswith("self_attn.o_proj.weight"):
            out[k] = cols(t, hq * D)
        elif k.endswith("mlp.gate_proj.weight") or k.endswith("mlp.up_proj.weight"):
            out[k] = rows(t, inter)
        elif k.endswith("mlp.down_proj.weight"):
            out[k] = cols(t, inter)
        elif k == "lm_head.weight":
            out[k] = rows(t, vocab)
        else:
            out[k] = t
    if "lm_head.weight" not in sd:          # tied embeddings: the head is a slice of the table
        out["lm_head.weight"] = rows(sd["model.embed_tokens.weight"], vocab)
    return out


def local_config(cfg: dict, tp_size: int) -> dict:
    """Per-rank head / feature counts (the model dims a rank's kernels see)."""
    check_divisible(cfg, tp_size)
    out = {"num_attention_heads": cfg["num_attention_heads"] // tp_size,
           "num_key_value_heads": local_kv_heads(cfg, tp_size),
           "intermediate_size": cfg["intermediate_size"] // tp_size,
           "vocab_size": cfg["vocab_size"] // tp_size}
    if cfg.get("num_experts"):
        out["num_experts"] = cfg["num_experts"] // tp_size
    return out


# ------------------------------------------------------------------- signal points
def point_o_proj(layer: int) -> int:
    """o_proj partials pushed to their owners."""
    return 4 * layer


def point_attn_norm(layer: int) -> int:
    """Rows normalised after attention (post_attention_layernorm) all-gathered."""
    return 4 * layer + 1


def point_down(layer: int) -> int:
    """down_proj partials pushed to their owners."""
    return 4 * layer + 2


def point_mlp_norm(layer: int) -> int:
    """Rows normalised after the MLP (next input_layernorm, or the final norm) all-gathered."""
    return 4 * layer + 3


def point_logits(num_layers: int) -> int:
    """lm_head columns all-gathered."""
    return 4 * num_layers


# --------------------------------------------------------------------- heap layout
def _align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


@dataclass
class HeapLayout:
    """Byte offsets of the symmetric buffers; identical on every rank."""
    xn: int          # [B, H] bf16 normalised activations (every rank writes its rows into all)
    recv_o: int      # receive area of the o_proj push
    recv_down: int   # receive area of the down_proj push
    logits: int      # [B, V] bf16 full logits
    total: int


def plan_heap(signal_bytes: int, batch: int, hidden: int, vocab: int, recv_o_bytes: int,
              recv_down_bytes: int) -> HeapLayout:
    off = _align(signal_bytes)
    xn = off
    off = _align(off + batch * hidden * 2)
    recv_o = off
    off = _align(off + recv_o_bytes)
    recv_down = off
    off = _align(off + recv_down_bytes)
    logits = off
    off = _align(off + batch * vocab * 2)
    return HeapLayout(xn, recv_o, recv_down, logits, off)


class SymmetricHeap:
    """One device allocation per rank, mapped into every other rank's address space (CUDA IPC),
    plus the ``mvb_tp_comm`` that the TP kernels take."""

    def __init__(self, nbytes: int, rank: int, world: int, group=None):
        import torch.distributed as dist

        from . import _native as N

        self.lib = N.lib()
        self.rank, self.world, self.nbytes = rank, world, int(nbytes)
        base = C.c_void_p()
        handle = C.create_string_buffer(64)
        N.check(self.lib.mvb_tp_heap_alloc(self.nbytes, C.byref(base), handle), "mvb_tp_heap_alloc")
        self.base = base.value
        handles: list = [handle.raw]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, handle.raw, group=group)
        blob = b"".join(handles)
        comm = C.c_void_p()
        N.check(self.lib.mvb_tp_comm_init(rank, world, C.c_void_p(self.base), blob, self.nbytes, C.byref(comm)),
                "mvb_tp_comm_init")
        self.comm = comm.value

    def tensor(self, offset: int, shape: tuple, dtype: torch.dtype, device) -> torch.Tensor:
        """A torch view of this rank's heap at ``offset`` (no copy; the heap outlives it)."""
        numel = 1
        for s in shape:
            numel *= s
        nbytes = numel * torch.empty((), dtype=dtype).element_size()
        if offset < 0 or offset + nbytes > self.nbytes:
            raise ValueError("view outside the heap")
        return _device_view(self.base + offset, shape, dtype, device)

    def close(self) -> None:
        if self.comm:
            self.lib.mvb_tp_comm_destroy(C.c_void_p(self.comm))
            self.comm = None
        if self.base:
            self.lib.mvb_tp_heap_free(C.c_void_p(self.base))
            self.base = None


def _device_view(ptr: int, shape: tuple, dtype: torch.dtype, device) -> torch.Tensor:
    """Wraps raw device memory as a tensor through ``__cuda_array_interface__`` (no ownership)."""
    typestr = {torch.bfloat16: "<i2", torch.float32: "<f4", torch.int32: "<i4", torch.uint8: "|u1"}[dtype]

    class _Mem:
        __cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False), "version": 3,
                                    "strides": None}

    t = torch.as_tensor(_Mem(), device=device)
    return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t
