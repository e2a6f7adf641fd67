"""ctypes binding of the C ABI in ``include/mvb200.h`` (``libmvb200.so``).

The library is loaded from the package directory (built in-tree by
``llm_pytorch_inference_b200.build``).  There is no fallback: if it is missing or a
call fails, a ``RuntimeError`` carries the library's own message.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libmvb200.so"

MVB_OK = 0
F32, F16, BF16, I32, I64 = 0, 1, 2, 3, 4
NORM_OPS, NORM_MODEL = 0, 1
ACT_SILU, ACT_GELU_TANH = 0, 1
EPI_STORE, EPI_SWIGLU, EPI_RESADD, EPI_PARTIALS, EPI_SWIGLU_PARTIALS = 0, 1, 2, 3, 4
DEV_WAIT_TIMEOUT, DEV_BAD_BLOCK, DEV_BAD_POSITION, DEV_BAD_TOKEN, DEV_SAMPLER_TIES = 0x1, 0x2, 0x4, 0x8, 0x10

_vp, _i64, _i32, _f32, _u64, _u32p = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_uint64, C.POINTER(C.c_uint)
_vpp = C.POINTER(C.c_void_p)

# name -> (restype, argtypes); the exact list of entry points the header declares.
SIGNATURES: dict[str, tuple] = {
    "mvb_last_error": (C.c_char_p, []),
    "mvb_version": (_i32, []),
    "mvb_num_sms": (_i32, [_i32]),
    "mvb_device_status": (_i32, [_u32p, _i32, _vp]),
    "mvb_set_pdl": (_i32, [_i32]),
    "mvb_rmsnorm": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _f32, _i32, _i32, _i32, _vp]),
    "mvb_fused_add_rmsnorm": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _f32, _i32, _i32, _i32, _vp]),
    "mvb_fused_add_rmsnorm_gemm": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _f32, _i32, _vp]),
    "mvb_fused_norm_add_rmsnorm_gemm": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp, _f32, _i32, _vp]),
    "mvb_rotary_pos_emb": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i32, _vp]),
    "mvb_activation": (_i32, [_vp, _vp, _i64, _i32, _i32, _vp]),
    "mvb_gated_activation": (_i32, [_vp, _vp, _vp, _i64, _i32, _i32, _vp]),
    "mvb_fused_mlp": (_i32, [_vp, _vp, _i64, _i64, _i32, _i32, _vp]),
    "mvb_embedding": (_i32, [_vp, _vp, _i32, _vp, _i64, _i64, _i64, _f32, _i32, _vp]),
    "mvb_softmax": (_i32, [_vp, _vp, _i64, _i64, _i32, _vp]),
    "mvb_greedy_sample": (_i32, [_vp, _vp, _i64, _i64, _i64, _i32, _vp]),
    "mvb_top_k_top_p_filter": (_i32, [_vp, _i64, _i64, _i32, _f32, _i32, _vp]),
    "mvb_softmax_multinomial_sample": (_i32, [_vp, _vp, _i64, _i64, _f32, _u64, _u64, _i32, _vp]),
    "mvb_sample": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _u64, _u64, _vp, _i32, _vp]),
    "mvb_qk_norm_rope_kv_write": (_i32, [_vp, _vp, _vp, _i64, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _i64, _i64,
                                         _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _vp]),
    "mvb_qk_norm_rope_kv_write_gemm": (_i32, [_vp, _vp, _vp, _i64, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _i64, _i64,
                                              _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _vp]),
    "mvb_paged_attention_workspace_bytes": (_i64, [_i64, _i64, _i64, _i32]),
    "mvb_paged_attention_decode": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _i64,
                                          _i64, _i64, _i64, _i64, _f32, _vp, _i64, _vp]),
    "mvb_prefill_attention": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
                                     _i64, _i64, _i64, _i64, _i64, _f32, _vp]),
    "mvb_paged_attention_decode_ex": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _i64,
                                             _i64, _i64, _i64, _i64, _f32, _f32, _i64, _vp, _i64, _vp]),
    "mvb_paged_attention_decode_noalloc": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _i64, _i64, _i64,
                                                  _i64, _i64, _i64, _i64, _i64, _f32, _vp]),
    "mvb_gemm_workspace_bytes": (_i64, [_i64, _i64, _i64, _i32]),
    "mvb_gemm_bf16": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _i32, _vp, _i64, _vp, _i64, _vp]),
    "mvb_swiglu_gemm": (_i32, [_vp, _i64, _vp, _i64, _i64, _i64, _vp]),
    "mvb_gated_gemm": (_i32, [_vp, _i64, _vp, _i64, _i64, _i64, _i32, _vp]),
    "mvb_softcap": (_i32, [_vp, _i64, _f32, _i32, _vp]),
    "mvb_feed_ids": (_i32, [_vp, _vp, _vp, _i64, _vp]),
    "mvb_decoder_layer_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64, _i64, _i32]),
    "mvb_decoder_layer_tail": (_i32, [_vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                      _vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                      _i64, _i64, _f32, _vp, _i64, _vp, _vp]),
    "mvb_tp_decoder_layer_tail": (_i32, [_vp, _i32, _vp, _i64] + [_vp] * 9 + [_i64] + [_vp] * 5 +
                                  [_i64, _vp, _vp, _i64] + [_i64] * 10 + [_f32, _i64, _i64, _vp, _i64, _vp, _vp]),
    "mvb_moe_route": (_i32, [_vp, _i64, _i64, _i64, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "mvb_moe_gather": (_i32, [_vp, _vp, _i64, _vp, _i64, _vp]),
    "mvb_moe_gemm_bf16": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _i32, _vp, _vp, _vp]),
    "mvb_moe_combine": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "mvb_moe_combine_experts": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp]),
    "mvb_moe_gemm_bf16_experts": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i32,
                                         _vp, _vp, _vp]),
    "mvb_tp_moe_combine": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _vp]),
    "mvb_tp_signal_bytes": (_i64, []),
    "mvb_tp_heap_alloc": (_i32, [_i64, _vpp, C.c_char_p]),
    "mvb_tp_heap_free": (_i32, [_vp]),
    "mvb_tp_comm_init": (_i32, [_i32, _i32, _vp, C.c_char_p, _i64, _vpp]),
    "mvb_tp_comm_destroy": (_i32, [_vp]),
    "mvb_tp_begin_step": (_i32, [_vp, _vp]),
    "mvb_tp_recv_bytes": (_i64, [_i64, _i64, _i64, _i32, _i32]),
    "mvb_tp_gemm_bf16": (_i32, [_vp, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _i32, _vp, _i64, _i64, _i64, _i32, _i32,
                                _vp]),
    "mvb_tp_fused_add_rmsnorm_gemm": (_i32, [_vp, _vp, _i64, _i64, _i64, _vp, _f32, _i32, _i64, _i32, _i64, _i32,
                                             _vp]),
    "mvb_tp_fused_norm_add_rmsnorm_gemm": (_i32, [_vp, _vp, _i64, _i64, _i64, _vp, _vp, _f32, _i32, _i64, _i32,
                                                  _i64, _i32, _vp]),
    "mvb_tp_wait": (_i32, [_vp, _i32, _vp]),
}

_lock = threading.Lock()
_lib: C.CDLL | None = None


def load(path: str | Path = LIB_PATH) -> C.CDLL:
    """Load libmvb200.so once and attach the prototypes (no GPU needed)."""
    global _lib
    with _lock:
        if _lib is None:
            p = Path(path)
            if not p.exists():
                raise RuntimeError(f"{p} is missing: build it with `python -m llm_pytorch_inference_b200.build`")
            lib = C.CDLL(str(p))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
        return _lib


def lib() -> C.CDLL:
    return _lib if _lib is not None else load()


def check(rc: int, what: str) -> None:
    if rc != MVB_OK:
        msg = lib().mvb_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed (status {rc}): {msg}")


_DT = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16, torch.int32: I32, torch.int64: I64}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise RuntimeError(f"unsupported dtype {t.dtype}") from None


def require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("llm_pytorch_inference_b200 kernels run on CUDA tensors only (no CPU path)")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_status(clear: bool = True, stream: int | None = None) -> int:
    """OR of MVB_DEV_* bits the kernels reported on the current device (synchronises)."""
    v = C.c_uint(0)
    check(lib().mvb_device_status(C.byref(v), 1 if clear else 0, stream if stream is not None else stream_handle()),
          "mvb_device_status")
    return int(v.value)


def set_pdl(enable: bool) -> bool:
    return bool(lib().mvb_set_pdl(1 if enable else 0))
