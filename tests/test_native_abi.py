"""The C-ABI library loads without a GPU and exports exactly what include/mvb200.h declares."""
import ctypes
import re
from pathlib import Path

import pytest

from llm_pytorch_inference_b200 import _native as N

HEADER = Path(__file__).resolve().parent.parent / "include" / "mvb200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mvb_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not N.LIB_PATH.exists():
        from llm_pytorch_inference_b200.build import build
        build()
    return N.load()


def test_header_declares_entry_points():
    names = declared_functions()
    assert "mvb_gemm_bf16" in names and "mvb_paged_attention_decode" in names and len(names) >= 20


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_ctypes_table_covers_header(lib):
    assert sorted(N.SIGNATURES) == declared_functions()


def test_calls_that_need_no_gpu(lib):
    assert lib.mvb_version() == 1
    assert lib.mvb_set_pdl(0) in (0, 1)
    # argument validation fails before any CUDA call and sets the message
    rc = lib.mvb_rmsnorm(None, 0, None, 0, None, 1, 1, 1e-6, 0, 0, N.BF16, None)
    assert rc == 1 and b"null pointer" in lib.mvb_last_error()
    rc = lib.mvb_gemm_bf16(1, 64, 1, 64, 1, 64, 300, 64, 64, N.EPI_PARTIALS, None, 0, 1, 0, None)
    assert rc == 1 and b"m=300" in lib.mvb_last_error()   # > 256 rows: not in split-K partial form


def test_check_raises_with_library_message(lib):
    rc = lib.mvb_paged_attention_decode(None, 0, None, 0, None, None, 0, None, 1, 1, 1, 128, 1, 0, 1, 16, 1.0,
                                        None, 0, None)
    with pytest.raises(RuntimeError, match="null pointer"):
        N.check(rc, "paged_attention_decode")
