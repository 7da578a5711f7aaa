"""C-ABI checks that need no GPU: libcormorant_cuda.so loads, exports every
function include/cormorant_cuda.h declares with the arity the ctypes binding
uses, and reports errors through status codes instead of crashing."""
import re
from pathlib import Path

import pytest

from cormorant_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "cormorant_cuda.h"


def declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    out = {}
    for m in re.finditer(r"\b(cm_\w+)\s*\(([^;{]*?)\)\s*;", text):
        args = m.group(2).strip()
        out[m.group(1)] = 0 if args in ("", "void") else args.count(",") + 1
    return out


def test_header_declares_the_kernel_entries():
    d = declared()
    for name in ("cm_vectorop", "cm_matmul", "cm_conv", "cm_pool", "cm_init", "cm_buf_alloc"):
        assert name in d
    assert d["cm_vectorop"] == 8 and d["cm_matmul"] == 10 and d["cm_conv"] == 21 and d["cm_pool"] == 19


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    d = declared()
    missing = [n for n in d if not hasattr(L, n)]
    assert not missing, missing
    assert set(d) == set(_lib.SIGNATURES), set(d) ^ set(_lib.SIGNATURES)
    for name, nargs in d.items():
        assert len(_lib.SIGNATURES[name][1]) == nargs, name


def test_calls_before_init_report_enoinit():
    L = _lib.lib()
    assert L.cm_device() in (_lib.CM_ENOINIT,) or L.cm_device() >= 0
    if L.cm_device() >= 0:
        pytest.skip("already initialised in this process")
    assert L.cm_vectorop(None, None, None, 16, 0, 1, 0, 0) == _lib.CM_ENOINIT
    assert L.cm_matmul(None, None, None, 1, 1, 1, 1, 0, 0, 0) == _lib.CM_ENOINIT
    assert L.cm_conv(None, None, None, None, *([1] * 17)) == _lib.CM_ENOINIT
    assert L.cm_pool(None, None, *([1] * 17)) == _lib.CM_ENOINIT
    # the prepared-weights entries refuse the same way and leave the result pointer null
    import ctypes as C
    out = C.c_void_p(12345)
    assert L.cm_conv_weights_create(None, None, *([1] * 17), C.byref(out)) == _lib.CM_ENOINIT
    assert out.value is None
    assert L.cm_conv_prepared(None, None, None, None, None, 0, None, None) == _lib.CM_ENOINIT
    L.cm_conv_weights_destroy(None)                       # null is accepted
    assert b"cm_init" in L.cm_last_error()


def test_strerror_covers_codes():
    L = _lib.lib()
    for code in (0, -1, -2, -3, -4, -5, -6):
        assert L.cm_strerror(code) and L.cm_strerror(code) != b"unknown status"


def test_init_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    L = _lib.lib()
    rc = L.cm_init(b"0")
    assert rc < 0 and L.cm_last_error()
    assert L.cm_init(b"bogus") == _lib.CM_EINVAL
