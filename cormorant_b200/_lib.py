"""ctypes binding of libcormorant_cuda.so (C ABI declared in include/cormorant_cuda.h).

The library is built in-tree (``python -m cormorant_b200.build``).  There is no
fallback: if it is missing or cannot be loaded, ``lib()`` raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libcormorant_cuda.so"

CM_OK = 0
CM_EINVAL = -1
CM_EUNSUPPORTED = -2
CM_ECUDA = -3
CM_ETIMEOUT = -4
CM_ENOMEM = -5
CM_ENOINIT = -6

_p = C.c_void_p
_u = C.c_uint

# name -> (restype, argtypes); every function declared in include/cormorant_cuda.h
SIGNATURES: dict[str, tuple] = {
    "cm_init": (C.c_int, [C.c_char_p]),
    "cm_release": (C.c_int, []),
    "cm_device": (C.c_int, []),
    "cm_strerror": (C.c_char_p, [C.c_int]),
    "cm_last_error": (C.c_char_p, []),
    "cm_synchronize": (C.c_int, [_p]),
    "cm_launch_count": (C.c_uint64, []),
    "cm_set_direct_limit": (C.c_uint64, [C.c_uint64]),
    "cm_set_gemm_split": (C.c_int, [C.c_int]),
    "cm_version": (C.c_char_p, []),
    "cm_selftest_wait_timeout": (C.c_int, [_u]),
    "cm_int8_mma_rate": (C.c_int, [_u, _u, C.POINTER(C.c_double), C.POINTER(C.c_double), C.POINTER(C.c_double)]),
    "cm_profile_begin": (C.c_int, []),
    "cm_profile_end": (C.c_int, []),
    "cm_profile_read": (C.c_int, [C.c_char_p, C.POINTER(C.c_double), C.POINTER(C.c_uint64)]),
    "cm_profile_gemm_clock": (C.c_int, [C.POINTER(C.c_double)]),
    "cm_vectorop": (C.c_int, [_p, _p, _p] + [_u] * 5),
    "cm_vectorop_async": (C.c_int, [_p, _p, _p] + [_u] * 5 + [_p]),
    "cm_matmul": (C.c_int, [_p, _p, _p] + [_u] * 7),
    "cm_matmul_async": (C.c_int, [_p, _p, _p] + [_u] * 7 + [_p]),
    "cm_matmul_fused": (C.c_int, [_p, _p, _p] + [_u] * 8 + [_p]),
    "cm_matmul_fused_async": (C.c_int, [_p, _p, _p] + [_u] * 8 + [_p, _p]),
    "cm_matmul_at": (C.c_int, [_p, _u, _p, _u, _p, _u] + [_u] * 7),
    "cm_matmul_noalloc": (C.c_int, [_p, _p, _p] + [_u] * 7 + [_p]),
    "cm_conv": (C.c_int, [_p, _p, _p, _p] + [_u] * 17),
    "cm_conv_async": (C.c_int, [_p, _p, _p, _p] + [_u] * 17 + [_p]),
    "cm_conv_fused": (C.c_int, [_p, _p, _p, _p] + [_u] * 18 + [_p]),
    "cm_conv_fused_async": (C.c_int, [_p, _p, _p, _p] + [_u] * 18 + [_p, _p]),
    "cm_conv_pool": (C.c_int, [_p, _p, _p, _p] + [_u] * 18 + [_p] + [_u] * 17),
    "cm_conv_pool_async": (C.c_int, [_p, _p, _p, _p] + [_u] * 18 + [_p] + [_u] * 17 + [_p]),
    "cm_planes_create": (_p, [_u] * 8),
    "cm_planes_destroy": (None, [_p]),
    "cm_planes_fill": (C.c_int, [_p, _p]),
    "cm_planes_fill_async": (C.c_int, [_p, _p, _p]),
    "cm_pool_planes": (C.c_int, [_p, _p] + [_u] * 17),
    "cm_pool_planes_async": (C.c_int, [_p, _p] + [_u] * 17 + [_p]),
    "cm_pool_nhwc": (C.c_int, [_p, _p] + [_u] * 17),
    "cm_pool_nhwc_async": (C.c_int, [_p, _p] + [_u] * 17 + [_p]),
    "cm_pool_nhwc_planes": (C.c_int, [_p, _p] + [_u] * 15),
    "cm_pool_nhwc_planes_async": (C.c_int, [_p, _p] + [_u] * 15 + [_p]),
    "cm_conv_plane_frame": (C.c_int, [_u] * 17 + [C.POINTER(_u)]),
    "cm_conv_writes_nhwc": (C.c_int, [_u] * 17),
    "cm_conv_planes": (C.c_int, [_p] * 6 + [_u] * 18 + [_p, _p]),
    "cm_conv_planes_async": (C.c_int, [_p] * 6 + [_u] * 18 + [_p, _p, _p]),
    "cm_matmul_weights_create": (C.c_int, [_p, _u, _u, C.POINTER(_p)]),
    "cm_matmul_weights_destroy": (None, [_p]),
    "cm_matmul_prepared": (C.c_int, [_p, _p, _p] + [_u] * 5 + [_p]),
    "cm_matmul_prepared_async": (C.c_int, [_p, _p, _p] + [_u] * 5 + [_p, _p]),
    "cm_conv_weights_create": (C.c_int, [_p, _p] + [_u] * 17 + [C.POINTER(_p)]),
    "cm_conv_weights_destroy": (None, [_p]),
    "cm_conv_prepared": (C.c_int, [_p] * 5 + [_u, _p, _p]),
    "cm_conv_prepared_async": (C.c_int, [_p] * 5 + [_u, _p, _p, _p]),
    "cm_calls_supported": (C.c_int, [_p, _u]),
    "cm_calls": (C.c_int, [_p, _u]),
    "cm_calls_async": (C.c_int, [_p, _u, _p]),
    "cm_pool": (C.c_int, [_p, _p] + [_u] * 17),
    "cm_pool_async": (C.c_int, [_p, _p] + [_u] * 17 + [_p]),
    "cm_ipc_export": (C.c_int, [_p, _p]),
    "cm_ipc_open": (C.c_int, [_p, C.POINTER(_p)]),
    "cm_ipc_close": (C.c_int, [_p]),
    "cm_copy_async": (C.c_int, [_p, _p, C.c_size_t, _p]),
    "cm_buf_alloc": (_p, [_u]),
    "cm_buf_free": (None, [_p]),
    "cm_buf_retain": (None, [_p]),
    "cm_buf_release": (None, [_p]),
    "cm_buf_ptr": (_p, [_p]),
    "cm_buf_dev": (C.c_uint64, [_p]),
    "cm_buf_count": (_u, [_p]),
    "cm_buf_init_view": (None, [_p, _p, _u, _u]),
    "cm_buf_sync_to_device": (C.c_int, [_p]),
    "cm_buf_sync_from_device": (C.c_int, [_p]),
    "cm_buf_sync_to_device_async": (C.c_int, [_p, _p]),
    "cm_buf_sync_from_device_async": (C.c_int, [_p, _p]),
}


class CormorantError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status


_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is not built; run `python -m cormorant_b200.build`")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != CM_OK:
        msg = lib().cm_last_error()
        raise CormorantError(rc, (msg or b"").decode(errors="replace") or lib().cm_strerror(rc).decode())
