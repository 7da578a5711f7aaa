"""Mirror of the reference's generated host runtime for the four kernels.

``InferenceBuf`` mirrors ``inference_buf_t`` (inference-scheduler/src/codegen/
_buf_impl.py:25-236): an owner buffer is a device allocation plus a pinned host
mirror; ``phys()`` returns the device address the kernels are given (the
reference programs the DMA physical address); views alias a slice of an owner.

``run_op`` / ``run_matmul`` / ``run_matmul_at`` / ``run_conv`` / ``run_pool``
mirror the static helpers the reference code generator emits
(_source.py:174-421): same names, same argument order, blocking until the
kernel is done.  They raise ``CormorantError`` where the reference helpers
(void) had no error path.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import CormorantError, check, lib


class CmBuf(C.Structure):
    """Layout of cm_buf_t in include/cormorant_cuda.h."""

    _fields_ = [("virt", C.c_void_p), ("dev", C.c_uint64), ("count", C.c_uint), ("refcount", C.c_uint),
                ("is_owner", C.c_uint), ("device", C.c_int)]


class InferenceBuf:
    BYTES_PER_ELEM = 2  # INFERENCE_BYTES_PER_ELEM for ap_fixed<16,8>

    def __init__(self, struct_ptr, keep=None):
        self._p = struct_ptr
        self._keep = keep          # owner kept alive by a view

    @classmethod
    def alloc(cls, n_elem: int) -> "InferenceBuf":
        p = lib().cm_buf_alloc(int(n_elem))
        if not p:
            raise CormorantError(-5, (lib().cm_last_error() or b"cm_buf_alloc failed").decode())
        return cls(C.cast(p, C.POINTER(CmBuf)))

    @classmethod
    def init_view(cls, base: "InferenceBuf", offset_elems: int, count_elems: int) -> "InferenceBuf":
        view = CmBuf()
        lib().cm_buf_init_view(C.byref(view), base._p, int(offset_elems), int(count_elems))
        obj = cls(C.pointer(view), keep=base)
        obj._struct = view
        return obj

    @property
    def handle(self):
        return self._p

    def ptr(self) -> np.ndarray:
        """The pinned host mirror as an int16 array (raw Q8.8 words)."""
        s = self._p.contents
        buf = (C.c_int16 * s.count).from_address(s.virt)
        return np.ctypeslib.as_array(buf)

    def phys(self) -> int:
        return int(self._p.contents.dev)

    def count(self) -> int:
        return int(self._p.contents.count)

    def sync_to_device(self) -> None:
        check(lib().cm_buf_sync_to_device(self._p))

    def sync_from_device(self) -> None:
        check(lib().cm_buf_sync_from_device(self._p))

    def retain(self) -> None:
        lib().cm_buf_retain(self._p)

    def release(self) -> None:
        lib().cm_buf_release(self._p)

    def free(self) -> None:
        if self._p is not None and self._keep is None:
            lib().cm_buf_free(self._p)
        self._p = None


def _dev(buf: InferenceBuf | None, off: int = 0) -> int | None:
    return None if buf is None else buf.phys() + off * InferenceBuf.BYTES_PER_ELEM


def run_op(a, b, c, size, op, outer, a_inc, b_inc) -> None:
    check(lib().cm_vectorop(_dev(a), _dev(b), _dev(c), size, op, outer, a_inc, b_inc))


def run_matmul(a, b, c, n, k, m, batch, a_stride, b_stride, c_stride) -> None:
    check(lib().cm_matmul(_dev(a), _dev(b), _dev(c), n, k, m, batch, a_stride, b_stride, c_stride))


def run_matmul_at(a, a_off, b, b_off, c, c_off, n, k, m, batch, a_stride, b_stride, c_stride) -> None:
    check(lib().cm_matmul(_dev(a, a_off), _dev(b, b_off), _dev(c, c_off), n, k, m, batch, a_stride, b_stride,
                          c_stride))


def run_conv(x, weight, bias, y, batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h, stride_w,
             dilation_h, dilation_w, pad_top, pad_left, has_bias, is_depthwise) -> None:
    check(lib().cm_conv(_dev(x), _dev(weight), _dev(bias), _dev(y), batch, in_ch, in_h, in_w, out_ch, out_h, out_w,
                        kh, kw, stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_left, has_bias,
                        is_depthwise))


def run_pool(x, y, batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h, stride_w, pad_top,
             pad_left, dil_h, dil_w, pool_type, lp_order, count_include_pad) -> None:
    check(lib().cm_pool(_dev(x), _dev(y), batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h,
                        stride_w, pad_top, pad_left, dil_h, dil_w, pool_type, lp_order, count_include_pad))
