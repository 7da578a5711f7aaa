"""Mirror of the reference's generated host runtime for the four kernels.

``InferenceBuf`` mirrors ``inference_buf_t`` (inference-scheduler/src/codegen/
_buf_impl.py:25-236): an owner buffer is a device allocation plus a pinned host
mirror; ``phys()`` returns the device address the kernels are given (the
reference programs the DMA physical address); views alias a slice of an owner.

``run_op`` / ``run_matmul`` / ``run_matmul_at`` / ``run_conv`` / ``run_pool``
mirror the static helpers the reference code generator emits
(_source.py:174-421): same names, same argument order, blocking until the
kernel is done.  They raise ``CormorantError`` where the reference helpers
(void) had no error path.  An optional trailing ``stream`` enqueues the call on
that CUDA stream instead (the ``_async`` entry) and returns at once.
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

    def sync_to_device(self, stream=None) -> None:
        """Host mirror -> device.  With `stream` (a torch.cuda.Stream or a raw cudaStream_t
        address) the copy is enqueued there and the call returns at once."""
        if stream is None:
            check(lib().cm_buf_sync_to_device(self._p))
        else:
            check(lib().cm_buf_sync_to_device_async(self._p, _stream_ptr(stream)))

    def sync_from_device(self, stream=None) -> None:
        """Device -> host mirror; with `stream`, enqueued there (read the mirror after the
        stream has reached it)."""
        if stream is None:
            check(lib().cm_buf_sync_from_device(self._p))
        else:
            check(lib().cm_buf_sync_from_device_async(self._p, _stream_ptr(stream)))

    def retain(self) -> None:
        lib().cm_buf_retain(self._p)

    def release(self) -> None:
        lib().cm_buf_release(self._p)

    def free(self) -> None:
        if self._p is not None and self._keep is None:
            lib().cm_buf_free(self._p)
        self._p = None


def _stream_ptr(stream) -> int:
    return int(getattr(stream, "cuda_stream", stream) or 0)


def _dev(buf: InferenceBuf | None, off: int = 0) -> int | None:
    return None if buf is None else buf.phys() + off * InferenceBuf.BYTES_PER_ELEM


def run_op(a, b, c, size, op, outer, a_inc, b_inc, stream=None) -> None:
    args = (_dev(a), _dev(b), _dev(c), size, op, outer, a_inc, b_inc)
    check(lib().cm_vectorop(*args) if stream is None else lib().cm_vectorop_async(*args, _stream_ptr(stream)))


def run_matmul(a, b, c, n, k, m, batch, a_stride, b_stride, c_stride, stream=None) -> None:
    args = (_dev(a), _dev(b), _dev(c), n, k, m, batch, a_stride, b_stride, c_stride)
    check(lib().cm_matmul(*args) if stream is None else lib().cm_matmul_async(*args, _stream_ptr(stream)))


def run_matmul_at(a, a_off, b, b_off, c, c_off, n, k, m, batch, a_stride, b_stride, c_stride, stream=None) -> None:
    args = (_dev(a, a_off), _dev(b, b_off), _dev(c, c_off), n, k, m, batch, a_stride, b_stride, c_stride)
    check(lib().cm_matmul(*args) if stream is None else lib().cm_matmul_async(*args, _stream_ptr(stream)))


def run_conv(x, weight, bias, y, batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h, stride_w,
             dilation_h, dilation_w, pad_top, pad_left, has_bias, is_depthwise, stream=None) -> None:
    args = (_dev(x), _dev(weight), _dev(bias), _dev(y), batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw,
            stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_left, has_bias, is_depthwise)
    check(lib().cm_conv(*args) if stream is None else lib().cm_conv_async(*args, _stream_ptr(stream)))


def run_pool(x, y, batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h, stride_w, pad_top,
             pad_left, dil_h, dil_w, pool_type, lp_order, count_include_pad, stream=None) -> None:
    args = (_dev(x), _dev(y), batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h, stride_w,
            pad_top, pad_left, dil_h, dil_w, pool_type, lp_order, count_include_pad)
    check(lib().cm_pool(*args) if stream is None else lib().cm_pool_async(*args, _stream_ptr(stream)))


class CopyOverlap:
    """Runs calls shaped like the reference's inference_run() -- copy the inputs to
    the device, run the kernel, copy the outputs back (_source.py:643-791) -- with
    the copies of one call overlapping the kernels of the others.

    Input copies go on an upload stream and output copies on a download stream
    (host-to-device and device-to-host use separate copy engines), kernels run on
    the caller's stream, and CUDA events order every reuse of a buffer: an upload
    into a buffer waits for the last kernel that read it, a kernel writing a buffer
    waits for the last download of it.  Calls whose buffers are distinct overlap;
    calls that share a buffer are ordered.  Buffers are ``InferenceBuf`` objects; a
    view is the element range it aliases in its owner, so views of one owner that do
    not overlap (batch chunks of one large buffer) are independent, and a view and
    its owner are ordered.
    """

    @staticmethod
    def _range(b) -> tuple:
        """(owner identity, first element, end element) of the words `b` covers."""
        if b._keep is None:
            return id(b), 0, b.count()
        start = (b.phys() - b._keep.phys()) // InferenceBuf.BYTES_PER_ELEM
        return id(b._keep), start, start + b.count()

    @staticmethod
    def _record(table: dict, rng: tuple, event) -> None:
        entries = table.setdefault(rng[0], [])
        entries[:] = [e for e in entries if (e[0], e[1]) != (rng[1], rng[2])]
        entries.append((rng[1], rng[2], event))

    @staticmethod
    def _overlapping(table: dict, rng: tuple):
        return [ev for (s, e, ev) in table.get(rng[0], ()) if s < rng[2] and rng[1] < e]

    def __init__(self):
        import torch
        self._torch = torch
        self.up = torch.cuda.Stream()
        self.down = torch.cuda.Stream()
        self._read = {}      # owner -> [(start, end, event of the last kernel that read the range)]
        self._drained = {}   # owner -> [(start, end, event of the last download of the range)]

    def start(self, event) -> None:
        """Copies issued from now on start no earlier than `event` (a recorded CUDA event)."""
        self.up.wait_event(event)
        self.down.wait_event(event)

    def call(self, inputs, outputs, run) -> None:
        """Upload `inputs`, then `run(stream)` on the current stream, then download `outputs`."""
        torch = self._torch
        cur = torch.cuda.current_stream()
        for b in inputs:
            rng = self._range(b)
            # the last kernel that read the range, and the download of a result written there
            for ev in self._overlapping(self._read, rng) + self._overlapping(self._drained, rng):
                self.up.wait_event(ev)
            b.sync_to_device(self.up)
        up_done = torch.cuda.Event()
        up_done.record(self.up)
        cur.wait_event(up_done)
        for b in outputs:
            for ev in self._overlapping(self._drained, self._range(b)):
                cur.wait_event(ev)
        run(cur)
        ran = torch.cuda.Event()
        ran.record(cur)
        for b in inputs:
            self._record(self._read, self._range(b), ran)
        self.down.wait_event(ran)
        for b in outputs:
            b.sync_from_device(self.down)
        down_done = torch.cuda.Event()
        down_done.record(self.down)
        for b in outputs:
            self._record(self._drained, self._range(b), down_done)

    def join(self) -> None:
        """Make the current stream wait for every copy issued so far."""
        cur = self._torch.cuda.current_stream()
        cur.wait_stream(self.up)
        cur.wait_stream(self.down)
