"""Host-side mirror of the reference kernel interface.

The four functions keep the names, argument order and meaning of the
reference kernels (kernels/*/include/*.h) with buffers given as device int16
tensors (or raw device addresses as ints).  Without ``stream`` a call blocks
until the kernel is done, like the reference's Start + ``while (!IsDone)``
helpers (inference-scheduler/src/codegen/_source.py:208-217); with ``stream``
(a ``torch.cuda.Stream`` or a raw ``cudaStream_t`` int) it is enqueued and
returns at once.  Failures raise ``CormorantError``; there is no CPU path.
"""
from __future__ import annotations

from typing import Any

from ._lib import CormorantError, check, lib  # noqa: F401

OP_ADD, OP_SUB, OP_MUL, OP_DIV, OP_RELU, OP_RELU6 = range(6)   # VectorOP.h:50-57
POOL_MAX, POOL_AVG, POOL_LP = 0, 1, 2                          # pool Config.h.in:47-49


def _addr(t: Any) -> int | None:
    """Device address of a torch tensor (int16, CUDA) or a raw int; None stays None."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    if getattr(t, "is_cuda", False):
        if str(t.dtype) not in ("torch.int16", "torch.uint16"):
            raise TypeError(f"expected an int16 tensor, got {t.dtype}")
        return int(t.data_ptr())
    raise TypeError("buffers must be CUDA tensors or device addresses")


def _stream(s: Any) -> int | None:
    if s is None:
        return None
    if isinstance(s, int):
        return s
    return int(s.cuda_stream)


def init(instance: str | int = "0") -> None:
    """Select the device (X<Kernel>_Initialize analogue, _source.py:602-608)."""
    check(lib().cm_init(str(instance).encode()))


def release() -> None:
    check(lib().cm_release())


def synchronize(stream: Any = None) -> None:
    check(lib().cm_synchronize(_stream(stream)))


def launch_count() -> int:
    return int(lib().cm_launch_count())


def VectorOPKernel(a, b, c, size, op, outer=1, a_inc=0, b_inc=0, stream=None) -> None:
    """c[o*(a_inc+b_inc)+i] = op(a[o*a_inc+i], b[o*b_inc+i]) -- VectorOP.h:86-95."""
    L = lib()
    args = (_addr(a), _addr(b), _addr(c), size, op, outer, a_inc, b_inc)
    check(L.cm_vectorop(*args) if stream is None else L.cm_vectorop_async(*args, _stream(stream)))


def MatmulKernel(a, b, c, n, k, m, batch=1, a_batch_stride=None, b_batch_stride=None, c_batch_stride=None,
                 stream=None) -> None:
    """Batched Q8.8 GEMM C[n][m] = A[n][k] x B[k][m] -- MatmulKernel.h:68-79.

    Omitted strides default to the dense packing (n*k, k*m, n*m)."""
    a_bs = n * k if a_batch_stride is None else a_batch_stride
    b_bs = k * m if b_batch_stride is None else b_batch_stride
    c_bs = n * m if c_batch_stride is None else c_batch_stride
    L = lib()
    args = (_addr(a), _addr(b), _addr(c), n, k, m, batch, a_bs, b_bs, c_bs)
    check(L.cm_matmul(*args) if stream is None else L.cm_matmul_async(*args, _stream(stream)))


def ConvKernel(x, weight, bias, y, batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h=1,
               stride_w=1, dilation_h=1, dilation_w=1, pad_top=0, pad_left=0, has_bias=None, is_depthwise=0,
               stream=None) -> None:
    """NCHW 2-D convolution -- ConvKernel.h:79-101."""
    if has_bias is None:
        has_bias = int(bias is not None)
    L = lib()
    args = (_addr(x), _addr(weight), _addr(bias), _addr(y), batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw,
            stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_left, int(has_bias), int(is_depthwise))
    check(L.cm_conv(*args) if stream is None else L.cm_conv_async(*args, _stream(stream)))


EPI_NONE, EPI_RELU, EPI_ADD, EPI_ADD_RELU = 0, 1, 2, 3
EPI_NHWC = 8    # ConvKernelPlanes / ConvKernelPrepared: y channels-last [batch][out_h][out_w][out_ch]


def ConvKernelFused(x, weight, bias, y, batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h=1,
                    stride_w=1, dilation_h=1, dilation_w=1, pad_top=0, pad_left=0, has_bias=None, is_depthwise=0,
                    epilogue=EPI_RELU, resid=None, stream=None) -> None:
    """ConvKernel followed by VectorOP ADD (with `resid`) and/or RELU, fused into the conv's
    epilogue (cm_conv_fused).  Not a reference kernel: the word-for-word result of the
    reference call sequence Conv -> [Add(resid)] -> [Relu]."""
    if has_bias is None:
        has_bias = int(bias is not None)
    L = lib()
    args = (_addr(x), _addr(weight), _addr(bias), _addr(y), batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw,
            stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_left, int(has_bias), int(is_depthwise),
            int(epilogue), _addr(resid))
    check(L.cm_conv_fused(*args) if stream is None else L.cm_conv_fused_async(*args, _stream(stream)))


def ConvPoolKernel(x, weight, bias, y, conv_args, epilogue, resid, pool_args, stream=None) -> None:
    """ConvKernel (+ the fused epilogue) followed by a MAX PoolingKernel of its output in one
    launch (cm_conv_pool): conv_args are the conv's 17 scalars, pool_args the pool's 17
    (cm_pool's order); y receives the pool's output.  Not a reference kernel: the words of
    Conv -> [Add] -> [Relu] -> MaxPool."""
    L = lib()
    args = ((_addr(x), _addr(weight), _addr(bias), _addr(y)) + tuple(int(v) for v in conv_args)
            + (int(epilogue), _addr(resid)) + tuple(int(v) for v in pool_args))
    check(L.cm_conv_pool(*args) if stream is None else L.cm_conv_pool_async(*args, _stream(stream)))


class PlaneImage:
    """A conv input held as channels-last int8 hi/lo planes with its padding frame
    (cm_planes_create): written by a producing conv's GEMM epilogue, read in place of
    the NCHW tensor by implicit-GEMM convs.  Not a reference object."""

    def __init__(self, batch, channels, h, w, frame=(0, 0, 0, 0)):
        self.shape = (int(batch), int(channels), int(h), int(w))
        self.frame = tuple(int(f) for f in frame)
        self.ptr = lib().cm_planes_create(*self.shape, *self.frame)
        if not self.ptr:
            msg = lib().cm_last_error()
            raise CormorantError(-5, (msg or b"cm_planes_create failed").decode(errors="replace"))

    def close(self) -> None:
        if getattr(self, "ptr", None):
            lib().cm_planes_destroy(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def conv_plane_frame(batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h=1, stride_w=1, dilation_h=1,
                     dilation_w=1, pad_top=0, pad_left=0, has_bias=1, is_depthwise=0):
    """The padding frame (top, left, bottom, right) a conv with these arguments needs
    in a PlaneImage it reads, or None when it reads its NCHW input instead."""
    import ctypes as C
    fr = (C.c_uint * 4)()
    ok = lib().cm_conv_plane_frame(batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h, stride_w,
                                   dilation_h, dilation_w, pad_top, pad_left, int(has_bias), int(is_depthwise), fr)
    return tuple(int(v) for v in fr) if ok else None


def conv_writes_nhwc(batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h=1, stride_w=1, dilation_h=1,
                     dilation_w=1, pad_top=0, pad_left=0, has_bias=1, is_depthwise=0) -> bool:
    """Whether a conv with these arguments can write a channels-last y (EPI_NHWC)."""
    return bool(lib().cm_conv_writes_nhwc(batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h, stride_w,
                                          dilation_h, dilation_w, pad_top, pad_left, int(has_bias), int(is_depthwise)))


def PlanesFill(planes, x, stream=None) -> None:
    """Split the NCHW tensor x into plane image `planes` (cm_planes_fill)."""
    L = lib()
    check(L.cm_planes_fill(planes.ptr, _addr(x)) if stream is None
          else L.cm_planes_fill_async(planes.ptr, _addr(x), _stream(stream)))


def PoolingKernelPlanes(xp, yp, batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h=1, stride_w=1,
                        pad_top=0, pad_left=0, dil_h=1, dil_w=1, pool_type=POOL_MAX, lp_order=2, count_include_pad=0,
                        stream=None) -> None:
    """PoolingKernel (MAX only) from plane image xp to plane image yp (cm_pool_planes)."""
    L = lib()
    args = (_planes(xp), _planes(yp), batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h, stride_w,
            pad_top, pad_left, dil_h, dil_w, pool_type, lp_order, count_include_pad)
    check(L.cm_pool_planes(*args) if stream is None else L.cm_pool_planes_async(*args, _stream(stream)))


def PoolingKernelNhwc(x, y, batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h=1, stride_w=1,
                      pad_top=0, pad_left=0, dil_h=1, dil_w=1, pool_type=POOL_MAX, lp_order=2, count_include_pad=0,
                      stream=None) -> None:
    """PoolingKernel's global pools on a channels-last tensor x [batch][in_h][in_w][channels]
    (a conv output written under EPI_NHWC); y [batch][channels] (cm_pool_nhwc)."""
    L = lib()
    args = (_addr(x), _addr(y), batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h, stride_w,
            pad_top, pad_left, dil_h, dil_w, pool_type, lp_order, count_include_pad)
    check(L.cm_pool_nhwc(*args) if stream is None else L.cm_pool_nhwc_async(*args, _stream(stream)))


def PoolingKernelNhwcPlanes(x, yp, batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h=1, stride_w=1,
                            pad_top=0, pad_left=0, dil_h=1, dil_w=1, pool_type=POOL_MAX, stream=None) -> None:
    """PoolingKernel (MAX only) from a channels-last tensor x [batch][in_h][in_w][channels]
    (a conv output written under EPI_NHWC) to plane image yp (cm_pool_nhwc_planes)."""
    L = lib()
    args = (_addr(x), _planes(yp), batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h, stride_w,
            pad_top, pad_left, dil_h, dil_w, pool_type)
    check(L.cm_pool_nhwc_planes(*args) if stream is None else L.cm_pool_nhwc_planes_async(*args, _stream(stream)))


CALL_VECTOROP, CALL_MATMUL, CALL_CONV, CALL_POOL = 0, 1, 2, 3
CALLS_MAX = 24


def _call_struct():
    import ctypes as C

    class CmCall(C.Structure):                       # cm_call_t (include/cormorant_cuda.h)
        _fields_ = [("kind", C.c_uint), ("epilogue", C.c_uint), ("in0", C.c_void_p), ("in1", C.c_void_p),
                    ("in2", C.c_void_p), ("resid", C.c_void_p), ("out", C.c_void_p), ("args", C.c_uint * 17)]
    return CmCall


_CmCall = None


def call_array(calls):
    """A cm_call_t array from (kind, epilogue, in0, in1, in2, resid, out, args) tuples
    (buffers as tensors or device addresses)."""
    global _CmCall
    if _CmCall is None:
        _CmCall = _call_struct()
    arr = (_CmCall * len(calls))()
    for d, (kind, epi, in0, in1, in2, resid, out, args) in zip(arr, calls):
        d.kind, d.epilogue = int(kind), int(epi)
        d.in0, d.in1, d.in2, d.resid, d.out = _addr(in0), _addr(in1), _addr(in2), _addr(resid), _addr(out)
        for k, v in enumerate(args):
            d.args[k] = int(v)
    return arr


def calls_supported(arr) -> bool:
    return bool(lib().cm_calls_supported(arr, len(arr)))


def RunCalls(arr, stream=None) -> None:
    """The whole small call list in one launch (cm_calls)."""
    L = lib()
    check(L.cm_calls(arr, len(arr)) if stream is None else L.cm_calls_async(arr, len(arr), _stream(stream)))


def _planes(p) -> int | None:
    return None if p is None else p.ptr


def ConvKernelPlanes(x, xp, weight, bias, y, yp, batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h=1,
                     stride_w=1, dilation_h=1, dilation_w=1, pad_top=0, pad_left=0, has_bias=None, is_depthwise=0,
                     epilogue=EPI_NONE, resid=None, resid_planes=None, stream=None) -> None:
    """ConvKernelFused with plane images (cm_conv_planes): `xp` (a PlaneImage or None)
    is read instead of `x` when this conv can; `yp` receives the output, and `y` may
    then be None; `resid_planes` (a PlaneImage of the output's shape) supplies the
    residual instead of `resid` when this conv reads plane images."""
    if has_bias is None:
        has_bias = int(bias is not None)
    L = lib()
    args = (_addr(x), _planes(xp), _addr(weight), _addr(bias), _addr(y), _planes(yp), batch, in_ch, in_h, in_w,
            out_ch, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_left,
            int(has_bias), int(is_depthwise), int(epilogue), _addr(resid), _planes(resid_planes))
    check(L.cm_conv_planes(*args) if stream is None else L.cm_conv_planes_async(*args, _stream(stream)))


class ConvWeights:
    """Conv weights prepared once for one call geometry (cm_conv_weights_create): the
    weight planes and column terms the tensor-core paths read, so repeated calls with
    constant weights (a network's parameters) skip that preparation.  `weight` and `bias`
    must keep the values they had at creation and stay allocated.  Not a reference
    object."""

    def __init__(self, weight, bias, batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h=1, stride_w=1,
                 dilation_h=1, dilation_w=1, pad_top=0, pad_left=0, has_bias=None, is_depthwise=0):
        import ctypes as C
        if has_bias is None:
            has_bias = int(bias is not None)
        self.geometry = (batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h,
                         dilation_w, pad_top, pad_left, int(has_bias), int(is_depthwise))
        self._keep = (weight, bias)            # the buffers the prepared calls still read
        out = C.c_void_p()
        self.ptr = None
        check(lib().cm_conv_weights_create(_addr(weight), _addr(bias), *self.geometry, C.byref(out)))
        self.ptr = out.value

    def close(self) -> None:
        if getattr(self, "ptr", None):
            lib().cm_conv_weights_destroy(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ConvKernelPrepared(w, x, xp, y, yp, epilogue=EPI_NONE, resid=None, resid_planes=None, stream=None) -> None:
    """The conv of ConvWeights `w`'s geometry (cm_conv_prepared): cm_conv_planes' inputs,
    outputs and epilogue, without the per-call weight preparation."""
    L = lib()
    args = (w.ptr, _addr(x), _planes(xp), _addr(y), _planes(yp), int(epilogue), _addr(resid), _planes(resid_planes))
    check(L.cm_conv_prepared(*args) if stream is None else L.cm_conv_prepared_async(*args, _stream(stream)))


class MatmulWeights:
    """A MatMul B operand (k x m, broadcast over the batch) prepared once
    (cm_matmul_weights_create): its planes and column terms, so repeated calls with constant
    weights (a network's Gemm) skip that preparation.  `b` must keep the values it had at
    creation and stay allocated.  Not a reference object."""

    def __init__(self, b, k, m):
        import ctypes as C
        self.k, self.m = int(k), int(m)
        self._keep = b                          # the buffer the other paths still read
        out = C.c_void_p()
        self.ptr = None
        check(lib().cm_matmul_weights_create(_addr(b), self.k, self.m, C.byref(out)))
        self.ptr = out.value

    def close(self) -> None:
        if getattr(self, "ptr", None):
            lib().cm_matmul_weights_destroy(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def MatmulKernelPrepared(w, a, c, n, batch=1, a_batch_stride=None, c_batch_stride=None, epilogue=EPI_NONE, bias=None,
                         stream=None) -> None:
    """MatmulKernelFused(a, B, c, n, w.k, w.m, batch, a_bs, 0, c_bs, epilogue, bias) with the
    MatmulWeights `w` of B (cm_matmul_prepared): the same words, without the per-call split
    of B."""
    a_bs = n * w.k if a_batch_stride is None else a_batch_stride
    c_bs = n * w.m if c_batch_stride is None else c_batch_stride
    L = lib()
    args = (w.ptr, _addr(a), _addr(c), n, batch, a_bs, c_bs, int(epilogue), _addr(bias))
    check(L.cm_matmul_prepared(*args) if stream is None else L.cm_matmul_prepared_async(*args, _stream(stream)))


def MatmulKernelFused(a, b, c, n, k, m, batch=1, a_batch_stride=None, b_batch_stride=None, c_batch_stride=None,
                      epilogue=EPI_ADD, bias=None, stream=None) -> None:
    """MatmulKernel followed by VectorOP ADD of a bias row broadcast over the n rows
    (size m, outer n, a_inc m, b_inc 0) and/or RELU, fused into the GEMM's epilogue
    (cm_matmul_fused).  Not a reference kernel: the word-for-word result of the
    scheduler's Gemm decomposition MatMul -> Add(bias) (graph.py:83-188) -> [Relu]."""
    a_bs = n * k if a_batch_stride is None else a_batch_stride
    b_bs = k * m if b_batch_stride is None else b_batch_stride
    c_bs = n * m if c_batch_stride is None else c_batch_stride
    L = lib()
    args = (_addr(a), _addr(b), _addr(c), n, k, m, batch, a_bs, b_bs, c_bs, int(epilogue), _addr(bias))
    check(L.cm_matmul_fused(*args) if stream is None else L.cm_matmul_fused_async(*args, _stream(stream)))


def PoolingKernel(x, y, batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h=1, stride_w=1,
                  pad_top=0, pad_left=0, dil_h=1, dil_w=1, pool_type=POOL_MAX, lp_order=2, count_include_pad=0,
                  stream=None) -> None:
    """Max / Average / Lp pooling and their Global variants -- PoolingKernel.h:63-83."""
    L = lib()
    args = (_addr(x), _addr(y), batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h, stride_w,
            pad_top, pad_left, dil_h, dil_w, pool_type, lp_order, count_include_pad)
    check(L.cm_pool(*args) if stream is None else L.cm_pool_async(*args, _stream(stream)))
