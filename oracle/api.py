"""ctypes front end for the CPU checkers (test infrastructure only).

Both libraries take raw int16 Q8.8 buffers and the reference kernels'
argument lists (kernels/*/include/*.h); this module adds numpy plumbing.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
REF_DIR = ORACLE_DIR / "_ref"


def _reference_tree() -> Path | None:
    """Where the reference tree is: CM_REFERENCE_TREE, else the reference_path that
    BASELINE.json (the repository's description of its reference) records; None when
    neither names an existing directory."""
    loc = os.environ.get("CM_REFERENCE_TREE")
    if not loc:
        meta = ORACLE_DIR.parent / "BASELINE.json"
        if meta.exists():
            import json
            loc = json.loads(meta.read_text()).get("reference_path")
    return Path(loc) if loc and Path(loc).is_dir() else None


REFERENCE_TREE = _reference_tree()

_u = C.c_uint
_p16 = C.POINTER(C.c_int16)


def build(with_ref: bool | None = None) -> None:
    """Compile liboracle.so and, when the reference tree is present, _ref/."""
    targets = ["port"]
    if with_ref is None:
        with_ref = REFERENCE_TREE is not None and (REFERENCE_TREE / "kernels").is_dir()
    if with_ref:
        if REFERENCE_TREE is None:
            raise FileNotFoundError("the reference tree is not known: set CM_REFERENCE_TREE")
        targets += ["ref", "reftests"]
    cmd = ["make", "-s", "-C", str(ORACLE_DIR), *targets]
    if with_ref:
        cmd.insert(4, f"REF={REFERENCE_TREE}")
    subprocess.run(cmd, check=True)


def have_ref() -> bool:
    return all((REF_DIR / f"libref_{k}.so").exists() for k in ("vectorop", "matmul", "conv", "pool"))


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.dtype == np.int16 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_p16)


def _i16(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int16)


class _Checker:
    """Common numpy interface; subclasses bind the four kernel symbols."""

    name = "?"

    def vectorop(self, a, b, size, op, outer=1, a_inc=0, b_inc=0, c=None, c_len=None):
        a = _i16(a)
        b = None if b is None else _i16(b)
        if c is None:
            if c_len is None:
                c_len = (outer - 1) * (a_inc + b_inc) + size if outer else 0
            c = np.zeros(max(int(c_len), 1), np.int16)
        self._vop(_ptr(a), _ptr(b), _ptr(c), size, op, outer, a_inc, b_inc)
        return c

    def matmul(self, a, b, n, k, m, batch=1, a_bs=None, b_bs=None, c_bs=None, c=None):
        a, b = _i16(a), _i16(b)
        a_bs = n * k if a_bs is None else a_bs
        b_bs = k * m if b_bs is None else b_bs
        c_bs = n * m if c_bs is None else c_bs
        if c is None:
            c = np.zeros(max((batch - 1) * c_bs + n * m, 1), np.int16)
        self._mm(_ptr(a), _ptr(b), _ptr(c), n, k, m, batch, a_bs, b_bs, c_bs)
        return c

    def conv(self, x, w, bias, batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw,
             stride_h=1, stride_w=1, dil_h=1, dil_w=1, pad_top=0, pad_left=0,
             has_bias=None, is_depthwise=0, y=None):
        x, w = _i16(x), _i16(w)
        if has_bias is None:
            has_bias = int(bias is not None)
        bias_arr = _i16(bias) if bias is not None else np.zeros(max(out_ch, 1), np.int16)
        if y is None:
            y = np.zeros(max(batch * out_ch * out_h * out_w, 1), np.int16)
        self._conv(_ptr(x), _ptr(w), _ptr(bias_arr), _ptr(y), batch, in_ch, in_h, in_w, out_ch,
                   out_h, out_w, kh, kw, stride_h, stride_w, dil_h, dil_w, pad_top, pad_left,
                   has_bias, is_depthwise)
        return y

    def pool(self, x, batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h=1,
             stride_w=1, pad_top=0, pad_left=0, dil_h=1, dil_w=1, pool_type=0, lp_order=2,
             count_include_pad=0, y=None):
        x = _i16(x)
        if y is None:
            y = np.zeros(max(batch * channels * out_h * out_w, 1), np.int16)
        self._pool(_ptr(x), _ptr(y), batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w,
                   stride_h, stride_w, pad_top, pad_left, dil_h, dil_w, pool_type, lp_order,
                   count_include_pad)
        return y


def _bind(fn, nptr, nuint):
    fn.argtypes = [_p16] * nptr + [_u] * nuint
    fn.restype = None
    return fn


class Port(_Checker):
    """liboracle.so -- the C restatement (oracle/cm_oracle.c)."""

    name = "port"

    def __init__(self, path: Path):
        self.lib = lib = C.CDLL(str(path))
        self._vop = _bind(lib.orc_vectorop, 3, 5)
        self._mm = _bind(lib.orc_matmul, 3, 7)
        self._conv = _bind(lib.orc_conv, 4, 17)
        self._pool = _bind(lib.orc_pool, 2, 17)
        lib.orc_set_threads.argtypes = [C.c_int]
        lib.orc_get_threads.restype = C.c_int
        lib.orc_vectorop_scalar.argtypes = [_u, C.c_int16, C.c_int16]
        lib.orc_vectorop_scalar.restype = C.c_int16
        lib.orc_vectorop_check_pairs.argtypes = [_u, C.c_int32, _u, _p16, C.POINTER(C.c_int64)]
        lib.orc_vectorop_check_pairs.restype = C.c_uint64
        lib.orc_matmul_rows.argtypes = [_p16, _p16, _u, _u, _u, _u, _u, C.POINTER(C.c_uint32),
                                        C.POINTER(C.c_uint32), _u, _p16]
        lib.orc_conv_planes.argtypes = [_p16, _p16, _p16] + [_u] * 16 + [C.POINTER(C.c_uint32),
                                                                         C.POINTER(C.c_uint32), _u, _p16]

    def set_threads(self, n: int) -> None:
        self.lib.orc_set_threads(int(n))

    def threads(self) -> int:
        return int(self.lib.orc_get_threads())

    def scalar(self, op: int, a: int, b: int) -> int:
        return int(self.lib.orc_vectorop_scalar(op, a, b))

    def check_pairs(self, op: int, a_first: int, got: np.ndarray) -> tuple[int, int]:
        """Count mismatches of got[(a - a_first) * 65536 + b + 32768] against op(a, b)."""
        got = _i16(got)
        assert got.size % 65536 == 0
        first = C.c_int64(-1)
        bad = self.lib.orc_vectorop_check_pairs(op, a_first, got.size // 65536, _ptr(got), C.byref(first))
        return int(bad), int(first.value)

    def matmul_rows(self, a, b, n, k, m, a_bs, b_bs, bidx, ridx):
        a, b = _i16(a), _i16(b)
        bidx = np.ascontiguousarray(bidx, np.uint32)
        ridx = np.ascontiguousarray(ridx, np.uint32)
        out = np.zeros((len(bidx), m), np.int16)
        self.lib.orc_matmul_rows(_ptr(a), _ptr(b), n, k, m, a_bs, b_bs,
                                 bidx.ctypes.data_as(C.POINTER(C.c_uint32)),
                                 ridx.ctypes.data_as(C.POINTER(C.c_uint32)), len(bidx), _ptr(out))
        return out

    def conv_planes(self, x, w, bias, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h,
                    stride_w, dil_h, dil_w, pad_top, pad_left, has_bias, is_depthwise, nidx, midx):
        x, w = _i16(x), _i16(w)
        bias_arr = _i16(bias) if bias is not None else np.zeros(max(out_ch, 1), np.int16)
        nidx = np.ascontiguousarray(nidx, np.uint32)
        midx = np.ascontiguousarray(midx, np.uint32)
        out = np.zeros((len(nidx), out_h * out_w), np.int16)
        self.lib.orc_conv_planes(_ptr(x), _ptr(w), _ptr(bias_arr), in_ch, in_h, in_w, out_ch, out_h,
                                 out_w, kh, kw, stride_h, stride_w, dil_h, dil_w, pad_top, pad_left,
                                 has_bias, is_depthwise, nidx.ctypes.data_as(C.POINTER(C.c_uint32)),
                                 midx.ctypes.data_as(C.POINTER(C.c_uint32)), len(nidx), _ptr(out))
        return out


class Ref(_Checker):
    """_ref/libref_*.so -- the reference kernels compiled against the shims.

    The reference kernels keep function-static buffers and are not
    re-entrant: call them from one thread per process.
    """

    name = "ref"

    def __init__(self, d: Path):
        self._libs = {k: C.CDLL(str(d / f"libref_{k}.so")) for k in ("vectorop", "matmul", "conv", "pool")}
        self._vop = _bind(self._libs["vectorop"].cmref_vectorop, 3, 5)
        self._mm = _bind(self._libs["matmul"].cmref_matmul, 3, 7)
        self._conv = _bind(self._libs["conv"].cmref_conv, 4, 17)
        self._pool = _bind(self._libs["pool"].cmref_pool, 2, 17)
        self.max_k = int(self._libs["matmul"].cmref_matmul_max_k())
        self.max_kh = int(self._libs["conv"].cmref_conv_max_kh())
        self.max_pool = int(self._libs["pool"].cmref_pool_max_window())


_port: Port | None = None
_ref: Ref | None = None


def port() -> Port:
    global _port
    if _port is None:
        path = ORACLE_DIR / "liboracle.so"
        if not path.exists():
            build(with_ref=False)
        _port = Port(path)
    return _port


def ref() -> Ref:
    global _ref
    if _ref is None:
        if not have_ref():
            raise FileNotFoundError("oracle/_ref is not built (needs the reference tree)")
        _ref = Ref(REF_DIR)
    return _ref
