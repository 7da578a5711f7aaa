"""Kernel-argument derivation of the reference's inference scheduler, restated.

The reference compiles an ONNX graph into run_op / run_matmul / run_matmul_at /
run_conv / run_pool calls over one buffer pool (inference-scheduler/src/graph.py,
src/nodes.py, src/codegen/_core.py).  This module takes the same graph -- tensors
with shapes and constant data, operators with their ONNX attributes -- in a plain
form (the `onnx` package is not needed) and derives the same calls, argument for
argument, as a `networks.Net` call list:

* Gemm (alpha = beta = 1, no transposes) -> MatMul + Add(bias)      graph.py:83-188
* Reshape / Squeeze / Unsqueeze / Dropout -> alias of the input     nodes.py:1426-1493
* Add / Sub / Mul / Div / Relu / Clip(0, 6) -> VectorOPKernel, one input broadcast
  over an outer loop whose chunk stride is rounded up to the 16-byte alignment
                                                      nodes.py:151-227, 320-400, 414-453
* MatMul -> MatmulKernel: 2-D, batched, either side broadcast, the 4-D x 3-D outer
  loop (run_matmul_at) and the row-strided form for gapped buffers
                                                      nodes.py:524-755, 771-821
* Conv -> ConvKernel: pads / auto_pad, dilations, group 1 or depthwise
                                                      nodes.py:896-1080, 1103-1119
* MaxPool / AveragePool / LpPool and their Global forms -> PoolingKernel
                                                      nodes.py:1205-1377, 1404-1418
* buffer layouts with alignment gaps, in three phases  codegen/_core.py:75-249

Shapes of intermediate tensors come from `infer_shapes` (the role ONNX shape
inference plays for the reference).  Constant data are raw Q8.8 words (int16).
`derive(graph)` returns the Net: node tuples are the calls, buffer sizes are the
layouts' allocations (alignment gaps included), constants are laid out in their
buffers' layouts (gap words zero).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .networks import Net

OP_ADD, OP_SUB, OP_MUL, OP_DIV, OP_RELU, OP_RELU6 = 0, 1, 2, 3, 4, 5
POOL_MAX, POOL_AVG, POOL_LP = 0, 1, 2
ALIGN_ELEMS = 8          # 16-byte alignment / 2-byte words (nodes.py _ALIGN_BYTES)

_VECTOROPS = {"Add": (OP_ADD, 2), "Sub": (OP_SUB, 2), "Mul": (OP_MUL, 2), "Div": (OP_DIV, 2),
              "Relu": (OP_RELU, 1), "Clip": (OP_RELU6, 1)}
_POOLS = {"MaxPool": POOL_MAX, "AveragePool": POOL_AVG, "LpPool": POOL_LP,
          "GlobalMaxPool": POOL_MAX, "GlobalAveragePool": POOL_AVG, "GlobalLpPool": POOL_LP}
_ALIASES = ("Reshape", "Squeeze", "Unsqueeze", "Dropout")


class SchedulerError(ValueError):
    """The graph cannot be mapped onto the four kernels (same conditions as the reference)."""


@dataclass
class Tensor:
    name: str
    shape: tuple
    data: np.ndarray | None = None      # raw Q8.8 words (int16) of a constant; int64 for shape tensors

    @property
    def numel(self) -> int:
        return max(int(np.prod(self.shape, dtype=np.int64)) if len(self.shape) else 1, 1)

    @property
    def is_const(self) -> bool:
        return self.data is not None


@dataclass
class Op:
    op_type: str
    inputs: list
    outputs: list
    attrs: dict = field(default_factory=dict)
    name: str = ""


@dataclass
class Graph:
    name: str
    tensors: dict = field(default_factory=dict)   # name -> Tensor
    ops: list = field(default_factory=list)
    inputs: list = field(default_factory=list)
    outputs: list = field(default_factory=list)

    def add(self, name: str, shape, data=None) -> str:
        self.tensors[name] = Tensor(name, tuple(int(d) for d in shape), data)
        return name

    def op(self, op_type: str, inputs, outputs, **attrs) -> None:
        self.ops.append(Op(op_type, list(inputs), list(outputs), dict(attrs), f"{op_type}_{len(self.ops)}"))


# ----------------------------------------------------------------------------------
# shape inference (what ONNX shape inference provides the reference)
# ----------------------------------------------------------------------------------
def _window_out(n: int, k: int, s: int, d: int, p0: int, p1: int, auto_pad: str) -> int:
    if auto_pad in ("SAME_UPPER", "SAME_LOWER"):
        return -(-n // s)
    if auto_pad == "VALID":
        return -(-(n - d * (k - 1)) // s)
    return (n + p0 + p1 - d * (k - 1) - 1) // s + 1


def _broadcast_shape(a, b):
    out = []
    for i in range(max(len(a), len(b))):
        x = a[len(a) - 1 - i] if i < len(a) else 1
        y = b[len(b) - 1 - i] if i < len(b) else 1
        if x != y and x != 1 and y != 1:
            raise SchedulerError(f"shapes {list(a)} and {list(b)} do not broadcast")
        out.append(max(x, y))
    return tuple(reversed(out))


def infer_shapes(g: Graph) -> None:
    """Give every operator output a shape (in place), in operator order."""
    T = g.tensors
    for op in g.ops:
        if op.outputs[0] in T:
            continue
        t = op.op_type
        x = T[op.inputs[0]].shape
        a = op.attrs
        if t in ("Add", "Sub", "Mul", "Div"):
            s = _broadcast_shape(x, T[op.inputs[1]].shape)
        elif t in ("Relu", "Clip", "Dropout"):
            s = x
        elif t == "MatMul":
            b = T[op.inputs[1]].shape
            s = _broadcast_shape(x[:-2], b[:-2]) + (x[-2], b[-1])
        elif t == "Gemm":
            s = (x[0], T[op.inputs[1]].shape[1])
        elif t in ("Conv", "MaxPool", "AveragePool", "LpPool"):
            if t == "Conv":
                w = T[op.inputs[1]].shape
                ch, kh, kw = w[0], w[2], w[3]
            else:
                ch, (kh, kw) = x[1], a["kernel_shape"]
            sh, sw = a.get("strides", (1, 1))
            dh, dw = a.get("dilations", (1, 1))
            p = a.get("pads", (0, 0, 0, 0))
            ap = a.get("auto_pad", "NOTSET")
            s = (x[0], ch, _window_out(x[2], kh, sh, dh, p[0], p[2], ap), _window_out(x[3], kw, sw, dw, p[1], p[3], ap))
        elif t.startswith("Global"):
            s = (x[0], x[1], 1, 1)
        elif t == "Reshape":
            spec = list(a["shape"]) if "shape" in a else [int(v) for v in T[op.inputs[1]].data]
            total = int(np.prod(x))
            spec = [x[i] if v == 0 else v for i, v in enumerate(spec)]
            if -1 in spec:
                known = int(np.prod([v for v in spec if v != -1]))
                spec[spec.index(-1)] = total // known
            s = tuple(spec)
        elif t == "Squeeze":
            axes = [ax % len(x) for ax in a.get("axes", [i for i, d in enumerate(x) if d == 1])]
            s = tuple(d for i, d in enumerate(x) if i not in axes)
        elif t == "Unsqueeze":
            s = list(x)
            for ax in sorted(ax % (len(x) + len(a["axes"])) for ax in a["axes"]):
                s.insert(ax, 1)
            s = tuple(s)
        else:
            raise SchedulerError(f"no shape rule for {t}")
        g.add(op.outputs[0], s)


# ----------------------------------------------------------------------------------
# resolved nodes
# ----------------------------------------------------------------------------------
@dataclass
class _Node:
    kind: str                 # vectorop | matmul | conv | pool | alias
    op: Op
    inputs: list              # Tensors read (vectorop: after Clip's bound inputs are dropped)
    output: Tensor
    # vectorop
    code: int = 0
    arity: int = 1
    outer: int = 1
    chunk: int = 0
    stride: int = 0           # chunk rounded up to the alignment
    a_adv: bool = True
    b_adv: bool = True
    # matmul
    mm: tuple = ()            # n, k, m, batch, a_bs, b_bs, c_bs
    mm_outer: tuple = ()      # outer_count, a_os, b_os, c_os
    # conv / pool: the 17 kernel scalars
    args: tuple = ()


def _broadcast_info(t: Tensor, out: Tensor, ae: int):
    """(outer, chunk, aligned chunk, advances) of t against the output (nodes.py:151-227):
    t equal to the output strides through it; a smaller t repeats, its shape right-aligned
    to the output's with the size-1 dimensions forming one leading block."""
    if t.numel == out.numel:
        return 1, out.numel, out.numel, True
    if out.numel % t.numel:
        raise SchedulerError(f"'{t.name}' ({t.numel} elements) does not divide '{out.name}' ({out.numel})")
    ts = (1,) * (len(out.shape) - len(t.shape)) + tuple(t.shape)
    matched = False
    for td, od in zip(ts, out.shape):
        if td == od:
            matched = True
        elif td == 1:
            if matched:
                raise SchedulerError(f"'{t.name}' {list(t.shape)}: broadcast dimensions must lead")
        else:
            raise SchedulerError(f"'{t.name}' {list(t.shape)} does not broadcast to {list(out.shape)}")
    return out.numel // t.numel, t.numel, (t.numel + ae - 1) & ~(ae - 1), False


def _vectorop(op: Op, T: dict, ae: int) -> _Node:
    code, arity = _VECTOROPS[op.op_type]
    ins = [T[n] for n in op.inputs if n]
    out = T[op.outputs[0]]
    if op.op_type == "Clip":
        lo, hi = op.attrs.get("min"), op.attrs.get("max")
        if lo is None and len(ins) > 1 and ins[1].is_const:
            lo = float(ins[1].data.reshape(-1)[0]) / 256.0
        if hi is None and len(ins) > 2 and ins[2].is_const:
            hi = float(ins[2].data.reshape(-1)[0]) / 256.0
        if lo != 0.0 or hi != 6.0:
            raise SchedulerError(f"Clip({lo}, {hi}): only Clip(0, 6) maps to RELU6")
        ins = ins[:1]
    if len(ins) != arity:
        raise SchedulerError(f"{op.op_type} takes {arity} input(s), got {len(ins)}")
    nd = _Node("vectorop", op, ins, out, code=code, arity=arity)
    if arity == 1:
        if ins[0].numel != out.numel:
            raise SchedulerError(f"{op.op_type}: {ins[0].numel} elements in, {out.numel} out")
        nd.outer, nd.chunk, nd.stride = 1, out.numel, out.numel
        return nd
    ao, _, _, a_adv = _broadcast_info(ins[0], out, ae)
    bo, _, _, b_adv = _broadcast_info(ins[1], out, ae)
    if not a_adv and not b_adv:
        raise SchedulerError(f"{op.op_type}: only one input may broadcast")
    nd.outer = max(ao, bo)
    nd.chunk = out.numel // nd.outer
    nd.stride = (nd.chunk + ae - 1) & ~(ae - 1)
    nd.a_adv, nd.b_adv = a_adv, b_adv
    return nd


def _prod(dims) -> int:
    p = 1
    for d in dims:
        p *= d
    return p


def _matmul(op: Op, T: dict) -> _Node:
    A, B, Y = T[op.inputs[0]], T[op.inputs[1]], T[op.outputs[0]]
    sa, sb = tuple(A.shape), tuple(B.shape)
    if not (2 <= len(sa) <= 5 and 2 <= len(sb) <= 5):
        raise SchedulerError(f"MatMul rank 2-5 only: {list(sa)} @ {list(sb)}")
    n, k, m = sa[-2], sa[-1], sb[-1]
    if sb[-2] != k:
        raise SchedulerError(f"MatMul inner sizes {k} and {sb[-2]} differ")
    ab, bb = sa[:-2], sb[:-2]
    nd = _Node("matmul", op, [A, B], Y)
    nd.mm_outer = (1, 0, 0, 0)
    if not ab and not bb:
        nd.mm = (n, k, m, 1, 0, 0, 0)
    elif not bb:
        nd.mm = (n, k, m, _prod(ab), n * k, 0, n * m)
    elif not ab:
        nd.mm = (n, k, m, _prod(bb), 0, k * m, n * m)
    else:
        L = max(len(ab), len(bb))
        ae, be = (1,) * (L - len(ab)) + ab, (1,) * (L - len(bb)) + bb
        ob = []
        for x, y in zip(ae, be):
            if x != y and x != 1 and y != 1:
                raise SchedulerError(f"MatMul batch dims {list(ab)} and {list(bb)} do not broadcast")
            ob.append(max(x, y))
        # leading dims where exactly one side is 1 drive an outer loop; the rest are the
        # kernel's own batch loop
        a_drives, split = None, L
        for i, (x, y) in enumerate(zip(ae, be)):
            if (x > 1 and y > 1) or (x == 1 and y == 1):
                split = i
                break
            if a_drives is None:
                a_drives = x > 1
            elif a_drives != (x > 1):
                raise SchedulerError("MatMul outer broadcast in both directions")
        outer, batch = _prod(ob[:split]), _prod(ob[split:])
        if batch <= 1:
            strides = (0, 0, 0)
        else:
            strides = (n * k if any(ae[i] > 1 for i in range(split, L)) else 0,
                       k * m if any(be[i] > 1 for i in range(split, L)) else 0, n * m)
        nd.mm = (n, k, m, batch) + strides
        if outer > 1:
            nd.mm_outer = (outer, batch * n * k if a_drives else 0, 0 if a_drives else batch * k * m, batch * n * m)
    return nd


def _pads(a: dict, kh: int, kw: int, sh: int, sw: int, dh: int, dw: int, x, y):
    ap = a.get("auto_pad", "NOTSET")
    if ap == "NOTSET":
        p = list(a.get("pads", (0, 0, 0, 0)))
        return (p[0] if len(p) > 0 else 0), (p[1] if len(p) > 1 else 0)
    if ap == "VALID":
        return 0, 0
    if ap in ("SAME_UPPER", "SAME_LOWER"):
        ph = max(0, (y[2] - 1) * sh + dh * (kh - 1) + 1 - x[2])
        pw = max(0, (y[3] - 1) * sw + dw * (kw - 1) + 1 - x[3])
        if ap == "SAME_UPPER":
            return ph // 2, pw // 2
        return (ph + 1) // 2, (pw + 1) // 2
    raise SchedulerError(f"auto_pad '{ap}' is not supported")


def _conv(op: Op, T: dict) -> _Node:
    names = [n for n in op.inputs if n]
    if len(names) not in (2, 3):
        raise SchedulerError("Conv takes 2 or 3 inputs")
    X, W, Y = T[op.inputs[0]], T[op.inputs[1]], T[op.outputs[0]]
    bias = T[op.inputs[2]] if len(op.inputs) > 2 and op.inputs[2] else None
    if len(X.shape) != 4 or len(W.shape) != 4 or len(Y.shape) != 4:
        raise SchedulerError("Conv: 4-D input, weight and output only")
    nb, c, h, w = X.shape
    m, cw, kh, kw = W.shape
    group = op.attrs.get("group", 1)
    if group == 1:
        dw_ = 0
        if cw != c:
            raise SchedulerError(f"Conv weight channels {cw} != input channels {c}")
    elif group == c:
        dw_ = 1
        if cw != 1 or m != c:
            raise SchedulerError("depthwise Conv needs weight [C, 1, kh, kw]")
    else:
        raise SchedulerError(f"grouped Conv (group={group}) is not supported")
    if m != Y.shape[1]:
        raise SchedulerError("Conv output channels differ from the weight's")
    sh, sw = op.attrs.get("strides", (1, 1))
    dh, dw = op.attrs.get("dilations", (1, 1))
    pt, pl = _pads(op.attrs, kh, kw, sh, sw, dh, dw, X.shape, Y.shape)
    ins = [X, W] + ([bias] if bias is not None else [])
    return _Node("conv", op, ins, Y, args=(nb, c, h, w, m, Y.shape[2], Y.shape[3], kh, kw, sh, sw, dh, dw, pt, pl,
                                           int(bias is not None), dw_))


def _pool(op: Op, T: dict) -> _Node:
    X, Y = T[op.inputs[0]], T[op.outputs[0]]
    if len(X.shape) != 4 or len(Y.shape) != 4:
        raise SchedulerError("pooling: 4-D input and output only")
    nb, c, h, w = X.shape
    kind = _POOLS[op.op_type]
    a = op.attrs
    if op.op_type.startswith("Global"):
        ph, pw, sh, sw, pt, pl, dh, dw = h, w, 1, 1, 0, 0, 1, 1
    else:
        ks = list(a.get("kernel_shape", ()))
        if len(ks) != 2:
            raise SchedulerError("pooling: 2-D kernel_shape only")
        ph, pw = ks
        sh, sw = a.get("strides", (1, 1))
        dl = list(a.get("dilations", (1, 1)))
        dh, dw = (dl[0] if dl else 1), (dl[1] if len(dl) > 1 else 1)
        pt, pl = _pads(a, ph, pw, sh, sw, dh, dw, X.shape, Y.shape)
        if a.get("ceil_mode", 0):
            raise SchedulerError("pooling: ceil_mode = 1 is not supported")
    p = a.get("p", 2) if kind == POOL_LP else 2
    if kind == POOL_LP and p not in (1, 2):
        raise SchedulerError(f"LpPool p = {p}: only 1 and 2")
    cip = a.get("count_include_pad", 0) if kind == POOL_AVG else 0
    return _Node("pool", op, [X], Y, args=(nb, c, h, w, Y.shape[2], Y.shape[3], ph, pw, sh, sw, pt, pl, dh, dw,
                                           kind, p, cip))


def _decompose_gemm(g: Graph) -> list:
    """Gemm(A, B[, C]) -> MatMul(A, B) -> tmp, then Add(tmp, C); without C the MatMul
    writes Y.  alpha, beta other than 1 or a transpose are refused (graph.py:83-188)."""
    ops, count = [], 0
    for op in g.ops:
        if op.op_type != "Gemm":
            ops.append(op)
            continue
        a = op.attrs
        if abs(a.get("alpha", 1.0) - 1.0) > 1e-6 or abs(a.get("beta", 1.0) - 1.0) > 1e-6:
            raise SchedulerError("Gemm: only alpha = beta = 1")
        if a.get("transA", 0) or a.get("transB", 0):
            raise SchedulerError("Gemm: no transposed operands")
        count += 1
        A, B = op.inputs[0], op.inputs[1]
        C = op.inputs[2] if len(op.inputs) > 2 and op.inputs[2] else None
        Y = op.outputs[0]
        if C:
            tmp = f"_gemm_mm_out_{count}"
            g.add(tmp, tuple(g.tensors[A].shape[:-1]) + (g.tensors[B].shape[-1],))
            ops.append(Op("MatMul", [A, B], [tmp], name=f"_gemm_matmul_{count}"))
            ops.append(Op("Add", [tmp, C], [Y], name=f"_gemm_add_{count}"))
        else:
            ops.append(Op("MatMul", [A, B], [Y], name=f"_gemm_matmul_{count}"))
    return ops


def resolve(g: Graph, ae: int = ALIGN_ELEMS) -> list:
    """The graph's operators as resolved nodes, Gemm decomposed (graph.py:280-302)."""
    infer_shapes(g)
    nodes = []
    for op in _decompose_gemm(g):
        t = op.op_type
        if t == "MatMul":
            nodes.append(_matmul(op, g.tensors))
        elif t == "Conv":
            nodes.append(_conv(op, g.tensors))
        elif t in _POOLS:
            nodes.append(_pool(op, g.tensors))
        elif t in _ALIASES:
            src, dst = g.tensors[op.inputs[0]], g.tensors[op.outputs[0]]
            if src.numel != dst.numel:
                raise SchedulerError(f"{t}: {src.numel} elements in, {dst.numel} out (views only)")
            nodes.append(_Node("alias", op, [src], dst))
        elif t in _VECTOROPS:
            nodes.append(_vectorop(op, g.tensors, ae))
        else:
            raise SchedulerError(f"operator {t} is not supported")
    return nodes


# ----------------------------------------------------------------------------------
# layouts (codegen/_core.py:75-249)
# ----------------------------------------------------------------------------------
@dataclass(frozen=True)
class Layout:
    numel: int
    alloc: int
    n_chunks: int
    chunk: int
    stride: int

    @property
    def gap(self) -> int:
        return self.stride - self.chunk

    @staticmethod
    def flat(n: int) -> "Layout":
        return Layout(n, n, 1, n, n)

    @staticmethod
    def advancing(n: int, chunks: int, stride: int) -> "Layout":
        return Layout(n, chunks * stride, chunks, n // chunks, stride)

    @staticmethod
    def block(n: int, alloc: int) -> "Layout":
        return Layout(n, alloc, 1, n, alloc)


def layouts(nodes: list) -> dict:
    """Buffer layout of every tensor the nodes touch.  Phase 1: all flat.  Phase 2: a
    broadcast vector op gives its output and advancing inputs n chunks at the aligned
    stride, its repeating input one padded block.  Phase 3, in node order: a
    non-broadcast vector op's output inherits a larger input allocation (and its chunks
    when strided), and smaller co-inputs are raised to the output's.  MatMul, Conv, Pool
    and aliases take no part in phases 2 and 3; a Conv or Pool output left strided is
    refused (the kernels write flat NCHW)."""
    lay = {}
    for nd in nodes:
        for t in nd.inputs + [nd.output]:
            lay.setdefault(t.name, Layout.flat(t.numel))
    vec = [nd for nd in nodes if nd.kind == "vectorop"]
    for nd in vec:
        if nd.outer <= 1:
            continue
        alloc = nd.outer * nd.stride

        def advance(t):
            cur = lay[t.name]
            if cur.n_chunks == 1 or alloc > cur.alloc:
                lay[t.name] = Layout.advancing(t.numel, nd.outer, nd.stride)

        def repeat(t):
            if nd.stride > lay[t.name].alloc:
                lay[t.name] = Layout.block(t.numel, nd.stride)
        advance(nd.output)
        (advance if nd.a_adv else repeat)(nd.inputs[0])
        if nd.arity == 2:
            (advance if nd.b_adv else repeat)(nd.inputs[1])
    for nd in vec:
        if nd.outer > 1:
            continue
        ins = [lay[t.name] for t in nd.inputs]
        top = max(x.alloc for x in ins)
        out = lay[nd.output.name]
        dom = None
        for x in ins:
            if x.n_chunks > 1 and (dom is None or x.alloc > dom.alloc):
                dom = x
        if top > out.alloc:
            out = (Layout.advancing(out.numel, dom.n_chunks, dom.stride) if dom is not None
                   else Layout.block(out.numel, top))
            lay[nd.output.name] = out
        for t in nd.inputs:
            cur = lay[t.name]
            if cur.alloc >= out.alloc:
                continue
            lay[t.name] = (Layout.advancing(cur.numel, out.n_chunks, out.stride) if out.n_chunks > 1
                           else Layout.block(cur.numel, out.alloc))
    for nd in nodes:
        if nd.kind in ("conv", "pool") and lay[nd.output.name].n_chunks > 1:
            raise SchedulerError(f"{nd.op.op_type} output '{nd.output.name}' feeds a broadcast vector op "
                                 "(a strided layout the kernel does not write)")
    return lay


# ----------------------------------------------------------------------------------
# calls
# ----------------------------------------------------------------------------------
def calls(nodes: list, lay: dict) -> list:
    """The kernel calls of the nodes, in order, as Net node tuples (aliases emit nothing)."""
    out = []
    for nd in nodes:
        if nd.kind == "vectorop":
            a = nd.inputs[0].name
            b = nd.inputs[1].name if nd.arity == 2 else None
            if nd.outer == 1:
                args = (lay[nd.output.name].alloc, nd.code, 1, 0, 0)
            else:
                a_inc = nd.stride if nd.a_adv else 0
                b_inc = (nd.stride if nd.b_adv else 0) if nd.arity == 2 else 0
                args = (nd.chunk, nd.code, nd.outer, a_inc, b_inc)
            out.append(("vectorop", a, b, nd.output.name, args))
        elif nd.kind == "matmul":
            n, k, m, batch, a_bs, b_bs, c_bs = nd.mm
            A, B, Y = nd.inputs[0].name, nd.inputs[1].name, nd.output.name
            if nd.mm_outer[0] == 1:
                ga, gy = lay[A], lay[Y]
                a_row = ga.stride if ga.gap > 0 else 0
                c_row = gy.stride if gy.gap > 0 else 0
                if a_row or c_row:
                    # gapped rows: n calls of one row, the batch stride stepping over the gaps
                    out.append(("matmul", A, B, Y, (1, k, m, n, a_row or k, b_bs, c_row or m)))
                else:
                    out.append(("matmul", A, B, Y, nd.mm))
            else:
                outer, a_os, b_os, c_os = nd.mm_outer
                for i in range(outer):
                    out.append(("matmul_at", A, B, Y, (i * a_os, i * b_os, i * c_os) + nd.mm))
        elif nd.kind == "conv":
            bias = nd.inputs[2].name if len(nd.inputs) > 2 else None
            out.append(("conv", nd.inputs[0].name, nd.inputs[1].name, bias, nd.output.name, nd.args))
        elif nd.kind == "pool":
            out.append(("pool", nd.inputs[0].name, nd.output.name, nd.args))
    return out


def _const_words(t: Tensor, L: Layout) -> np.ndarray:
    """A constant's words in its buffer layout: chunks at the stride, gap words zero."""
    data = np.asarray(t.data, np.int16).reshape(-1)
    out = np.zeros(max(L.alloc, 1), np.int16)
    if L.n_chunks > 1:
        for c in range(L.n_chunks):
            out[c * L.stride:c * L.stride + L.chunk] = data[c * L.chunk:(c + 1) * L.chunk]
    else:
        out[:data.size] = data
    return out


def derive(g: Graph, ae: int = ALIGN_ELEMS) -> Net:
    """The reference scheduler's call list for graph `g` (one input, one output)."""
    if len(g.inputs) != 1 or len(g.outputs) != 1:
        raise SchedulerError("one graph input and one graph output")
    nodes = resolve(g, ae)
    lay = layouts(nodes)
    net = Net(g.name, int(g.tensors[g.inputs[0]].shape[0]), g.inputs[0], g.outputs[0])
    for nd in nodes:
        if nd.kind == "alias":
            net.aliases[nd.output.name] = nd.inputs[0].name
    for name, L in lay.items():
        t = g.tensors[name]
        if name in net.aliases:
            continue
        if t.is_const:
            net.consts[name] = _const_words(t, L)
        else:
            net.buffers[name] = L.alloc
    net.buffers.setdefault(g.inputs[0], g.tensors[g.inputs[0]].numel)
    net.nodes = calls(nodes, lay)
    net.layouts = lay
    macs = 0
    for nd in nodes:
        if nd.kind == "conv":
            a = nd.args
            macs += a[0] * a[4] * a[5] * a[6] * (1 if a[16] else a[1]) * a[7] * a[8]
        elif nd.kind == "matmul":
            n, k, m, batch = nd.mm[:4]
            macs += nd.mm_outer[0] * batch * n * k * m
    net.macs_per_image = macs // max(net.batch, 1)
    return net
