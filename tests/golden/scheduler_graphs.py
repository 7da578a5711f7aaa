"""Operator graphs whose call lists are pinned against the reference scheduler
(test infrastructure; see make_calllists.py).  Each builder returns a
cormorant_b200.scheduler.Graph with one input and one output; ERROR_GRAPHS are
graphs the reference refuses (SchedulerError).

They cover what the reference scheduler derives for the four kernels
(inference-scheduler/src/nodes.py, src/graph.py, src/codegen/_core.py): the two
BASELINE networks, one-input broadcasting with and without alignment gaps (a
repeating input first or second, strided constant co-inputs), Clip(0, 6) by
attributes and by constant inputs, every MatMul batch form (2-D, either side
broadcast, flat batch, the 4-D x 3-D outer loop, the row-strided form on gapped
buffers), Conv padding modes / dilation / depthwise / no bias, every pool type with
padding, dilation, count_include_pad, p = 1 and the Global forms, and the alias ops.
"""
import numpy as np

from cormorant_b200 import networks
from cormorant_b200.scheduler import Graph, infer_shapes


def _rand(rng, shape, lo=-512, hi=512):
    return rng.integers(lo, hi, size=int(np.prod(shape))).astype(np.int16)


class _G:
    """Small builder: named tensors, ops with inferred output shapes."""

    def __init__(self, name, x_shape, seed=1):
        self.g = Graph(name)
        self.g.add("x", x_shape)
        self.g.inputs = ["x"]
        self.rng = np.random.default_rng(seed)
        self.n = 0

    def const(self, shape, lo=-512, hi=512, data=None):
        self.n += 1
        name = f"c{self.n}"
        self.g.add(name, shape, _rand(self.rng, shape, lo, hi) if data is None else data)
        return name

    def op(self, op_type, inputs, **attrs):
        self.n += 1
        out = f"t{self.n}_{op_type.lower()}"
        self.g.op(op_type, inputs, [out], **attrs)
        infer_shapes(self.g)
        return out

    def done(self, out):
        self.g.outputs = [out]
        return self.g


def g_broadcast():
    b = _G("broadcast", (2, 5, 6))
    y = b.op("Add", ["x", b.const((6,))])                 # bias repeats: chunk 6, stride 8 (gaps)
    y = b.op("Relu", [y])                                 # inherits the strided layout
    y = b.op("Mul", [y, b.const((2, 5, 6))])              # co-input raised to the strided layout
    y = b.op("Sub", [b.const((5, 6)), y])                 # first input repeats, second advances
    y = b.op("Div", [y, b.const((1, 6), 1, 512)])
    return b.done(b.op("Clip", [y], min=0.0, max=6.0))


def g_broadcast_aligned():
    b = _G("broadcast_aligned", (3, 4, 16))
    y = b.op("Mul", ["x", b.const((4, 16))])               # chunk 64: no gaps
    y = b.op("Clip", [y, b.const((), data=np.array([0], np.int16)), b.const((), data=np.array([1536], np.int16))])
    return b.done(b.op("Add", [y, y]))


def g_matmul_forms():
    b = _G("matmul_forms", (4, 5, 7))
    y = b.op("MatMul", ["x", b.const((7, 3))])             # B broadcast over A's batch
    y = b.op("Relu", [y])
    y = b.op("MatMul", [b.const((6, 5)), y])               # A broadcast over B's batch: [4, 6, 3]
    y = b.op("MatMul", [y, b.const((4, 3, 9))])            # flat batch
    return b.done(y)


def g_matmul_outer():
    b = _G("matmul_outer", (2, 3, 5, 7))
    y = b.op("MatMul", ["x", b.const((3, 7, 4))])          # 4-D x 3-D: outer loop of 2
    y = b.op("MatMul", [b.const((3, 6, 5)), y])            # 3-D x 4-D: B drives the outer loop
    return b.done(b.op("Relu", [y]))


def g_matmul_gapped():
    b = _G("matmul_gapped", (3, 20))
    y = b.op("MatMul", ["x", b.const((20, 12))])           # output feeds a gapped Add: row-strided C
    y = b.op("Add", [y, b.const((12,))])                   # chunk 12 -> stride 16
    y = b.op("Relu", [y])
    y = b.op("MatMul", [y, b.const((12, 10))])             # gapped A: row-strided A
    y = b.op("Add", [y, b.const((10,))])                   # stride 16 again
    return b.done(y)


def g_conv_forms():
    b = _G("conv_forms", (2, 3, 11, 13))
    y = b.op("Conv", ["x", b.const((4, 3, 3, 3)), b.const((4,))], strides=(2, 2), auto_pad="SAME_UPPER")
    y = b.op("Conv", [y, b.const((5, 4, 2, 3))], auto_pad="SAME_LOWER")                 # no bias
    y = b.op("Conv", [y, b.const((5, 1, 3, 3)), b.const((5,))], group=5, pads=(1, 1, 1, 1))   # depthwise
    y = b.op("Conv", [y, b.const((6, 5, 3, 2)), b.const((6,))], dilations=(2, 1), strides=(1, 2),
             pads=(2, 0, 1, 1))
    return b.done(b.op("Conv", [y, b.const((2, 6, 2, 2))], auto_pad="VALID"))


def g_pool_forms():
    b = _G("pool_forms", (2, 4, 17, 15))
    y = b.op("AveragePool", ["x"], kernel_shape=(3, 3), strides=(2, 2), pads=(1, 1, 1, 1), count_include_pad=1)
    y = b.op("MaxPool", [y], kernel_shape=(2, 3), dilations=(2, 1), pads=(1, 0, 1, 0))
    y = b.op("LpPool", [y], kernel_shape=(2, 2), p=1, auto_pad="SAME_UPPER")
    y = b.op("AveragePool", [y], kernel_shape=(2, 2), auto_pad="SAME_LOWER")
    return b.done(b.op("GlobalLpPool", [y], p=2))


def g_global_pools():
    b = _G("global_pools", (3, 8, 7, 5))
    y = b.op("GlobalMaxPool", ["x"])
    y = b.op("Squeeze", [y], axes=[2, 3])
    y = b.op("Unsqueeze", [y], axes=[2])
    y = b.op("Dropout", [y])
    y = b.op("GlobalAveragePool", [b.op("Unsqueeze", [y], axes=[3])])
    sh = b.const((2,), data=np.array([3, -1], np.int64))
    return b.done(b.op("Reshape", [y, sh]))


def g_gemm_nobias():
    b = _G("gemm_nobias", (5, 9))
    y = b.op("Gemm", ["x", b.const((9, 4))])
    return b.done(b.op("Gemm", [y, b.const((4, 6)), b.const((6,))], alpha=1.0, beta=1.0))


GRAPHS = {
    "lenet5_b1": lambda: networks.lenet5_graph(batch=1),
    "lenet5_b3": lambda: networks.lenet5_graph(batch=3),
    "resnet18_b2": lambda: networks.resnet18_graph(batch=2),
    "broadcast": g_broadcast,
    "broadcast_aligned": g_broadcast_aligned,
    "matmul_forms": g_matmul_forms,
    "matmul_outer": g_matmul_outer,
    "matmul_gapped": g_matmul_gapped,
    "conv_forms": g_conv_forms,
    "pool_forms": g_pool_forms,
    "global_pools": g_global_pools,
    "gemm_nobias": g_gemm_nobias,
}


def e_gemm_trans():
    b = _G("e_gemm_trans", (5, 9))
    b.g.add("c_w", (4, 9), _rand(b.rng, (4, 9)))
    b.g.op("Gemm", ["x", "c_w"], ["y"], transB=1)
    b.g.add("y", (5, 4))
    return b.done("y")


def e_grouped_conv():
    b = _G("e_grouped_conv", (1, 4, 6, 6))
    return b.done(b.op("Conv", ["x", b.const((4, 2, 3, 3))], group=2))


def e_ceil_mode():
    b = _G("e_ceil_mode", (1, 2, 7, 7))
    b.g.op("MaxPool", ["x"], ["y"], kernel_shape=(2, 2), strides=(2, 2), ceil_mode=1)
    b.g.add("y", (1, 2, 4, 4))
    return b.done("y")


def e_lp3():
    b = _G("e_lp3", (1, 2, 6, 6))
    return b.done(b.op("LpPool", ["x"], kernel_shape=(2, 2), p=3))


def e_clip():
    b = _G("e_clip", (2, 8))
    return b.done(b.op("Clip", ["x"], min=0.0, max=5.0))


def e_both_broadcast():
    b = _G("e_both_broadcast", (3, 1))
    b.g.add("c_b", (1, 4), _rand(b.rng, (1, 4)))
    b.g.op("Add", ["x", "c_b"], ["y"])
    b.g.add("y", (3, 4))
    return b.done("y")


def e_conv_then_broadcast():
    b = _G("e_conv_then_broadcast", (2, 2, 5, 5))
    y = b.op("Conv", ["x", b.const((3, 2, 3, 3))])          # [2, 3, 3, 3]
    return b.done(b.op("Add", [y, b.const((3, 3, 3))]))     # chunk 27 -> stride 32 on the conv output


ERROR_GRAPHS = {
    "e_gemm_trans": e_gemm_trans,
    "e_grouped_conv": e_grouped_conv,
    "e_ceil_mode": e_ceil_mode,
    "e_lp3": e_lp3,
    "e_clip": e_clip,
    "e_both_broadcast": e_both_broadcast,
    "e_conv_then_broadcast": e_conv_then_broadcast,
}
