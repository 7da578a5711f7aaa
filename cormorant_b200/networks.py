"""The two whole-network configurations of the benchmark, as kernel-call lists.

The reference compiles an ONNX graph into a sequence of run_op / run_matmul /
run_conv / run_pool calls over one buffer pool (inference-scheduler/src/graph.py,
src/nodes.py, src/codegen/_source.py).  Each network here is built as the same
operator graph (`lenet5_graph`, `resnet18_graph`: Conv with bias, Relu, MaxPool,
residual Add, GlobalAveragePool, Reshape to [N, -1], Gemm) and its call list is
derived by `scheduler.derive`, which restates the reference scheduler's argument
derivation (Gemm -> MatMul + broadcast Add, Reshape -> buffer alias, alignment gaps
and the row-strided MatMul form where a row width is not a multiple of 8 words).

Each node is a plain tuple; `execute` walks the list on any backend that offers
the four kernels (the GPU backend here; the tests replay the same list on the
CPU oracle).  `fuse` and `chain` rewrite a list into its fused / plane-image forms.
Weights are seeded synthetic data with the configurations' shapes and
distributions.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

OP_ADD, OP_RELU = 0, 4
EPI_NHWC = 8          # conv epilogue bit 3: y channels-last (cm_conv_planes)


def conv_out(n: int, k: int, s: int, p: int, d: int = 1) -> int:
    return (n + 2 * p - d * (k - 1) - 1) // s + 1


@dataclass
class Net:
    name: str
    batch: int
    input: str
    output: str
    buffers: dict = field(default_factory=dict)      # name -> number of int16 words
    consts: dict = field(default_factory=dict)       # name -> int16 array (weights, biases)
    nodes: list = field(default_factory=list)        # (kind, args...) -- see execute()
    aliases: dict = field(default_factory=dict)      # Reshape: name -> name
    macs_per_image: int = 0
    source_kinds: tuple = ()                         # kernel kinds of the call list before fusion
    planes: dict = field(default_factory=dict)       # plane image -> (batch, C, H, W, frame)
    layouts: dict = field(default_factory=dict)      # tensor -> scheduler.Layout (buffers with alignment gaps)

    def buf(self, name: str, words: int) -> str:
        self.buffers[name] = int(words)
        return name

    def resolve(self, name: str) -> str:
        while name in self.aliases:
            name = self.aliases[name]
        return name


def q88_floor(v: np.ndarray) -> np.ndarray:
    return np.clip(np.floor(v * 256.0), -32768, 32767).astype(np.int16)


def q88_round(v: np.ndarray) -> np.ndarray:
    """dtype.py quantize(): clip, round half to even at 2^-8."""
    return np.clip(np.round(np.clip(v, -128.0, 127.99609375) * 256.0), -32768, 32767).astype(np.int16)


class _GraphBuilder:
    """Builds the ONNX-shaped operator graph of a network (scheduler.Graph); the call list
    is then derived from it exactly as the reference scheduler derives it."""

    def __init__(self, name: str, batch: int, x_shape, weight_fn):
        from .scheduler import Graph
        self.g = Graph(name)
        self.g.add("x", (batch,) + tuple(x_shape))
        self.g.inputs = ["x"]
        self.weight_fn = weight_fn
        self.count = 0

    def _name(self, kind: str) -> str:
        self.count += 1
        return f"{kind}{self.count}"

    def _op(self, op_type, inputs, outputs, **attrs):
        from .scheduler import infer_shapes
        self.g.op(op_type, inputs, outputs, **attrs)
        infer_shapes(self.g)

    def conv(self, x, m, k, s, p, bias=True):
        c = self.g.tensors[x].shape[1]
        wn, bn = self._name("W"), self._name("B")
        self.g.add(wn, (m, c, k, k), self.weight_fn((m, c, k, k), c * k * k))
        ins = [x, wn]
        if bias:
            self.g.add(bn, (m,), self.weight_fn((m,), None))
            ins.append(bn)
        y = self._name("conv")
        self._op("Conv", ins, [y], kernel_shape=(k, k), strides=(s, s), pads=(p, p, p, p))
        return y

    def relu(self, x):
        y = self._name("relu")
        self._op("Relu", [x], [y])
        return y

    def add(self, a, b):
        y = self._name("add")
        self._op("Add", [a, b], [y])
        return y

    def maxpool(self, x, k, s, p):
        y = self._name("pool")
        self._op("MaxPool", [x], [y], kernel_shape=(k, k), strides=(s, s), pads=(p, p, p, p))
        return y

    def global_avgpool(self, x):
        y = self._name("pool")
        self._op("GlobalAveragePool", [x], [y])
        return y

    def flatten(self, x):
        """Reshape to [N, -1] (the shape given as a constant int64 input, as ONNX does)."""
        y, sh = self._name("reshape"), self._name("shape")
        self.g.add(sh, (2,), np.array([self.g.tensors[x].shape[0], -1], np.int64))
        self._op("Reshape", [x, sh], [y])
        return y

    def gemm(self, x, k, m):
        wn, bn = self._name("W"), self._name("B")
        self.g.add(wn, (k, m), self.weight_fn((k, m), k))
        self.g.add(bn, (m,), self.weight_fn((m,), None))
        y = self._name("gemm")
        self._op("Gemm", [x, wn, bn], [y])
        return y

    def finish(self, out: str):
        self.g.outputs = [out]
        return self.g


def lenet5_graph(batch: int = 1, seed: int = 42):
    """BASELINE config 0 as an operator graph: LeNet-5-style CNN, 1x1x28x28 input; weights
    and biases uniform [-0.5, 0.5) rounded down to a multiple of 1/256."""
    rng = np.random.default_rng(seed)
    wfn = lambda shape, fan_in: q88_floor(rng.uniform(-0.5, 0.5, size=shape)).reshape(-1)  # noqa: E731
    b = _GraphBuilder("lenet5", batch, (1, 28, 28), wfn)
    y = b.maxpool(b.relu(b.conv("x", 6, 5, 1, 2)), 2, 2, 0)
    y = b.maxpool(b.relu(b.conv(y, 16, 5, 1, 0)), 2, 2, 0)
    y = b.flatten(y)                                           # [N, 400]
    y = b.relu(b.gemm(y, 400, 120))
    y = b.relu(b.gemm(y, 120, 84))
    return b.finish(b.gemm(y, 84, 10))


def resnet18_graph(batch: int = 256, seed: int = 42, num_classes: int = 1000):
    """BASELINE config 3 as an operator graph: ResNet-18-shaped plain CNN (no normalisation
    layers), 3x224x224 input; He-scaled normal weights N(0, 2/fan_in) and N(0, 0.01^2)
    biases, rounded to Q8.8."""
    rng = np.random.default_rng(seed)

    def wfn(shape, fan_in):
        sd = np.sqrt(2.0 / fan_in) if fan_in else 0.01
        return q88_round(rng.normal(0.0, sd, size=shape)).reshape(-1)

    b = _GraphBuilder("resnet18", batch, (3, 224, 224), wfn)
    y = b.maxpool(b.relu(b.conv("x", 64, 7, 2, 3)), 3, 2, 1)   # 56 x 56
    c = 64
    for width, stride in ((64, 1), (128, 2), (256, 2), (512, 2)):
        for blk in range(2):
            s = stride if blk == 0 else 1
            t = b.relu(b.conv(y, width, 3, s, 1))
            t = b.conv(t, width, 3, 1, 1)
            sc = b.conv(y, width, 1, s, 0) if (s != 1 or c != width) else y
            y = b.relu(b.add(t, sc))
            c = width
    y = b.flatten(b.global_avgpool(y))                         # [N, 512]
    return b.finish(b.gemm(y, 512, num_classes))


def lenet5(batch: int = 1, seed: int = 42) -> Net:
    """LeNet-5's call list, derived from its graph as the reference
    scheduler derives it (scheduler.derive)."""
    from .scheduler import derive
    return derive(lenet5_graph(batch, seed))


def resnet18(batch: int = 256, seed: int = 42, num_classes: int = 1000) -> Net:
    """the ResNet-18-shaped network's call list, derived from its graph
    as the reference scheduler derives it (scheduler.derive)."""
    from .scheduler import derive
    return derive(resnet18_graph(batch, seed, num_classes))


def make_input(net: Net, seed: int = 7) -> np.ndarray:
    """Input uniform [0, 1), rounded to Q8.8 (dtype.py quantize)."""
    rng = np.random.default_rng(seed)
    return q88_round(rng.uniform(0.0, 1.0, size=net.buffers[net.input]))


def _inputs(node) -> list:
    kind = node[0]
    if kind == "convpool":
        return [n for n in (node[1], node[2], node[3], node[7]) if n is not None]
    if kind == "conv":
        names = [node[1], node[2], node[3]] + ([node[7]] if len(node) > 7 else [])
        if len(node) > 8 and node[1] is None:
            names[0] = node[8]                       # read from its plane image only
        if len(node) > 10 and node[7] is None and node[10] is not None:
            names[3] = node[10]                      # residual from its plane image only
    elif kind in ("matmul", "matmul_at"):
        names = [node[1], node[2]] + ([node[6]] if len(node) > 6 else [])
    elif kind == "vectorop":
        names = [node[1], node[2]]
    else:                                            # pool, planes
        names = [node[1]]
    return [n for n in names if n is not None]


def output_of(node) -> str:
    if node[0] == "convpool":
        return node[4]
    if node[0] == "conv":
        return node[4] if node[4] is not None else node[9]
    return node[3] if node[0] in ("vectorop", "matmul", "matmul_at") else node[2]   # pool, planes: node[2]


def chain(net: Net, frame_fn=None, pool_planes: bool = False, nhwc_fn=None, pool_nhwc: bool = True) -> Net:
    """The call list with conv outputs that feed implicit-GEMM convs produced as plane
    images (cm_conv_planes): the producing conv's GEMM epilogue writes the consumers'
    channels-last operand, so their split pass disappears, and a residual those convs
    add comes from its plane image too.  `frame_fn(args)` gives the padding frame a
    conv reads its input with, or None when it reads the NCHW tensor (default: the
    library's cm_conv_plane_frame).  The NCHW output is still written when anything
    else reads it (a vector op, a non-MAX pool, a conv that cannot read plane images,
    the network output).  Conv nodes become
    ("conv", x, w, bias, y, args, epilogue, resid, xp, yp, rp) with x / y / resid None
    when unused.  With pool_planes=True a MAX pool between a conv and plane-reading convs
    runs plane image to plane image: ("poolp", xp, yp, args) (off by default: on
    ResNet-18's stem it measured slower than the NCHW pool plus one split).  With
    pool_nhwc=True (default) a MAX pool that is the only reader of a conv's output, whose
    own output only plane-reading convs read, and whose channels are a multiple of 16 (and
    whose conv can write channels-last, `nhwc_fn(args)`, default the library's
    cm_conv_writes_nhwc): the conv writes its output channels-last (epilogue bit 3) and
    the pool reads that and writes the plane image, ("poolnp", x, yp, args) -- no NCHW
    tensor, no split pass (ResNet-18's stem).  Likewise (pool_nhwc=True) a global pool that
    is the only reader of a conv's output (channels a multiple of 8, the conv's residual,
    if any, read from a plane image) takes that output channels-last: ("poolng", x, y,
    args), cm_pool_nhwc (ResNet-18's last block before GlobalAveragePool: its conv stores
    rows instead of scattered NCHW words).  A tensor no conv produced (the input, a pool
    output kept NCHW) that convs read at least twice as an operand or residual gets one
    ("planes", x, image) split pass right after its producer."""
    if frame_fn is None:
        from . import kernels
        frame_fn = lambda args: kernels.conv_plane_frame(*args)  # noqa: E731
    if nhwc_fn is None:
        from . import kernels
        nhwc_fn = lambda args: kernels.conv_writes_nhwc(*args)  # noqa: E731
    R = net.resolve
    nodes = [n if n[0] != "conv" or len(n) > 6 else (*n, 0, None) for n in net.nodes]
    reads_planes = {j: frame_fn(n[5]) for j, n in enumerate(nodes) if n[0] == "conv"}
    uses: dict = {}                                   # tensor -> [(node, role)]
    for j, node in enumerate(nodes):
        if node[0] == "conv":
            uses.setdefault(R(node[1]), []).append((j, "x"))
            for name in (node[2], node[3]):
                if name is not None:
                    uses.setdefault(R(name), []).append((j, "other"))
            if node[7] is not None:
                uses.setdefault(R(node[7]), []).append((j, "resid"))
        elif node[0] == "pool" and node[3][14] == 0:
            uses.setdefault(R(node[1]), []).append((j, "maxpool"))
        else:
            for name in _inputs(node):
                uses.setdefault(R(name), []).append((j, "other"))
    uses.setdefault(R(net.output), []).append((-1, "other"))
    produced = {R(n[4]): i for i, n in enumerate(nodes) if n[0] == "conv"}

    def plane_readers(t):
        """(x readers with their frames, residual readers) that can take t's plane image."""
        readers = uses.get(t, [])
        x_ok = [(j, reads_planes[j]) for j, role in readers if role == "x" and reads_planes[j] is not None]
        r_ok = [j for j, role in readers if role == "resid" and reads_planes[j] is not None]
        return x_ok, r_ok

    # MAX pools whose conv writes channels-last for them (the pool its only reader) and
    # whose output only plane-reading convs read
    poolnp, nhwc_convs = {}, set()
    for j, node in enumerate(nodes):
        if not pool_nhwc or node[0] != "pool" or node[3][14] != 0 or R(node[1]) not in produced:
            continue
        t, u = R(node[1]), R(node[2])
        i = produced[t]
        if uses.get(t) != [(j, "maxpool")] or node[3][1] % 16 or nodes[i][7] is not None or not nhwc_fn(nodes[i][5]):
            continue
        x_ok, r_ok = plane_readers(u)
        if (x_ok or r_ok) and len(x_ok) + len(r_ok) == len(uses.get(u, [])):
            poolnp[j] = (x_ok, r_ok)
            nhwc_convs.add(i)
    # global pools whose conv writes channels-last for them (the pool its only reader)
    poolng = set()
    for j, node in enumerate(nodes):
        if not pool_nhwc or node[0] != "pool" or R(node[1]) not in produced:
            continue
        a, t = node[3], R(node[1])
        i = produced[t]
        glob = a[4] == 1 and a[5] == 1 and a[6] == a[2] and a[7] == a[3] and a[10] == 0 and a[11] == 0
        res = nodes[i][7]
        res_ok = res is None or i in plane_readers(R(res))[1]
        if (glob and a[1] % 8 == 0 and len(uses.get(t, [])) == 1 and uses[t][0][0] == j and res_ok
                and nhwc_fn(nodes[i][5])):
            poolng.add(j)
            nhwc_convs.add(i)
    # MAX pools that can run plane to plane: conv input, output read only by plane-reading convs
    poolp = {}
    for j, node in enumerate(nodes):
        if (not pool_planes or j in poolnp or node[0] != "pool" or node[3][14] != 0
                or R(node[1]) not in produced):
            continue
        u = R(node[2])
        x_ok, r_ok = plane_readers(u)
        if (x_ok or r_ok) and len(x_ok) + len(r_ok) == len(uses.get(u, [])):
            poolp[j] = (x_ok, r_ok)
    xp_of, rp_of, keep_of, planes, fills = {}, {}, {}, {}, {}

    def image(t, a, x_ok, r_ok, keep):
        frame = tuple(max([f[k] for _, f in x_ok] + [0]) for k in range(4))
        pname = t + "@planes"
        planes[pname] = (net.batch, a[0], a[1], a[2], frame)
        for j, _ in x_ok:
            xp_of[j] = (pname, keep)
        for j in r_ok:
            rp_of[j] = (pname, keep)
        return pname

    for t, i in produced.items():
        readers = uses.get(t, [])
        x_ok, r_ok = plane_readers(t)
        pools = [j for j, role in readers if role == "maxpool" and j in poolp]
        if not x_ok and not r_ok and not pools:
            continue
        served = {(j, "x") for j, _ in x_ok} | {(j, "resid") for j in r_ok} | {(j, "maxpool") for j in pools}
        keep = any((j, role) not in served for j, role in readers)
        a = nodes[i][5]
        keep_of[i] = (image(t, (a[4], a[5], a[6]), x_ok, r_ok, keep), keep)
    pool_io = {}
    for j, (x_ok, r_ok) in poolp.items():
        node = nodes[j]
        t, u, a = R(node[1]), R(node[2]), node[3]
        pool_io[j] = (keep_of[produced[t]][0], image(u, (a[1], a[4], a[5]), x_ok, r_ok, False))
    pool_nhwc_io = {}
    for j, (x_ok, r_ok) in poolnp.items():
        node = nodes[j]
        u, a = R(node[2]), node[3]
        pool_nhwc_io[j] = (node[1], image(u, (a[1], a[4], a[5]), x_ok, r_ok, False))
    others = {R(output_of(n)): j for j, n in enumerate(nodes)
              if n[0] != "conv" and j not in poolp and j not in poolnp}
    others.setdefault(R(net.input), -1)
    for t, i in others.items():
        x_ok, r_ok = plane_readers(t)
        if not x_ok or len(x_ok) + len(r_ok) < 2:
            continue
        a = nodes[x_ok[0][0]][5]
        fills.setdefault(i, []).append((t, image(t, (a[1], a[2], a[3]), x_ok, r_ok, True)))
    out = [("planes", t, pname) for t, pname in fills.get(-1, [])]
    for i, node in enumerate(nodes):
        if i in pool_io:
            out.append(("poolp", pool_io[i][0], pool_io[i][1], node[3]))
            continue
        if i in pool_nhwc_io:
            out.append(("poolnp", pool_nhwc_io[i][0], pool_nhwc_io[i][1], node[3]))
            continue
        if i in poolng:
            out.append(("poolng", node[1], node[2], node[3]))
            continue
        if node[0] != "conv":
            out.append(node)
            out.extend(("planes", t, pname) for t, pname in fills.get(i, []))
            continue
        _, x, wn, bn, y, args, epi, resid = node
        xp = yp = rp = None
        if i in xp_of:
            xp, keep = xp_of[i]
            x = x if keep else None
        if i in rp_of:
            rp, keep = rp_of[i]
            resid = resid if keep else None
        if i in keep_of:
            yp, keep = keep_of[i]
            y = y if keep else None
        if i in nhwc_convs:
            epi |= EPI_NHWC                              # y channels-last, read only by its pool
        out.append(("conv", x, wn, bn, y, args, epi, resid, xp, yp, rp))
    names = set(net.buffers) | set(net.aliases)
    used = {R(n) for node in out for n in _inputs(node) if n in names}
    used |= {R(output_of(node)) for node in out if output_of(node) in names}
    used |= {R(net.input), R(net.output)}
    return Net(net.name + "+planes", net.batch, net.input, net.output,
               buffers={k: v for k, v in net.buffers.items() if k in used}, consts=dict(net.consts), nodes=out,
               aliases=dict(net.aliases), macs_per_image=net.macs_per_image,
               source_kinds=net.source_kinds or tuple(sorted({n[0] for n in net.nodes})), planes=planes)


def fuse(net: Net, residual: bool = True, gemm: bool = True, conv_pool_macs: int = 1 << 22) -> Net:
    """The call list with Conv -> Relu chains and (residual=True) Conv -> Add and
    Conv -> Add -> Relu chains folded into one conv call with a fused epilogue
    (cm_conv_fused), and (gemm=True) the Gemm decomposition MatMul -> Add(bias row) and
    MatMul -> [Add(bias row)] -> Relu folded into one cm_matmul_fused call: the same
    words, without writing and re-reading the intermediate tensors.  A conv of at most
    `conv_pool_macs` multiply-adds (a launch-bound size) whose output only a MAX pool reads
    becomes one ("convpool", x, w, bias, y, args, epi, resid, pool_args) call, cm_conv_pool
    (0 turns it off).  A chain is folded only when each intermediate result has no other
    reader (and is not the network output)."""
    R = net.resolve
    reads: dict = {}
    for node in net.nodes:
        for name in _inputs(node):
            reads[R(name)] = reads.get(R(name), 0) + 1
    reads[R(net.output)] = reads.get(R(net.output), 0) + 1

    def whole(node, words):                  # a full-tensor elementwise call (no broadcast)
        return node[0] == "vectorop" and node[4][0] == words and node[4][2:] == (1, 0, 0)

    def relu_of(node, y):
        return whole(node, net.buffers[y]) and node[4][1] == OP_RELU and R(node[1]) == y

    def add_with(node, y):
        return (whole(node, net.buffers[y]) and node[4][1] == OP_ADD and node[2] is not None
                and y in (R(node[1]), R(node[2])) and R(node[1]) != R(node[2]))

    nodes = list(net.nodes)
    if residual:
        # Conv D; Conv C; Add(C's output, D's output): the Add is folded into the conv that
        # runs right before it.  When D has the longer reduction (a 3x3 conv against ResNet's
        # 1x1 projection shortcut) and neither reads the other's output, C runs first, so the
        # residual read sits in the epilogue of the conv whose mainloop hides it.  ADD is
        # symmetric (sat16(a + b)): the words do not change.
        for i in range(1, len(nodes) - 1):
            d, c, nxt = nodes[i - 1], nodes[i], nodes[i + 1]
            if not (d[0] == "conv" and c[0] == "conv" and len(d) == 6 and len(c) == 6):
                continue
            yd, yc = R(d[4]), R(c[4])
            if not (add_with(nxt, yc) and add_with(nxt, yd) and reads.get(yd, 0) == 1 and reads.get(yc, 0) == 1):
                continue
            if yd in {R(n) for n in _inputs(c)} or yc in {R(n) for n in _inputs(d)}:
                continue
            red = lambda a: a[7] * a[8] * (1 if a[16] else a[1])     # noqa: E731  taps x channels per output
            if red(d[5]) > red(c[5]):
                nodes[i - 1], nodes[i] = c, d
    out, i = [], 0
    while i < len(nodes):
        node = nodes[i]
        if node[0] == "conv" and len(node) == 6 and i + 1 < len(nodes) and reads.get(R(node[4]), 0) == 1:
            _, x, wn, bn, y, args = node
            y, nxt = R(y), nodes[i + 1]
            if relu_of(nxt, y):
                out.append(("conv", x, wn, bn, nxt[3], args, 1, None))
                i += 2
                continue
            if residual and add_with(nxt, y):
                other = nxt[2] if R(nxt[1]) == y else nxt[1]
                c = R(nxt[3])
                if i + 2 < len(nodes) and reads.get(c, 0) == 1 and relu_of(nodes[i + 2], c):
                    out.append(("conv", x, wn, bn, nodes[i + 2][3], args, 3, other))
                    i += 3
                else:
                    out.append(("conv", x, wn, bn, nxt[3], args, 2, other))
                    i += 2
                continue
        if gemm and node[0] == "matmul" and len(node) == 5 and i + 1 < len(nodes) and reads.get(R(node[3]), 0) == 1:
            _, a, b, c, args = node
            n, _, m, batch, _, b_bs, c_bs = args
            c, nxt = R(c), nodes[i + 1]
            # the output as rows of m words at a pitch: one matrix (batch 1), or the
            # row-strided form (n = 1, B shared, one row per batch step c_bs apart)
            rows, pitch = (n, m) if batch == 1 else ((batch, c_bs) if n == 1 and b_bs == 0 else (0, 0))
            # the Gemm's bias Add: the bias row broadcast over those rows (at one row the
            # scheduler emits a plain whole-tensor Add)
            bias_forms = {(m, OP_ADD, rows, pitch, 0)} | ({(m, OP_ADD, 1, 0, 0)} if rows == 1 else set())
            if (rows and nxt[0] == "vectorop" and tuple(nxt[4]) in bias_forms
                    and R(nxt[1]) == c and nxt[2] is not None and R(nxt[2]) != c):
                y, epi, step = nxt[3], 2, 2
                if i + 2 < len(nodes) and reads.get(R(y), 0) == 1 and relu_of(nodes[i + 2], R(y)):
                    y, epi, step = nodes[i + 2][3], 3, 3
                out.append(("matmul", a, b, y, args, epi, nxt[2]))
                i += step
                continue
            if rows and relu_of(nxt, c):
                out.append(("matmul", a, b, nxt[3], args, 1, None))
                i += 2
                continue
        out.append(node)
        i += 1
    if conv_pool_macs:
        folded, i = [], 0
        while i < len(out):
            node = out[i]
            if node[0] == "conv" and i + 1 < len(out) and out[i + 1][0] == "pool":
                args, p = node[5], out[i + 1]
                pa, y = p[3], R(node[4])
                macs = args[0] * args[4] * args[5] * args[6] * args[1] * args[7] * args[8]
                if (R(p[1]) == y and reads.get(y, 0) == 1 and pa[14] == 0 and not args[16] and macs <= conv_pool_macs
                        and tuple(pa[:4]) == (args[0], args[4], args[5], args[6])):
                    epi, resid = (node[6], node[7]) if len(node) > 6 else (0, None)
                    folded.append(("convpool", node[1], node[2], node[3], p[2], args, epi, resid, pa))
                    i += 2
                    continue
            folded.append(node)
            i += 1
        out = folded
    used = {R(n) for node in out for n in _inputs(node)} | {R(output_of(node)) for node in out}
    used |= {R(net.input), R(net.output)}
    fused = Net(net.name + "+fused", net.batch, net.input, net.output,
                buffers={k: v for k, v in net.buffers.items() if k in used}, consts=dict(net.consts), nodes=out,
                aliases=dict(net.aliases), macs_per_image=net.macs_per_image,
                source_kinds=net.source_kinds or tuple(sorted({n[0] for n in net.nodes})))
    return fused


def calls_of(net: Net, bufs: dict):
    """The call list as (kind, epilogue, in0, in1, in2, resid, out, args) tuples for
    cm_calls, or None when a node has no one-launch form (plane images)."""
    from . import kernels as k
    R = lambda name: None if name is None else bufs[net.resolve(name)]  # noqa: E731
    out = []
    for node in net.nodes:
        kind = node[0]
        if kind == "conv" and len(node) <= 8:
            _, x, wn, bn, y, args = node[:6]
            epi, resid = (node[6], node[7]) if len(node) > 6 else (0, None)
            out.append((k.CALL_CONV, epi, R(x), R(wn), R(bn), R(resid), R(y), args))
        elif kind == "matmul":
            _, a, b, c, args = node[:5]
            epi, bias = (node[5], node[6]) if len(node) > 5 else (0, None)
            out.append((k.CALL_MATMUL, epi, R(a), R(b), R(bias), None, R(c), args))
        elif kind == "pool":
            _, x, y, args = node
            out.append((k.CALL_POOL, 0, R(x), None, None, None, R(y), args))
        elif kind == "vectorop":
            _, a, b, c, args = node
            out.append((k.CALL_VECTOROP, 0, R(a), R(b), None, None, R(c), args))
        else:
            return None
    return out


def execute(net: Net, backend, bufs: dict) -> None:
    """Run every node of `net` on `backend` over `bufs` (name -> backend buffer).

    backend offers vectorop(a, b, c, size, op, outer, a_inc, b_inc),
    matmul(a, b, c, n, k, m, batch, a_bs, b_bs, c_bs), matmul_at(a, b, c, a_off, b_off, c_off,
    n, k, m, batch, a_bs, b_bs, c_bs) (the reference's run_matmul_at), conv(x, w, bias, y, *17 scalars),
    pool(x, y, *17 scalars) and, for fused call lists, conv_fused(x, w, bias, y, *17
    scalars, epilogue, resid) and matmul_fused(a, b, c, *7 scalars, epilogue, bias)."""
    if getattr(backend, "one_launch", False) and backend.run_list(net, bufs):
        return
    R = lambda name: None if name is None else bufs[net.resolve(name)]  # noqa: E731
    for node in net.nodes:
        kind = node[0]
        if kind == "conv" and len(node) > 8:
            _, x, wn, bn, y, args, epi, resid, xp, yp, rp = node
            backend.conv_planes(R(x), R(xp), R(wn), R(bn), R(y), R(yp), *args, epi, R(resid), R(rp))
        elif kind == "conv" and len(node) > 6:
            _, x, wn, bn, y, args, epi, resid = node
            backend.conv_fused(R(x), R(wn), R(bn), R(y), *args, epi, R(resid))
        elif kind == "conv":
            _, x, wn, bn, y, args = node
            backend.conv(R(x), R(wn), R(bn), R(y), *args)
        elif kind == "vectorop":
            _, a, bb, c, args = node
            backend.vectorop(R(a), R(bb), R(c), *args)
        elif kind == "pool":
            _, x, y, args = node
            backend.pool(R(x), R(y), *args)
        elif kind == "planes":
            _, x, p = node
            backend.planes_fill(R(x), R(p))
        elif kind == "poolp":
            _, xp, yp, args = node
            backend.pool_planes(R(xp), R(yp), *args)
        elif kind == "poolnp":
            _, x, yp, args = node
            backend.pool_nhwc_planes(R(x), R(yp), *args)
        elif kind == "poolng":
            _, x, y, args = node
            backend.pool_nhwc(R(x), R(y), *args)
        elif kind == "convpool":
            _, x, wn, bn, y, args, epi, resid, pargs = node
            backend.conv_pool(R(x), R(wn), R(bn), R(y), args, epi, R(resid), pargs)
        elif kind == "matmul" and len(node) > 5:
            _, a, bb, c, args, epi, bias = node
            backend.matmul_fused(R(a), R(bb), R(c), *args, epi, R(bias))
        elif kind == "matmul":
            _, a, bb, c, args = node
            backend.matmul(R(a), R(bb), R(c), *args)
        elif kind == "matmul_at":
            _, a, bb, c, args = node
            backend.matmul_at(R(a), R(bb), R(c), *args)
        else:
            raise ValueError(kind)


class GpuBackend:
    """The four kernels of libcormorant_cuda.so on one CUDA stream (asynchronous)."""

    def __init__(self, stream=None, one_launch: bool = False, weights: dict | None = None):
        from . import kernels
        self.k = kernels
        self.stream = stream
        # weights: prepared conv weights (prepare_weights) looked up by the call's weight and
        # bias buffers and geometry; convs without an entry prepare their weights per call
        self.weights = weights or {}
        # one_launch: a call list that cm_calls accepts (small batch-1 networks) runs as
        # one kernel launch instead of one launch per call
        self.one_launch = one_launch
        self._lists: dict = {}

    def run_list(self, net, bufs) -> bool:
        key = (id(net), id(bufs))
        if key not in self._lists:
            calls = calls_of(net, bufs)
            arr = None
            if calls is not None and 0 < len(calls) <= self.k.CALLS_MAX:
                arr = self.k.call_array(calls)
                if not self.k.calls_supported(arr):
                    arr = None
            self._lists[key] = arr
        arr = self._lists[key]
        if arr is None:
            return False
        self.k.RunCalls(arr, stream=self.stream)
        return True

    def vectorop(self, a, b, c, size, op, outer, a_inc, b_inc):
        self.k.VectorOPKernel(a, b, c, size, op, outer, a_inc, b_inc, stream=self.stream)

    def _prepared_b(self, b, k, m, batch, b_bs):
        if not self.weights or (batch > 1 and b_bs != 0):
            return None
        return self.weights.get(matmul_weights_key(b, k, m))

    def matmul(self, a, b, c, n, k, m, batch, a_bs, b_bs, c_bs):
        pw = self._prepared_b(b, k, m, batch, b_bs)
        if pw is not None:
            self.k.MatmulKernelPrepared(pw, a, c, n, batch, a_bs, c_bs, stream=self.stream)
        else:
            self.k.MatmulKernel(a, b, c, n, k, m, batch, a_bs, b_bs, c_bs, stream=self.stream)

    def matmul_at(self, a, b, c, a_off, b_off, c_off, n, k, m, batch, a_bs, b_bs, c_bs):
        # run_matmul_at: the element offsets move the three base addresses
        self.k.MatmulKernel(a.reshape(-1)[a_off:], b.reshape(-1)[b_off:], c.reshape(-1)[c_off:], n, k, m, batch,
                            a_bs, b_bs, c_bs, stream=self.stream)

    def matmul_fused(self, a, b, c, n, k, m, batch, a_bs, b_bs, c_bs, epi, bias):
        pw = self._prepared_b(b, k, m, batch, b_bs)
        if pw is not None:
            self.k.MatmulKernelPrepared(pw, a, c, n, batch, a_bs, c_bs, epilogue=epi, bias=bias, stream=self.stream)
        else:
            self.k.MatmulKernelFused(a, b, c, n, k, m, batch, a_bs, b_bs, c_bs, epilogue=epi, bias=bias,
                                     stream=self.stream)

    def _prepared(self, w, bias, geo):
        return self.weights.get(weights_key(w, bias, geo)) if self.weights else None

    def conv(self, x, w, bias, y, *args):
        pw = self._prepared(w, bias, args)
        if pw is not None:
            self.k.ConvKernelPrepared(pw, x, None, y, None, stream=self.stream)
        else:
            self.k.ConvKernel(x, w, bias, y, *args, stream=self.stream)

    def conv_fused(self, x, w, bias, y, *args):
        *geo, epi, resid = args
        pw = self._prepared(w, bias, geo)
        if pw is not None:
            self.k.ConvKernelPrepared(pw, x, None, y, None, epilogue=epi, resid=resid, stream=self.stream)
        else:
            self.k.ConvKernelFused(x, w, bias, y, *geo, epilogue=epi, resid=resid, stream=self.stream)

    def conv_planes(self, x, xp, w, bias, y, yp, *args):
        *geo, epi, resid, rp = args
        pw = self._prepared(w, bias, geo)
        if pw is not None:
            self.k.ConvKernelPrepared(pw, x, xp, y, yp, epilogue=epi, resid=resid, resid_planes=rp, stream=self.stream)
        else:
            self.k.ConvKernelPlanes(x, xp, w, bias, y, yp, *geo, epilogue=epi, resid=resid, resid_planes=rp,
                                    stream=self.stream)

    def pool(self, x, y, *args):
        self.k.PoolingKernel(x, y, *args, stream=self.stream)

    def planes_fill(self, x, p):
        self.k.PlanesFill(p, x, stream=self.stream)

    def pool_planes(self, xp, yp, *args):
        self.k.PoolingKernelPlanes(xp, yp, *args, stream=self.stream)

    def pool_nhwc_planes(self, x, yp, *args):
        self.k.PoolingKernelNhwcPlanes(x, yp, *args[:15], stream=self.stream)

    def pool_nhwc(self, x, y, *args):
        self.k.PoolingKernelNhwc(x, y, *args, stream=self.stream)

    def conv_pool(self, x, w, bias, y, args, epi, resid, pargs):
        self.k.ConvPoolKernel(x, w, bias, y, args, epi, resid, pargs, stream=self.stream)


def weights_key(w, bias, geo) -> tuple:
    """Lookup key of a conv call's prepared weights: its weight and bias buffers and the 17
    geometry scalars."""
    def addr(t):
        return 0 if t is None else (t.data_ptr() if hasattr(t, "data_ptr") else int(t))
    return (addr(w), addr(bias), tuple(int(v) for v in geo))


def matmul_weights_key(b, k, m) -> tuple:
    """Lookup key of a MatMul call's prepared B: its buffer and (k, m)."""
    return ("matmul", b.data_ptr() if hasattr(b, "data_ptr") else int(b), int(k), int(m))


def prepare_weights(net: Net, bufs: dict) -> dict:
    """Prepared weights of the call list, built once from the device buffers `bufs`
    (gpu_buffers) holds: kernels.ConvWeights for every conv and kernels.MatmulWeights for
    every MatMul whose B is a constant shared by its batch steps (a Gemm's weights).  Pass
    the result to GpuBackend so that runs skip the per-call weight preparation.  The
    network's weights are constants; the buffers must keep their values while the result
    is used."""
    from . import kernels
    R = lambda name: None if name is None else bufs[net.resolve(name)]  # noqa: E731
    out = {}
    for node in net.nodes:
        if node[0] == "matmul":
            n, k, m, batch, _, b_bs = node[4][:6]
            if net.resolve(node[2]) in net.consts and (batch == 1 or b_bs == 0):
                b = R(node[2])
                key = matmul_weights_key(b, k, m)
                if key not in out:
                    out[key] = kernels.MatmulWeights(b, k, m)
            continue
        if node[0] != "conv":
            continue
        w, b, geo = R(node[2]), R(node[3]), node[5]
        key = weights_key(w, b, geo)
        if key not in out:
            out[key] = kernels.ConvWeights(w, b, *geo)
    return out


def gpu_buffers(net: Net, x=None):
    """Device buffers for every activation and constant of `net` (torch int16 tensors),
    zeroed: the alignment gaps of strided buffers are never written by the kernels and
    hold 0, as the reference's zero-filled buffer pool does."""
    import torch
    bufs = {}
    for name, words in net.buffers.items():
        bufs[name] = torch.zeros(max(words, 1), dtype=torch.int16, device="cuda")
    for name, arr in net.consts.items():
        bufs[name] = torch.from_numpy(np.ascontiguousarray(arr)).cuda()
    if net.planes:
        from .kernels import PlaneImage
        for name, (n, c, h, w, frame) in net.planes.items():
            bufs[name] = PlaneImage(n, c, h, w, frame)
    if x is not None:
        bufs[net.input].copy_(torch.from_numpy(np.ascontiguousarray(x, np.int16)))
    return bufs
