"""Whole-network parity: the LeNet-5 and ResNet-18-shaped
(config 3) kernel-call lists, run through libcormorant_cuda.so and through the CPU
oracle, must agree word for word on every activation (LeNet) / on the logits of
sampled images at the full batch of 256 (ResNet)."""
import numpy as np
import pytest

import oracle
from cormorant_b200 import networks
from tests._util import assert_same


class OracleBackend:
    """Replays kernel calls on numpy buffers through a CPU checker (port or ref)."""

    def __init__(self, chk):
        self.chk = chk

    def vectorop(self, a, b, c, size, op, outer, a_inc, b_inc):
        c[:] = self.chk.vectorop(a, b, size, op, outer, a_inc, b_inc, c=c.copy())[: c.size]

    def matmul(self, a, b, c, n, k, m, batch, a_bs, b_bs, c_bs):
        # written in place: words between output rows (alignment gaps) keep their values
        c[:] = self.chk.matmul(a, b, n, k, m, batch, a_bs, b_bs, c_bs, c=c.copy())[: c.size]

    def matmul_at(self, a, b, c, a_off, b_off, c_off, n, k, m, batch, a_bs, b_bs, c_bs):
        view = c[c_off:]
        self.matmul(a[a_off:], b[b_off:], view, n, k, m, batch, a_bs, b_bs, c_bs)

    def matmul_fused(self, a, b, c, n, k, m, batch, a_bs, b_bs, c_bs, epi, bias):
        """The reference call sequence MatMul -> [Add(bias row)] -> [Relu] on the checker;
        the output rows are one n x m matrix, or one row per batch step c_bs apart."""
        t = c.copy()
        self.matmul(a, b, t, n, k, m, batch, a_bs, b_bs, c_bs)
        rows, pitch = (n, m) if batch == 1 else (batch, c_bs)
        if epi & 2:
            t = self.chk.vectorop(t, bias, m, networks.OP_ADD, rows, pitch, 0, c=t.copy())[: c.size]
        if epi & 1:
            t = self.chk.vectorop(t, None, c.size, networks.OP_RELU, 1, 0, 0)[: c.size]
        c[:] = t

    def conv(self, x, w, bias, y, *args):
        y[:] = self.chk.conv(x, w, bias, *args)[: y.size]

    def conv_fused(self, x, w, bias, y, *args):
        """The reference call sequence Conv -> [Add(resid)] -> [Relu] on the checker."""
        *geo, epi, resid = args
        t = self.chk.conv(x, w, bias, *geo)[: y.size]
        if epi & 2:
            t = self.chk.vectorop(t, resid, y.size, networks.OP_ADD, 1, 0, 0)[: y.size]
        if epi & 1:
            t = self.chk.vectorop(t, None, y.size, networks.OP_RELU, 1, 0, 0)[: y.size]
        y[:] = t

    def conv_planes(self, x, xp, w, bias, y, yp, *args):
        """A plane image on the checker is the NCHW tensor itself; epilogue bit 3 writes y
        channels-last ([batch][out_h][out_w][out_ch])."""
        *geo, epi, resid, rp = args
        src = x if x is not None else xp
        out = np.zeros(geo[0] * geo[4] * geo[5] * geo[6], np.int16)
        self.conv_fused(src, w, bias, out, *geo, epi & 3, resid if resid is not None else rp)
        if y is not None:
            y[:] = nchw_to_nhwc(out, geo[0], geo[4], geo[5], geo[6]) if epi & networks.EPI_NHWC else out
        if yp is not None:
            yp[:] = out

    def pool(self, x, y, *args):
        y[:] = self.chk.pool(x, *args)[: y.size]

    def planes_fill(self, x, p):
        p[:] = x[: p.size]

    def pool_planes(self, xp, yp, *args):
        self.pool(xp, yp, *args)

    def pool_nhwc_planes(self, x, yp, *args):
        """MAX pool of a channels-last tensor into a plane image (= its NCHW tensor here)."""
        n, c, h, w = args[:4]
        self.pool(nhwc_to_nchw(x, n, c, h, w), yp, *args)

    def conv_pool(self, x, w, bias, y, args, epi, resid, pargs):
        """Conv -> [Add] -> [Relu] -> MaxPool as the reference call sequence."""
        t = np.zeros(args[0] * args[4] * args[5] * args[6], np.int16)
        self.conv_fused(x, w, bias, t, *args, epi, resid)
        self.pool(t, y, *pargs)

    def pool_nhwc(self, x, y, *args):
        """Global pool of a channels-last tensor (its [n][c] output is the same in both layouts)."""
        n, c, h, w = args[:4]
        self.pool(nhwc_to_nchw(x, n, c, h, w), y, *args)


def nchw_to_nhwc(t, n, c, h, w):
    return np.ascontiguousarray(np.asarray(t)[: n * c * h * w].reshape(n, c, h, w).transpose(0, 2, 3, 1)).reshape(-1)


def nhwc_to_nchw(t, n, c, h, w):
    return np.ascontiguousarray(np.asarray(t)[: n * c * h * w].reshape(n, h, w, c).transpose(0, 3, 1, 2)).reshape(-1)


def cpu_buffers(net, x):
    bufs = {name: np.zeros(max(w, 1), np.int16) for name, w in net.buffers.items()}
    bufs.update({name: np.asarray(a, np.int16) for name, a in net.consts.items()})
    for name, (n, c, h, w, _) in net.planes.items():
        bufs[name] = np.zeros(n * c * h * w, np.int16)
    bufs[net.input][:] = x
    return bufs


def test_lenet_macs_and_shapes():
    net = networks.lenet5()
    assert net.macs_per_image == 416520          # the configuration's MAC count
    assert net.buffers[net.resolve(net.output)] == 10


def test_resnet_macs():
    net = networks.resnet18(batch=1)
    assert abs(net.macs_per_image - 1.814e9) / 1.814e9 < 0.01


@pytest.mark.skipif(not oracle.have_ref(), reason="oracle/_ref not built")
def test_lenet_port_equals_reference_cpu(port):
    """The C restatement and the reference kernels agree on the whole LeNet call list."""
    net = networks.lenet5()
    x = networks.make_input(net)
    a, b = cpu_buffers(net, x), cpu_buffers(net, x)
    networks.execute(net, OracleBackend(port), a)
    networks.execute(net, OracleBackend(oracle.ref()), b)
    for name in net.buffers:
        assert_same(a[name], b[name], f"lenet buffer {name}")


@pytest.mark.gpu
def test_lenet_gpu_every_activation(cm, port):
    import torch
    net = networks.lenet5()
    x = networks.make_input(net)
    want = cpu_buffers(net, x)
    networks.execute(net, OracleBackend(port), want)
    bufs = networks.gpu_buffers(net, x)
    networks.execute(net, networks.GpuBackend(), bufs)
    torch.cuda.synchronize()
    for name in net.buffers:
        assert_same(bufs[name].cpu().numpy(), want[name], f"lenet buffer {name}")


@pytest.mark.gpu
def test_resnet18_batch256_sampled_images(cm, port):
    import torch
    net = networks.resnet18(batch=256)
    x = networks.make_input(net)
    bufs = networks.gpu_buffers(net, x)
    networks.execute(net, networks.GpuBackend(), bufs)
    torch.cuda.synchronize()
    logits = bufs[net.resolve(net.output)].cpu().numpy().reshape(256, -1)
    # the same weights (construction order does not depend on the batch), two of the images
    small = networks.resnet18(batch=2)
    per = 3 * 224 * 224
    xs = np.concatenate([x[:per], x[255 * per:256 * per]])
    want = cpu_buffers(small, xs)
    networks.execute(small, OracleBackend(port), want)
    got = np.concatenate([logits[0], logits[255]])
    assert_same(got, want[small.resolve(small.output)], "resnet18 logits of images 0 and 255")
    assert len(np.unique(got)) > 10                       # not a degenerate (saturated) network


def test_fusion_pass_shapes():
    """Conv -> Relu (with residual=True also Conv -> Add -> Relu) and (gemm=True) MatMul ->
    Add(bias row) -> [Relu] chains fold; nothing else changes."""
    def kinds(net):
        return [(n[0], n[6] if n[0] in ("conv", "convpool") and len(n) > 6 else n[5] if n[0] == "matmul" and len(n) > 5
                 else None) for n in net.nodes]
    rn = kinds(networks.fuse(networks.resnet18(batch=1), residual=True))
    assert rn.count(("conv", 1)) == 9 and rn.count(("conv", 3)) == 8 and rn.count(("conv", None)) == 3
    assert rn.count(("matmul", 2)) == 1 and rn.count(("vectorop", None)) == 0    # classifier: MatMul+Add
    rn = kinds(networks.fuse(networks.resnet18(batch=1), residual=False, gemm=False))
    assert rn.count(("conv", 1)) == 9 and rn.count(("conv", None)) == 11 and rn.count(("vectorop", None)) == 17
    assert rn.count(("matmul", None)) == 1
    ln = networks.fuse(networks.lenet5())
    assert kinds(ln) == [("convpool", 1), ("convpool", 1), ("matmul", 3), ("matmul", 3), ("matmul", 2)]
    ln = networks.fuse(networks.lenet5(), conv_pool_macs=0)
    assert kinds(ln) == [("conv", 1), ("pool", None), ("conv", 1), ("pool", None), ("matmul", 3), ("matmul", 3),
                         ("matmul", 2)]
    assert ln.source_kinds == ("conv", "matmul", "pool", "vectorop")
    ln = networks.fuse(networks.lenet5(), gemm=False)
    assert [n[0] for n in ln.nodes].count("vectorop") == 5 and all(len(n) == 8 for n in ln.nodes if n[0] == "conv")


def test_fused_call_list_equals_reference_sequence_on_cpu(port):
    """The folded LeNet call list, replayed on the checker with the reference's call
    sequence for each fused conv, gives the same logits as the original list."""
    net = networks.lenet5()
    fn = networks.fuse(net)
    x = networks.make_input(net)
    a, b = cpu_buffers(net, x), cpu_buffers(fn, x)
    networks.execute(net, OracleBackend(port), a)
    networks.execute(fn, OracleBackend(port), b)
    assert_same(b[fn.resolve(fn.output)], a[net.resolve(net.output)], "fused lenet logits")


@pytest.mark.gpu
def test_lenet_fused_gpu_every_activation(cm, port):
    net = networks.fuse(networks.lenet5())
    x = networks.make_input(net)
    want = cpu_buffers(net, x)
    networks.execute(net, OracleBackend(port), want)
    for limit in (0, 1 << 26):                  # tensor-core and CUDA-core conv paths
        old = cm.lib().cm_set_direct_limit(limit)
        try:
            bufs = networks.gpu_buffers(net, x)
            networks.execute(net, networks.GpuBackend(), bufs)
            import torch
            torch.cuda.synchronize()
        finally:
            cm.lib().cm_set_direct_limit(old)
        for name in net.buffers:
            assert_same(bufs[name].cpu().numpy(), want[name], f"fused lenet buffer {name} (direct limit {limit})")


@pytest.mark.gpu
def test_resnet18_fused_batch256_sampled_images(cm, port):
    import torch
    net = networks.fuse(networks.resnet18(batch=256), residual=True)
    x = networks.make_input(net)
    bufs = networks.gpu_buffers(net, x)
    networks.execute(net, networks.GpuBackend(), bufs)
    torch.cuda.synchronize()
    logits = bufs[net.resolve(net.output)].cpu().numpy().reshape(256, -1)
    small = networks.resnet18(batch=2)                    # the unfused reference call list
    per = 3 * 224 * 224
    xs = np.concatenate([x[:per], x[255 * per:256 * per]])
    want = cpu_buffers(small, xs)
    networks.execute(small, OracleBackend(port), want)
    got = np.concatenate([logits[0], logits[255]])
    assert_same(got, want[small.resolve(small.output)], "fused resnet18 logits of images 0 and 255")


def test_chain_pass_resnet_structure():
    """Conv outputs read by implicit-GEMM convs become plane images; NCHW outputs stay only
    where a residual, a pool or the network output reads them.  The stem writes its output
    channels-last for the max pool, which writes the layer-1 convs' plane image."""
    net = networks.chain(networks.fuse(networks.resnet18(batch=2)))
    convs = [n for n in net.nodes if n[0] == "conv"]
    assert len(convs) == 20 and len(net.planes) == 19
    assert [n[0] for n in net.nodes[:2]] == ["conv", "poolnp"]
    assert convs[0][6] == 1 | networks.EPI_NHWC and net.nodes[1][1:3] == ("relu4", "pool5@planes")
    assert not [n for n in net.nodes if n[0] == "planes"]       # no split pass left
    assert sum(1 for n in convs if n[8] is not None) == 19      # every conv but the stem
    assert sum(1 for n in convs if n[1] is None) == 19          # inputs read only from plane images
    assert sum(1 for n in convs if n[4] is None) == 18          # outputs written only as plane images
    assert sum(1 for n in convs if n[10] is not None) == 8      # residuals read from plane images
    assert sum(1 for n in convs if n[7] is not None) == 0       # no residual read as NCHW
    assert all(n[8] is not None for n in convs if n[1] is None)
    assert all(n[9] is not None for n in convs if n[4] is None)
    assert set(net.buffers) == {"x", "relu4", "relu86", "pool87", "gemm92"}   # relu4, relu86 channels-last
    assert [n[0] for n in net.nodes[-3:-1]] == ["conv", "poolng"]       # the last block's conv -> global pool
    assert net.nodes[-3][6] == 3 | networks.EPI_NHWC and net.nodes[-2][1:3] == ("relu86", "pool87")
    old = networks.chain(networks.fuse(networks.resnet18(batch=2)), pool_nhwc=False)
    assert [n[1] for n in old.nodes if n[0] == "planes"] == ["pool5"]   # the max pool's output, split once
    assert set(old.buffers) == {"x", "relu4", "pool5", "relu86", "pool87", "gemm92"}
    pp = networks.chain(networks.fuse(networks.resnet18(batch=2)), pool_planes=True, pool_nhwc=False)
    assert [n[0] for n in pp.nodes[:2]] == ["conv", "poolp"] and len(pp.planes) == 20
    assert set(pp.buffers) == {"x", "relu86", "pool87", "gemm92"}
    for name, (b, c, h, w, frame) in net.planes.items():
        assert b == 2 and len(frame) == 4 and min(frame) >= 0
    assert networks.chain(networks.fuse(networks.lenet5())).planes == {}    # batch-1 convs read NCHW


def test_chained_call_list_equals_reference_sequence_on_cpu(port):
    """The plane-chained ResNet call list, replayed on the checker (a plane image = its
    NCHW tensor), gives the unchained list's logits."""
    net = networks.resnet18(batch=1)
    fn = networks.chain(networks.fuse(net), frame_fn=lambda a: (1, 1, 1, 1) if a[7] > 1 and a[9] == 1 else None,
                        nhwc_fn=lambda a: a[7] == 7)
    assert [n[0] for n in fn.nodes[:2]] == ["conv", "poolnp"]
    x = networks.make_input(net)
    a, b = cpu_buffers(net, x), cpu_buffers(fn, x)
    networks.execute(net, OracleBackend(port), a)
    networks.execute(fn, OracleBackend(port), b)
    assert_same(b[fn.resolve(fn.output)], a[net.resolve(net.output)], "chained resnet logits")


@pytest.mark.gpu
@pytest.mark.parametrize("pool_planes,prepared", [(False, False), (True, False), (False, True)])
def test_resnet18_chained_batch4_every_output(cm, port, pool_planes, prepared):
    """Plane images on the GPU: every NCHW tensor the chained list still writes, and the
    logits, equal the oracle's (also with the conv and Gemm weights prepared once)."""
    import torch
    from cormorant_b200 import kernels
    net = networks.chain(networks.fuse(networks.resnet18(batch=4)), pool_planes=pool_planes, pool_nhwc=not pool_planes)
    assert net.planes
    assert [n[0] for n in net.nodes[:2]] == ["conv", "poolp" if pool_planes else "poolnp"]
    x = networks.make_input(net)
    want = cpu_buffers(net, x)
    networks.execute(net, OracleBackend(port), want)
    bufs = networks.gpu_buffers(net, x)
    weights = networks.prepare_weights(net, bufs) if prepared else None
    if prepared:
        # every conv's weights and the classifier Gemm's B (a constant)
        assert len(weights) == sum(1 for n in net.nodes if n[0] == "conv") + 1
        assert sum(1 for w in weights.values() if isinstance(w, kernels.MatmulWeights)) == 1
    networks.execute(net, networks.GpuBackend(weights=weights), bufs)
    torch.cuda.synchronize()
    for name in net.buffers:
        assert_same(bufs[name].cpu().numpy()[: net.buffers[name]], want[name][: net.buffers[name]], f"resnet {name}")


def test_one_launch_call_list_qualifies_on_cpu():
    """LeNet's folded call list runs in one cm_calls launch; ResNet-18's does not (too large)."""
    from cormorant_b200 import kernels
    net = networks.fuse(networks.lenet5(), conv_pool_macs=0)
    fake = {n: 256 * (i + 1) for i, n in enumerate(list(net.buffers) + list(net.consts))}
    arr = kernels.call_array(networks.calls_of(net, fake))
    assert len(arr) == 7 and kernels.calls_supported(arr)
    rn = networks.fuse(networks.resnet18(batch=1))
    calls = networks.calls_of(rn, {n: 256 for n in list(rn.buffers) + list(rn.consts)})
    assert len(calls) > kernels.CALLS_MAX or not kernels.calls_supported(kernels.call_array(calls[:24]))
    # a DIV or an AVG pool is refused
    bad = [(kernels.CALL_VECTOROP, 0, 256, 512, None, None, 768, (16, 3, 1, 0, 0))]
    assert not kernels.calls_supported(kernels.call_array(bad))
    bad = [(kernels.CALL_POOL, 0, 256, None, None, None, 768, (1, 1, 4, 4, 2, 2, 2, 2, 2, 2, 0, 0, 1, 1, 1, 2, 0))]
    assert not kernels.calls_supported(kernels.call_array(bad))


@pytest.mark.gpu
@pytest.mark.parametrize("batch", [1, 3])
def test_lenet_one_launch_every_activation(cm, port, batch):
    import torch
    net = networks.fuse(networks.lenet5(batch=batch), conv_pool_macs=0)
    x = networks.make_input(net)
    want = cpu_buffers(net, x)
    networks.execute(net, OracleBackend(port), want)
    bufs = networks.gpu_buffers(net, x)
    l0 = cm.launch_count()
    be = networks.GpuBackend(one_launch=True)
    networks.execute(net, be, bufs)
    torch.cuda.synchronize()
    assert cm.launch_count() - l0 == 1
    for name in net.buffers:
        assert_same(bufs[name].cpu().numpy()[: net.buffers[name]], want[name][: net.buffers[name]], f"lenet {name}")


# ---- the scheduler edge-case graphs (tests/golden/scheduler_graphs.py) ------------
def _edge_graphs():
    from tests.golden.scheduler_graphs import GRAPHS
    return {k: f for k, f in GRAPHS.items() if not k.startswith(("lenet", "resnet"))}


@pytest.mark.parametrize("name", sorted(_edge_graphs()))
def test_edge_graph_reference_cpu_equals_port(port, name):
    """The derived call lists of the edge-case graphs (broadcast gaps, MatMul batch forms and
    outer loop, row-strided MatMul, conv and pool forms) on the C restatement and on the
    reference's own kernels: every buffer equal."""
    if not oracle.have_ref():
        pytest.skip("oracle/_ref not built")
    from cormorant_b200 import scheduler
    net = scheduler.derive(_edge_graphs()[name]())
    x = np.random.default_rng(3).integers(-1024, 1024, net.buffers[net.input]).astype(np.int16)
    a, b = cpu_buffers(net, x), cpu_buffers(net, x)
    networks.execute(net, OracleBackend(port), a)
    networks.execute(net, OracleBackend(oracle.ref()), b)
    for buf in net.buffers:
        assert_same(a[buf], b[buf], f"{name} buffer {buf}")


@pytest.mark.gpu
@pytest.mark.usefixtures("mac_path")
@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("name", sorted(_edge_graphs()))
def test_edge_graph_gpu_every_buffer(cm, port, name, fused):
    """The same call lists (and their fused forms) through the C ABI on the GPU, every buffer
    bit-exact against the oracle, on both MatMul / Conv paths."""
    import torch
    from cormorant_b200 import scheduler
    net = scheduler.derive(_edge_graphs()[name]())
    if fused:
        net = networks.fuse(net)
    x = np.random.default_rng(3).integers(-1024, 1024, net.buffers[net.input]).astype(np.int16)
    want = cpu_buffers(net, x)
    networks.execute(net, OracleBackend(port), want)
    bufs = networks.gpu_buffers(net, x)
    networks.execute(net, networks.GpuBackend(), bufs)
    torch.cuda.synchronize()
    for buf in net.buffers:
        assert_same(bufs[buf].cpu().numpy(), want[buf], f"{name} buffer {buf}")
