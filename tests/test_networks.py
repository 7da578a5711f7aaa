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
        c[:] = self.chk.matmul(a, b, n, k, m, batch, a_bs, b_bs, c_bs)[: c.size]

    def conv(self, x, w, bias, y, *args):
        y[:] = self.chk.conv(x, w, bias, *args)[: y.size]

    def pool(self, x, y, *args):
        y[:] = self.chk.pool(x, *args)[: y.size]


def cpu_buffers(net, x):
    bufs = {name: np.zeros(max(w, 1), np.int16) for name, w in net.buffers.items()}
    bufs.update({name: np.asarray(a, np.int16) for name, a in net.consts.items()})
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
