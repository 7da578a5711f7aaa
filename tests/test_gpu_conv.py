"""ConvKernel parity on the GPU: cm_conv (im2col split + tcgen05 GEMM; depthwise on
CUDA cores) vs the C restatement, bit-exact on raw int16 words.

The case list mirrors the reference's TestConvSim.cpp:284-628 geometries
(1x1, 3x3 with/without padding, stride 2, bias, batch, partial channel tiles,
dilation, 5x5, multi-tile, non-square, asymmetric padding, depthwise variants,
saturation), then adds the LeNet and ResNet-18 layer shapes of the BASELINE
configs and edge cases (empty reduction, wide reductions, full-range data).
"""
import numpy as np
import pytest

from tests._util import assert_same, dev, empty, host, rand16

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("mac_path")]


def osz(n, k, s, d, p0, p1):
    return (n + p0 + p1 - (d * (k - 1) + 1)) // s + 1


# (N, C, H, W, M, kh, kw, sh, sw, dh, dw, pt, pl, pb, pr, bias, dw_mode)
REF_CASES = [
    (1, 1, 5, 5, 1, 1, 1, 1, 1, 1, 1, 0, 0, 0, 0, 0, 0),
    (1, 1, 5, 5, 1, 3, 3, 1, 1, 1, 1, 0, 0, 0, 0, 0, 0),
    (1, 1, 5, 5, 1, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 0, 0),
    (1, 1, 6, 6, 1, 3, 3, 2, 2, 1, 1, 0, 0, 0, 0, 0, 0),
    (1, 1, 5, 5, 2, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0),
    (2, 1, 5, 5, 1, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 0, 0),
    (1, 21, 5, 5, 1, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 0, 0),
    (1, 1, 5, 5, 11, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0),
    (1, 1, 9, 9, 1, 3, 3, 1, 1, 2, 2, 0, 0, 0, 0, 0, 0),
    (1, 1, 7, 7, 1, 5, 5, 1, 1, 1, 1, 0, 0, 0, 0, 0, 0),
    (1, 35, 14, 14, 17, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0),
    (1, 1, 6, 8, 2, 3, 5, 1, 1, 1, 1, 0, 0, 0, 0, 0, 0),
    (1, 1, 7, 7, 1, 3, 3, 2, 2, 1, 1, 1, 1, 0, 0, 0, 0),
    (1, 4, 8, 8, 4, 3, 3, 1, 1, 1, 1, 0, 0, 0, 0, 0, 1),
    (1, 4, 8, 8, 4, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1),
    (1, 11, 6, 6, 11, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 0, 1),
    (1, 4, 9, 9, 4, 3, 3, 1, 1, 2, 2, 0, 0, 0, 0, 0, 1),
    (1, 8, 8, 8, 8, 3, 3, 2, 2, 1, 1, 1, 1, 1, 1, 0, 1),
    # LeNet-5 layers (config 0) and ResNet-18 layer shapes (config 3) at small batch
    (1, 1, 28, 28, 6, 5, 5, 1, 1, 1, 1, 2, 2, 2, 2, 1, 0),
    (1, 6, 14, 14, 16, 5, 5, 1, 1, 1, 1, 0, 0, 0, 0, 1, 0),
    (2, 3, 224, 224, 64, 7, 7, 2, 2, 1, 1, 3, 3, 3, 3, 1, 0),
    (2, 64, 56, 56, 64, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0),
    (2, 64, 56, 56, 128, 3, 3, 2, 2, 1, 1, 1, 1, 1, 1, 1, 0),
    (2, 64, 56, 56, 128, 1, 1, 2, 2, 1, 1, 0, 0, 0, 0, 1, 0),
    (2, 256, 14, 14, 512, 3, 3, 2, 2, 1, 1, 1, 1, 1, 1, 1, 0),
    (2, 512, 7, 7, 512, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0),
    # odd shapes: K not a multiple of 16, stride > kernel, dilation with padding
    (3, 5, 13, 11, 7, 2, 3, 3, 2, 2, 3, 1, 2, 0, 1, 1, 0),
    (1, 130, 9, 9, 129, 1, 1, 1, 1, 1, 1, 0, 0, 0, 0, 1, 0),
    # implicit-GEMM geometry (channels-last planes, TMA box per kernel row): 1x1 stride-2
    # shortcut, kw*C exactly 128 with row dilation, partial channel tile with images
    # past the batch in the last tile, output rows wider than one tile, strides 3 and 8
    (3, 128, 14, 14, 256, 1, 1, 2, 2, 1, 1, 0, 0, 0, 0, 1, 0),
    (2, 32, 9, 13, 40, 3, 4, 1, 2, 2, 1, 2, 1, 1, 0, 1, 0),
    (5, 64, 7, 7, 100, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 0, 0),
    (1, 96, 20, 150, 24, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0),
    (2, 64, 40, 40, 16, 3, 3, 3, 8, 1, 1, 1, 1, 0, 0, 1, 0),
    # explicit im2col (rows = pixels of several images): column dilation with more than
    # 64 output channels, and narrow input channels with row tiles spanning images
    (2, 5, 17, 19, 96, 3, 3, 1, 2, 2, 2, 2, 2, 2, 2, 1, 0),
    (4, 3, 30, 30, 24, 5, 5, 2, 2, 1, 1, 2, 2, 2, 2, 1, 0),
    # explicit im2col whose shared-memory window does not fit (direct gather), and one
    # whose output rows are wider than a window block
    (1, 600, 9, 300, 8, 3, 3, 1, 1, 1, 2, 1, 2, 1, 2, 1, 0),
    (2, 3, 11, 300, 20, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0),
    # space-to-depth form (stride s in both directions, s*s*C channels): odd sizes with
    # asymmetric padding, more than 64 output channels, stride 4
    (2, 3, 35, 29, 40, 7, 7, 2, 2, 1, 1, 3, 2, 3, 1, 1, 0),
    (1, 4, 33, 33, 100, 5, 5, 2, 2, 1, 1, 2, 2, 2, 2, 1, 0),
    (2, 2, 26, 26, 16, 4, 4, 4, 4, 1, 1, 1, 1, 1, 1, 1, 0),
    # maps with H*W not a multiple of 4: whole image in shared memory (odd word count, no
    # padding, asymmetric padding) and one whose image is too large for it
    (3, 37, 9, 7, 70, 3, 3, 1, 1, 1, 1, 0, 0, 0, 0, 1, 0),
    (2, 200, 5, 5, 130, 3, 3, 1, 1, 1, 1, 2, 1, 0, 1, 1, 0),
    (1, 1100, 7, 7, 8, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0),
]


def run(cm, port, case, dist, seed):
    N, C, H, W, M, kh, kw, sh, sw, dh, dw_, pt, pl, pb, pr, hb, dwm = case
    oh, ow = osz(H, kh, sh, dh, pt, pb), osz(W, kw, sw, dw_, pl, pr)
    rng = np.random.default_rng(seed)
    lo, hi = (-256, 256) if dist == "q8" else (-32768, 32768)
    x = rand16(rng, N * C * H * W, lo, hi)
    w = rand16(rng, M * (1 if dwm else C) * kh * kw, lo, hi)
    bias = rand16(rng, M, lo, hi)
    y = empty(N * M * oh * ow)
    cm.ConvKernel(dev(x), dev(w), dev(bias) if hb else None, y, N, C, H, W, M, oh, ow, kh, kw, sh, sw, dh, dw_, pt,
                  pl, hb, dwm)
    want = port.conv(x, w, bias if hb else None, N, C, H, W, M, oh, ow, kh, kw, sh, sw, dh, dw_, pt, pl, hb, dwm)
    assert_same(host(y), want, f"case {case} {dist}")


@pytest.mark.parametrize("case", REF_CASES)
@pytest.mark.parametrize("dist", ["q8", "full"])
def test_cases(cm, port, case, dist):
    run(cm, port, case, dist, seed=sum(case) * 13 + (dist == "full"))


def test_small_map_unaligned_input(cm, port):
    """A 7x7 input that starts 2 bytes past a 4-byte boundary (the whole-image split then
    reads 2-byte words)."""
    N, C, H, W, M = 3, 96, 7, 7, 80
    rng = np.random.default_rng(77)
    x = rand16(rng, N * C * H * W)
    w = rand16(rng, M * C * 9)
    b = rand16(rng, M)
    xd = dev(np.concatenate([np.zeros(1, np.int16), x]))[1:]
    y = empty(N * M * H * W)
    cm.ConvKernel(xd, dev(w), dev(b), y, N, C, H, W, M, H, W, 3, 3, 1, 1, 1, 1, 1, 1)
    assert_same(host(y), port.conv(x, w, b, N, C, H, W, M, H, W, 3, 3, 1, 1, 1, 1, 1, 1), "unaligned 7x7")


@pytest.mark.parametrize("w_val,b_val,sat", [(256, 32767, 32767), (-256, -32768, -32768)])
def test_saturation(cm, port, w_val, b_val, sat):
    """TestConvSim.cpp:594-628: x = AP_MAX, w = +-1.0, bias = AP_MAX / AP_MIN saturates."""
    x = np.full(9, 32767, np.int16)
    w = np.array([w_val], np.int16)
    b = np.array([b_val], np.int16)
    y = empty(9)
    cm.ConvKernel(dev(x), dev(w), dev(b), y, 1, 1, 3, 3, 1, 3, 3, 1, 1)
    got = host(y)
    assert (got == sat).all()
    assert_same(got, port.conv(x, w, b, 1, 1, 3, 3, 1, 3, 3, 1, 1), "saturation")


def test_empty_reduction_writes_bias(cm, port):
    b = np.array([5, -7, 300], np.int16)
    y = empty(2 * 3 * 4)
    cm.ConvKernel(dev(np.zeros(1, np.int16)), dev(np.zeros(1, np.int16)), dev(b), y, 2, 0, 2, 2, 3, 2, 2, 1, 1)
    assert_same(host(y), np.tile(np.repeat(b, 4), 2), "in_ch = 0")


@pytest.mark.big
def test_resnet_conv1_batch8_sampled(cm, port):
    """ResNet-18 stem at batch 8 (chunked im2col), checked plane by plane for a sample of (n, m)."""
    N, C, H, W, M = 8, 3, 224, 224, 64
    rng = np.random.default_rng(77)
    x = rand16(rng, N * C * H * W, 0, 256)
    w = rand16(rng, M * C * 49, -128, 128)
    bias = rand16(rng, M, -64, 64)
    y = empty(N * M * 112 * 112)
    cm.ConvKernel(dev(x), dev(w), dev(bias), y, N, C, H, W, M, 112, 112, 7, 7, 2, 2, 1, 1, 3, 3, 1, 0)
    nidx = rng.integers(0, N, 24)
    midx = rng.integers(0, M, 24)
    want = port.conv_planes(x, w, bias, C, H, W, M, 112, 112, 7, 7, 2, 2, 1, 1, 3, 3, 1, 0, nidx, midx)
    got = host(y).reshape(N, M, -1)[nidx, midx]
    assert_same(got, want, "stem sampled planes")


FUSED = [  # implicit GEMM (several layouts), explicit im2col (stem-like), 1x1 output plane
    (2, 64, 14, 14, 64, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0),
    (2, 64, 15, 15, 128, 3, 3, 2, 2, 1, 1, 1, 1, 1, 1, 1, 0),
    (2, 3, 30, 30, 24, 7, 7, 2, 2, 1, 1, 3, 3, 3, 3, 1, 0),
    (3, 32, 3, 3, 70, 3, 3, 1, 1, 1, 1, 0, 0, 0, 0, 1, 0),
    (2, 4, 8, 8, 4, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1),     # depthwise: epilogue pass
]


@pytest.mark.parametrize("case", FUSED)
@pytest.mark.parametrize("epi", [1, 2, 3])
def test_conv_fused_epilogue(cm, port, case, epi):
    """cm_conv_fused == ConvKernel then VectorOP ADD (residual) and/or RELU, word for word."""
    from cormorant_b200 import kernels
    N, C, H, W, M, kh, kw, sh, sw, dh, dw_, pt, pl, pb, pr, hb, dwm = case
    oh, ow = osz(H, kh, sh, dh, pt, pb), osz(W, kw, sw, dw_, pl, pr)
    rng = np.random.default_rng(sum(case) + epi)
    x = rand16(rng, N * C * H * W, -2048, 2048)
    w = rand16(rng, M * (1 if dwm else C) * kh * kw, -512, 512)
    bias = rand16(rng, M, -2048, 2048)
    r = rand16(rng, N * M * oh * ow)
    y = empty(N * M * oh * ow)
    kernels.ConvKernelFused(dev(x), dev(w), dev(bias), y, N, C, H, W, M, oh, ow, kh, kw, sh, sw, dh, dw_, pt, pl, hb,
                            dwm, epilogue=epi, resid=dev(r))
    size = N * M * oh * ow
    want = port.conv(x, w, bias, N, C, H, W, M, oh, ow, kh, kw, sh, sw, dh, dw_, pt, pl, hb, dwm)[:size]
    if epi & 2:
        want = port.vectorop(want, r, size, 0, 1, 0, 0)[:size]
    if epi & 1:
        want = port.vectorop(want, None, size, 4, 1, 0, 0)[:size]
    assert_same(host(y), want, f"fused {case} epi {epi}")


# conv (N, C, H, W, M, kh, kw, sh, sw, dh, dw, pt, pl, pb, pr, bias) and MAX pool (ph, pw, sh, sw, pt, pl, dh, dw)
CONV_POOL = [
    ((1, 1, 28, 28, 6, 5, 5, 1, 1, 1, 1, 2, 2, 2, 2, 1), (2, 2, 2, 2, 0, 0, 1, 1)),     # LeNet conv1 + pool
    ((1, 6, 14, 14, 16, 5, 5, 1, 1, 1, 1, 0, 0, 0, 0, 1), (2, 2, 2, 2, 0, 0, 1, 1)),    # LeNet conv2 + pool
    ((3, 4, 13, 11, 5, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 0), (3, 3, 2, 2, 1, 1, 1, 1)),     # overlapping padded windows
    ((2, 3, 17, 15, 7, 3, 2, 2, 1, 2, 1, 2, 0, 1, 1, 1), (2, 3, 1, 2, 0, 1, 2, 1)),     # dilations, odd strides
]


@pytest.mark.parametrize("case", CONV_POOL)
@pytest.mark.parametrize("epi", [0, 1, 3])
def test_conv_pool_one_launch(cm, port, case, epi):
    """cm_conv_pool == ConvKernel, then VectorOP ADD / RELU, then a MAX PoolingKernel, word for word."""
    from cormorant_b200 import kernels
    (N, C, H, W, M, kh, kw, sh, sw, dh, dw_, pt, pl, pb, pr, hb), (ph, pw, psh, psw, ppt, ppl, pdh, pdw) = case
    oh, ow = osz(H, kh, sh, dh, pt, pb), osz(W, kw, sw, dw_, pl, pr)
    qh, qw = osz(oh, ph, psh, pdh, ppt, ppt), osz(ow, pw, psw, pdw, ppl, ppl)
    rng = np.random.default_rng(sum(case[0]) + sum(case[1]) + epi)
    x = rand16(rng, N * C * H * W, -2048, 2048)
    w = rand16(rng, M * C * kh * kw, -512, 512)
    bias = rand16(rng, M, -2048, 2048)
    r = rand16(rng, N * M * oh * ow)
    conv_args = (N, C, H, W, M, oh, ow, kh, kw, sh, sw, dh, dw_, pt, pl, hb, 0)
    pool_args = (N, M, oh, ow, qh, qw, ph, pw, psh, psw, ppt, ppl, pdh, pdw, 0, 2, 0)
    size = N * M * oh * ow
    t = port.conv(x, w, bias, *conv_args)[:size]
    if epi & 2:
        t = port.vectorop(t, r, size, 0, 1, 0, 0)[:size]
    if epi & 1:
        t = port.vectorop(t, None, size, 4, 1, 0, 0)[:size]
    want = port.pool(t, *pool_args)[: N * M * qh * qw]
    y = empty(N * M * qh * qw)
    kernels.ConvPoolKernel(dev(x), dev(w), dev(bias), y, conv_args, epi, dev(r), pool_args)
    assert_same(host(y), want, f"conv+pool {case} epi {epi}")


def test_conv_pool_refusals(cm):
    """An AVG pool, or a pool whose input is not the conv's output, is refused."""
    from cormorant_b200 import kernels
    conv_args = (1, 1, 8, 8, 2, 8, 8, 3, 3, 1, 1, 1, 1, 1, 1, 0, 0)
    x, w = dev(np.zeros(64, np.int16)), dev(np.zeros(18, np.int16))
    with pytest.raises(cm.CormorantError):
        kernels.ConvPoolKernel(x, w, None, empty(32), conv_args, 0, None, (1, 2, 8, 8, 4, 4, 2, 2, 2, 2, 0, 0, 1, 1, 1, 2, 0))
    with pytest.raises(cm.CormorantError):
        kernels.ConvPoolKernel(x, w, None, empty(32), conv_args, 0, None, (1, 2, 7, 8, 4, 4, 2, 2, 2, 2, 0, 0, 1, 1, 0, 2, 0))


PREPARED = [REF_CASES[i] for i in (4, 13, 19, 20, 21, 24, 25, 34, 36, 39, 42)]


@pytest.mark.parametrize("case", PREPARED)
@pytest.mark.parametrize("epi", [0, 3])
def test_prepared_weights_match_reference(cm, port, case, epi):
    """cm_conv_prepared with weights prepared once (every conv path: CUDA-core small and
    depthwise convs, implicit GEMM, space-to-depth, explicit im2col) equals the reference
    conv (+ residual Add + Relu), word for word, over repeated calls."""
    from cormorant_b200 import kernels
    N, C, H, W, M, kh, kw, sh, sw, dh, dw_, pt, pl, pb, pr, hb, dwm = case
    oh, ow = osz(H, kh, sh, dh, pt, pb), osz(W, kw, sw, dw_, pl, pr)
    rng = np.random.default_rng(sum(case) * 3 + epi)
    x = rand16(rng, N * C * H * W, -2048, 2048)
    w = rand16(rng, M * (1 if dwm else C) * kh * kw, -512, 512)
    bias = rand16(rng, M, -2048, 2048)
    r = rand16(rng, N * M * oh * ow)
    size = N * M * oh * ow
    want = port.conv(x, w, bias if hb else None, N, C, H, W, M, oh, ow, kh, kw, sh, sw, dh, dw_, pt, pl, hb, dwm)[:size]
    if epi & 2:
        want = port.vectorop(want, r, size, 0, 1, 0, 0)[:size]
    if epi & 1:
        want = port.vectorop(want, None, size, 4, 1, 0, 0)[:size]
    wd, bd = dev(w), dev(bias) if hb else None
    pw = kernels.ConvWeights(wd, bd, N, C, H, W, M, oh, ow, kh, kw, sh, sw, dh, dw_, pt, pl, hb, dwm)
    for rep in range(2):
        y = empty(size)
        kernels.ConvKernelPrepared(pw, dev(x), None, y, None, epilogue=epi, resid=dev(r) if epi & 2 else None)
        assert_same(host(y), want, f"prepared {case} epi {epi} call {rep}")
    pw.close()


def test_prepared_weights_follow_the_direct_limit(cm, port):
    """A conv prepared for the tensor-core path and then called with the CUDA-core limit
    raised past it takes the CUDA-core path with the live weights: the same words."""
    from cormorant_b200 import _lib, kernels
    case = (2, 64, 14, 14, 64, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0)
    N, C, H, W, M, kh, kw, sh, sw, dh, dw_, pt, pl, pb, pr, hb, dwm = case
    rng = np.random.default_rng(5)
    x, w, bias = rand16(rng, N * C * H * W), rand16(rng, M * C * 9, -512, 512), rand16(rng, M)
    want = port.conv(x, w, bias, N, C, H, W, M, H, W, 3, 3, 1, 1, 1, 1, 1, 1, 1, 0)[: N * M * H * W]
    L = _lib.lib()
    old = L.cm_set_direct_limit(0)
    try:
        pw = kernels.ConvWeights(dev(w), dev(bias), N, C, H, W, M, H, W, 3, 3, 1, 1, 1, 1, 1, 1, 1, 0)
        L.cm_set_direct_limit(1 << 40)
        y = empty(N * M * H * W)
        kernels.ConvKernelPrepared(pw, dev(x), None, y, None)
    finally:
        L.cm_set_direct_limit(old)
    assert_same(host(y), want, "prepared weights, CUDA-core path at call time")


ONE_LAUNCH_CASES = [
    (1, 1, 28, 28, 6, 5, 5, 1, 1, 1, 1, 2, 2, 2, 2, 1, 0),
    (2, 6, 14, 14, 16, 5, 5, 1, 1, 1, 1, 0, 0, 0, 0, 1, 0),
    (3, 5, 13, 11, 7, 2, 3, 3, 2, 2, 3, 1, 2, 0, 1, 1, 0),
    (1, 8, 8, 8, 8, 3, 3, 2, 2, 1, 1, 1, 1, 1, 1, 0, 1),
]


@pytest.mark.parametrize("case", ONE_LAUNCH_CASES)
@pytest.mark.parametrize("epi", [0, 3])
def test_one_launch_conv_and_pool_match_entries(cm, port, case, epi):
    """cm_calls' conv (with the fused epilogue) and MAX pool equal cm_conv_fused / cm_pool."""
    from cormorant_b200 import kernels
    N, C, H, W, M, kh, kw, sh, sw, dh, dw_, pt, pl, pb, pr, hb, dwm = case
    oh, ow = osz(H, kh, sh, dh, pt, pb), osz(W, kw, sw, dw_, pl, pr)
    rng = np.random.default_rng(sum(case) + epi)
    x = rand16(rng, N * C * H * W)
    w = rand16(rng, M * (1 if dwm else C) * kh * kw)
    b = rand16(rng, M)
    r = rand16(rng, N * M * oh * ow)
    args = (N, C, H, W, M, oh, ow, kh, kw, sh, sw, dh, dw_, pt, pl, hb, dwm)
    y1, y2 = empty(N * M * oh * ow), empty(N * M * oh * ow)
    cm.ConvKernelFused(dev(x), dev(w), dev(b) if hb else None, y1, *args, epilogue=epi, resid=dev(r) if epi else None)
    ph = (oh + 1) // 2
    pool_args = (N, M, oh, ow, ph, (ow + 1) // 2, 3, 3, 2, 2, 1, 1, 1, 1, 0, 2, 0)
    p1 = empty(N * M * ph * ((ow + 1) // 2))
    p2 = empty(p1.numel())
    cm.PoolingKernel(y1, p1, *pool_args)
    arr = kernels.call_array([(kernels.CALL_CONV, epi, dev(x), dev(w), dev(b) if hb else None,
                               dev(r) if epi else None, y2, args),
                              (kernels.CALL_POOL, 0, y2, None, None, None, p2, pool_args)])
    assert kernels.calls_supported(arr)
    kernels.RunCalls(arr)
    assert_same(host(y2), host(y1), f"one-launch conv {case} epi {epi}")
    assert_same(host(p2), host(p1), f"one-launch pool after {case}")


# K-split tensor-core GEMMs: a tile's K blocks shared among units whose int32 partial sums
# add up (wrapping) before the one narrowing -- (N, C, H, W, M, kh, kw, sh, sw, dh, dw, pt,
# pl, pb, pr, bias, depthwise)
KSPLIT = [
    (2, 512, 7, 7, 512, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0),     # one row tile: single-CTA 128-column tiles
    (8, 256, 14, 14, 256, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0),   # CTA-pair tiles
    (4, 64, 28, 28, 48, 3, 3, 2, 2, 1, 1, 1, 1, 1, 1, 1, 0),     # packed 64-column tiles
    (3, 100, 9, 9, 200, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 0, 0),     # partial column tiles, no bias
]


@pytest.mark.parametrize("case", KSPLIT)
@pytest.mark.parametrize("splits", [0, 2, 3, 4])
@pytest.mark.parametrize("epi", [0, 3])
def test_k_split_units(cm, port, case, splits, epi):
    """Every K-split setting (0 = never; 2-4 units per tile) gives the reference words,
    with and without the fused residual Add + Relu; full-range words so the int32
    partial sums wrap."""
    from cormorant_b200 import _lib, kernels
    N, C, H, W, M, kh, kw, sh, sw, dh, dw_, pt, pl, pb, pr, hb, dwm = case
    oh, ow = osz(H, kh, sh, dh, pt, pb), osz(W, kw, sw, dw_, pl, pr)
    rng = np.random.default_rng(sum(case) + 7 * splits + epi)
    x = rand16(rng, N * C * H * W)
    w = rand16(rng, M * C * kh * kw)
    bias = rand16(rng, M)
    r = rand16(rng, N * M * oh * ow)
    size = N * M * oh * ow
    want = port.conv(x, w, bias if hb else None, N, C, H, W, M, oh, ow, kh, kw, sh, sw, dh, dw_, pt, pl, hb, dwm)[:size]
    if epi & 2:
        want = port.vectorop(want, r, size, 0, 1, 0, 0)[:size]
    if epi & 1:
        want = port.vectorop(want, None, size, 4, 1, 0, 0)[:size]
    L = _lib.lib()
    old = L.cm_set_gemm_split(splits)
    try:
        for rep in range(2):                       # the arrival counters are zero again after a launch
            y = empty(size)
            kernels.ConvKernelFused(dev(x), dev(w), dev(bias) if hb else None, y, N, C, H, W, M, oh, ow, kh, kw, sh,
                                    sw, dh, dw_, pt, pl, hb, dwm, epilogue=epi, resid=dev(r) if epi & 2 else None)
            assert_same(host(y), want, f"K-split {splits} {case} epi {epi} call {rep}")
    finally:
        L.cm_set_gemm_split(old)
