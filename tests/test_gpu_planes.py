"""Plane images (cm_conv_planes): a conv's output written by its GEMM epilogue as the
channels-last operand of the implicit-GEMM convs that read it.  Not a reference kernel:
every consumer's output must equal the reference call sequence producer -> consumer run
on NCHW tensors by the oracle, word for word."""
import numpy as np
import pytest

from tests._util import assert_same, dev, empty, host, rand16

pytestmark = pytest.mark.gpu


def osz(n, k, s, p):
    return (n + 2 * p - k) // s + 1


def geo(N, C, H, W, M, k, s, p):
    return (N, C, H, W, M, osz(H, k, s, p), osz(W, k, s, p), k, k, s, s, 1, 1, p, p, 1, 0)


def oracle(port, x, w, b, g, epi=0, resid=None):
    size = g[0] * g[4] * g[5] * g[6]
    y = port.conv(x, w, b, *g)[:size]
    if epi & 2:
        y = port.vectorop(y, resid, size, 0, 1, 0, 0)[:size]
    if epi & 1:
        y = port.vectorop(y, None, size, 4, 1, 0, 0)[:size]
    return y


def weights(rng, g):
    return rand16(rng, g[4] * g[1] * g[7] * g[8], -256, 256), rand16(rng, g[4], -256, 256)


# (producer N, C, H, W, M, k, s, p), (consumer M, k, s, p), producer epilogue
CASES = [
    ((3, 64, 14, 14, 64, 3, 1, 1), (64, 3, 1, 1), 1),      # 64-column producer tiles
    ((3, 64, 14, 14, 128, 3, 1, 1), (128, 3, 1, 1), 1),    # 128-column tiles on CTA pairs
    ((2, 32, 16, 16, 40, 3, 1, 1), (24, 3, 1, 1), 0),      # 40 channels: a partial 16-channel chunk
    ((4, 128, 28, 28, 64, 3, 1, 1), (96, 1, 2, 0), 1),     # consumer padding smaller than the frame
    ((2, 128, 28, 28, 64, 3, 1, 1), (96, 3, 2, 1), 1),     # stride-2 consumer
    ((2, 3, 64, 64, 64, 7, 2, 3), (64, 3, 1, 1), 1),       # space-to-depth producer (stem form)
    ((5, 64, 7, 7, 96, 3, 1, 1), (80, 3, 1, 1), 1),        # 7x7 maps, tile rows past the images
]


@pytest.mark.parametrize("prod,cons,epi", CASES)
@pytest.mark.parametrize("keep_y", [False, True])
def test_producer_consumer(cm, port, prod, cons, epi, keep_y):
    from cormorant_b200 import kernels
    rng = np.random.default_rng(sum(prod) * 31 + sum(cons) + epi)
    g1 = geo(*prod)
    N, M1, oh, ow = g1[0], g1[4], g1[5], g1[6]
    g2 = geo(N, M1, oh, ow, *cons)
    frame = kernels.conv_plane_frame(*g2)
    assert frame is not None, "consumer must read plane images"
    x = rand16(rng, N * g1[1] * g1[2] * g1[3], -1024, 1024)
    w1, b1 = weights(rng, g1)
    w2, b2 = weights(rng, g2)
    y1_want = oracle(port, x, w1, b1, g1, epi)
    y2_want = oracle(port, y1_want, w2, b2, g2)
    P = kernels.PlaneImage(N, M1, oh, ow, frame)
    y1 = empty(y1_want.size) if keep_y else None
    kernels.ConvKernelPlanes(dev(x), None, dev(w1), dev(b1), y1, P, *g1, epilogue=epi)
    y2 = empty(y2_want.size)
    kernels.ConvKernelPlanes(None, P, dev(w2), dev(b2), y2, None, *g2)
    if keep_y:
        assert_same(host(y1), y1_want, f"producer y {prod}")
    assert_same(host(y2), y2_want, f"consumer {prod} -> {cons}")


def test_producer_on_cuda_core_path_and_residual(cm, port):
    """A producer on the CUDA-core path fills the image by a split pass; a consumer with a
    residual epilogue and its own plane output chains a third conv."""
    from cormorant_b200 import _lib, kernels
    L = _lib.lib()
    rng = np.random.default_rng(5)
    g1 = geo(2, 16, 12, 12, 64, 3, 1, 1)
    g2 = geo(2, 64, 12, 12, 64, 3, 1, 1)
    x = rand16(rng, 2 * 16 * 144)
    w1, b1 = weights(rng, g1)
    w2, b2 = weights(rng, g2)
    w3, b3 = weights(rng, g2)
    r = rand16(rng, 2 * 64 * 144)
    y1 = oracle(port, x, w1, b1, g1, 1)
    y2 = oracle(port, y1, w2, b2, g2, 3, r)
    y3 = oracle(port, y2, w3, b3, g2, 1)
    fr = kernels.conv_plane_frame(*g2)
    P1, P2 = kernels.PlaneImage(2, 64, 12, 12, fr), kernels.PlaneImage(2, 64, 12, 12, fr)
    old = L.cm_set_direct_limit(1 << 40)                  # producer on the CUDA-core path
    try:
        kernels.ConvKernelPlanes(dev(x), None, dev(w1), dev(b1), None, P1, *g1, epilogue=1)
    finally:
        L.cm_set_direct_limit(0)                          # the rest on the tensor cores
    try:
        got2 = empty(y2.size)
        kernels.ConvKernelPlanes(None, P1, dev(w2), dev(b2), got2, P2, *g2, epilogue=3, resid=dev(r))
        got3 = empty(y3.size)
        kernels.ConvKernelPlanes(None, P2, dev(w3), dev(b3), got3, None, *g2, epilogue=1)
    finally:
        L.cm_set_direct_limit(old)
    assert_same(host(got2), y2, "residual consumer")
    assert_same(host(got3), y3, "third conv")


def test_unusable_image_needs_x(cm, port):
    """A conv that cannot read the image (column dilation: not the implicit path, or a
    frame too narrow) falls back to x, and without x reports CM_EINVAL."""
    from cormorant_b200 import CormorantError, kernels
    rng = np.random.default_rng(9)
    g1 = geo(2, 64, 14, 14, 64, 3, 1, 1)
    x = rand16(rng, 2 * 64 * 196)
    w1, b1 = weights(rng, g1)
    y1 = oracle(port, x, w1, b1, g1)
    P = kernels.PlaneImage(2, 64, 14, 14, (0, 0, 0, 0))  # no frame: a padded consumer cannot use it
    kernels.ConvKernelPlanes(dev(x), None, dev(w1), dev(b1), None, P, *g1)
    g2 = geo(2, 64, 14, 14, 64, 3, 1, 1)
    w2, b2 = weights(rng, g2)
    with pytest.raises(CormorantError):
        kernels.ConvKernelPlanes(None, P, dev(w2), dev(b2), empty(2 * 64 * 196), None, *g2)
    y2 = empty(2 * 64 * 196)
    kernels.ConvKernelPlanes(dev(y1), P, dev(w2), dev(b2), y2, None, *g2)   # falls back to x
    assert_same(host(y2), oracle(port, y1, w2, b2, g2), "fallback to x")
    # column dilation: explicit im2col path reads x only
    g3 = (2, 64, 14, 14, 32, 14, 12, 3, 3, 1, 1, 1, 2, 1, 1, 1, 0)
    from cormorant_b200 import kernels as k
    assert k.conv_plane_frame(*g3) is None
    w3, b3 = rand16(rng, 32 * 64 * 9, -256, 256), rand16(rng, 32, -256, 256)
    with pytest.raises(CormorantError):
        kernels.ConvKernelPlanes(None, P, dev(w3), dev(b3), empty(2 * 32 * 14 * 12), None, *g3)
    with pytest.raises(CormorantError):                  # output image of another shape
        kernels.ConvKernelPlanes(dev(x), None, dev(w1), dev(b1), None, kernels.PlaneImage(2, 64, 7, 7), *g1)


def test_residual_from_plane_image(cm, port):
    """Conv -> Add(residual) -> Relu with the residual read from its plane image (the
    block input of a residual block): no NCHW copy of the residual is needed; a conv that
    cannot read plane images needs the NCHW residual."""
    from cormorant_b200 import CormorantError, _lib, kernels
    rng = np.random.default_rng(21)
    for (N, C, H) in ((3, 64, 14), (2, 128, 28)):
        g0 = geo(N, 16, H, H, C, 3, 1, 1)
        g1 = geo(N, C, H, H, C, 3, 1, 1)
        x = rand16(rng, N * 16 * H * H)
        w0, b0 = weights(rng, g0)
        w1, b1 = weights(rng, g1)
        r = oracle(port, x, w0, b0, g0, 1)                 # the block input
        want = oracle(port, r, w1, b1, g1, 3, r)           # conv(r) + r, then Relu
        R = kernels.PlaneImage(N, C, H, H, kernels.conv_plane_frame(*g1))
        kernels.ConvKernelPlanes(dev(x), None, dev(w0), dev(b0), None, R, *g0, epilogue=1)
        got = empty(want.size)
        kernels.ConvKernelPlanes(None, R, dev(w1), dev(b1), got, None, *g1, epilogue=3, resid=None, resid_planes=R)
        assert_same(host(got), want, f"residual from planes {N}x{C}x{H}")
    L = _lib.lib()
    old = L.cm_set_direct_limit(1 << 40)                  # the consumer on the CUDA-core path
    try:
        with pytest.raises(CormorantError):
            kernels.ConvKernelPlanes(dev(r), None, dev(w1), dev(b1), empty(want.size), None, *g1, epilogue=3,
                                     resid=None, resid_planes=R)
        got = empty(want.size)
        kernels.ConvKernelPlanes(dev(r), None, dev(w1), dev(b1), got, None, *g1, epilogue=3, resid=dev(r),
                                 resid_planes=R)
    finally:
        L.cm_set_direct_limit(old)
    assert_same(host(got), want, "NCHW residual on the CUDA-core path")


@pytest.mark.parametrize("splits", [0, 3])
def test_k_split_plane_output_and_residual(cm, port, splits):
    """A residual block of plane images (conv -> planes; conv(planes) + residual planes ->
    planes + y) on K-split GEMMs: the same words as the unsplit ones and the reference."""
    from cormorant_b200 import _lib, kernels
    rng = np.random.default_rng(77 + splits)
    N, C, H = 4, 256, 14
    g0 = geo(N, 64, H, H, C, 3, 1, 1)
    g1 = geo(N, C, H, H, C, 3, 1, 1)
    g2 = geo(N, C, H, H, 96, 3, 1, 1)
    x = rand16(rng, N * 64 * H * H)
    w0, b0 = weights(rng, g0)
    w1, b1 = weights(rng, g1)
    w2, b2 = weights(rng, g2)
    r = oracle(port, x, w0, b0, g0, 1)
    y1_want = oracle(port, r, w1, b1, g1, 3, r)
    y2_want = oracle(port, y1_want, w2, b2, g2)
    L = _lib.lib()
    old = L.cm_set_gemm_split(splits)
    try:
        R = kernels.PlaneImage(N, C, H, H, kernels.conv_plane_frame(*g1))
        kernels.ConvKernelPlanes(dev(x), None, dev(w0), dev(b0), None, R, *g0, epilogue=1)
        P = kernels.PlaneImage(N, C, H, H, kernels.conv_plane_frame(*g2))
        y1 = empty(y1_want.size)
        kernels.ConvKernelPlanes(None, R, dev(w1), dev(b1), y1, P, *g1, epilogue=3, resid=None, resid_planes=R)
        y2 = empty(y2_want.size)
        kernels.ConvKernelPlanes(None, P, dev(w2), dev(b2), y2, None, *g2)
    finally:
        L.cm_set_gemm_split(old)
    assert_same(host(y1), y1_want, f"K-split {splits}: block output")
    assert_same(host(y2), y2_want, f"K-split {splits}: conv of the block's plane image")


@pytest.mark.parametrize("N,C,H,W", [(3, 64, 14, 14), (2, 40, 7, 9), (2, 64, 56, 56)])
def test_planes_fill_then_conv_and_residual(cm, port, N, C, H, W):
    """cm_planes_fill splits an NCHW tensor no conv produced (a pool output) into a plane
    image; a conv reads it as its operand and as its residual."""
    from cormorant_b200 import kernels
    rng = np.random.default_rng(N * C + H)
    g = geo(N, C, H, W, C, 3, 1, 1)
    x = rand16(rng, N * C * H * W, -2048, 2048)
    w, b = weights(rng, g)
    want = oracle(port, x, w, b, g, 3, x)
    P = kernels.PlaneImage(N, C, H, W, kernels.conv_plane_frame(*g) or (1, 1, 1, 1))
    kernels.PlanesFill(P, dev(x))
    got = empty(want.size)
    if kernels.conv_plane_frame(*g) is None:
        pytest.skip("this conv runs on the CUDA-core path")
    kernels.ConvKernelPlanes(None, P, dev(w), dev(b), got, None, *g, epilogue=3, resid=None, resid_planes=P)
    assert_same(host(got), want, f"fill {N}x{C}x{H}x{W}")


@pytest.mark.parametrize("C,M", [(64, 64), (32, 44)])
@pytest.mark.parametrize("res", ["nchw", "planes"])
@pytest.mark.parametrize("prepared", [False, True])
def test_plane_only_output_with_residual(cm, port, C, M, res, prepared):
    """A conv of at most 64 output channels whose output is only a plane image (the
    weights-as-A GEMM form) with a fused residual Add + Relu, the residual as NCHW words
    or as its own plane image: the image holds the reference sequence's words (read back
    through an identity 1x1 conv, which also checks its channel sums)."""
    from cormorant_b200 import kernels
    rng = np.random.default_rng(C * 7 + M + len(res))
    N, H, W = 2, 28, 28
    g1 = geo(N, C, H, W, M, 3, 1, 1)
    x = rand16(rng, N * C * H * W, -1024, 1024)
    w1, b1 = weights(rng, g1)
    r = rand16(rng, N * M * H * W, -4096, 4096)
    want = oracle(port, x, w1, b1, g1, 3, r)
    P = kernels.PlaneImage(N, M, H, W, kernels.conv_plane_frame(*geo(N, M, H, W, 64, 3, 1, 1)))
    R = None
    if res == "planes":
        R = kernels.PlaneImage(N, M, H, W, (0, 0, 0, 0))
        kernels.PlanesFill(R, dev(r))
    rd = None if R is not None else dev(r)
    if prepared:                                   # the weights-as-A rows built once
        wd, bd = dev(w1), dev(b1)
        pw = kernels.ConvWeights(wd, bd, *g1)
        kernels.ConvKernelPrepared(pw, dev(x), None, None, P, epilogue=3, resid=rd, resid_planes=R)
    else:
        kernels.ConvKernelPlanes(dev(x), None, dev(w1), dev(b1), None, P, *g1, epilogue=3, resid=rd, resid_planes=R)
    assert_same(_identity_readback(kernels, P, N, M, H, W), want, f"plane-only output, {res} residual, M={M}")


def _identity_readback(kernels, P, N, C, H, W):
    """The NCHW words of plane image P: a 1x1 conv with identity weights (1.0 = 256) reads it."""
    import torch
    from cormorant_b200 import _lib
    w = np.zeros((C, C), np.int16)
    np.fill_diagonal(w, 256)
    g = (N, C, H, W, C, H, W, 1, 1, 1, 1, 1, 1, 0, 0, 0, 0)
    L = _lib.lib()
    old = L.cm_set_direct_limit(0)                        # the tensor-core path, whatever the size
    try:
        assert kernels.conv_plane_frame(*g) is not None
        y = empty(N * C * H * W)
        kernels.ConvKernelPlanes(None, P, dev(w.reshape(-1)), None, y, None, *g)
        torch.cuda.synchronize()
    finally:
        L.cm_set_direct_limit(old)
    return host(y)


@pytest.mark.parametrize("N,H,W,k,s,p,d", [(4, 112, 112, 3, 2, 1, 1), (3, 30, 26, 3, 2, 1, 2), (8, 20, 20, 2, 2, 1, 1),
                                           (16, 9, 13, 3, 1, 1, 1), (40, 4, 4, 5, 3, 2, 1)])
def test_max_pool_plane_to_plane(cm, port, N, H, W, k, s, p, d):
    """cm_pool_planes equals cm_pool's MAX on the NCHW tensors, windows with no tap in the
    image included (they give -32768); read back through an identity 1x1 conv."""
    from cormorant_b200 import kernels
    C = 64
    rng = np.random.default_rng(N + H + k)
    x = rand16(rng, N * C * H * W)
    oh, ow = (H + 2 * p - d * (k - 1) - 1) // s + 1, (W + 2 * p - d * (k - 1) - 1) // s + 1
    pa = (N, C, H, W, oh, ow, k, k, s, s, p, p, d, d, 0, 2, 0)
    want = port.pool(x, *pa)[: N * C * oh * ow]
    X = kernels.PlaneImage(N, C, H, W)
    kernels.PlanesFill(X, dev(x))
    Y = kernels.PlaneImage(N, C, oh, ow)
    kernels.PoolingKernelPlanes(X, Y, *pa)
    assert_same(_identity_readback(kernels, Y, N, C, oh, ow), want, f"max pool planes {pa}")


def _nchw_to_nhwc(t, n, c, h, w):
    return np.ascontiguousarray(np.asarray(t)[: n * c * h * w].reshape(n, c, h, w).transpose(0, 2, 3, 1)).reshape(-1)


@pytest.mark.parametrize("N,C,H,W,k,s,p,d,frame", [(4, 64, 112, 112, 3, 2, 1, 1, (1, 1, 1, 1)),
                                                   (3, 32, 30, 26, 3, 2, 1, 2, (0, 0, 0, 0)),
                                                   (2, 128, 20, 20, 2, 2, 1, 1, (1, 1, 1, 1)),
                                                   (5, 64, 9, 13, 3, 1, 1, 1, (2, 1, 0, 3)),
                                                   (40, 64, 4, 4, 5, 3, 2, 1, (0, 0, 0, 0))])
def test_max_pool_nhwc_to_planes(cm, port, N, C, H, W, k, s, p, d, frame):
    """cm_pool_nhwc_planes: the MAX pool of a channels-last tensor written as a plane image
    (hi / lo' planes and channel sums, inside a frame) equals cm_pool's MAX on the NCHW
    tensor, windows with no tap in the image included; read back through an identity 1x1
    conv, whose row terms come from the image's channel sums."""
    from cormorant_b200 import kernels
    rng = np.random.default_rng(N * 31 + C + H + k)
    x = rand16(rng, N * C * H * W)
    oh, ow = (H + 2 * p - d * (k - 1) - 1) // s + 1, (W + 2 * p - d * (k - 1) - 1) // s + 1
    pa = (N, C, H, W, oh, ow, k, k, s, s, p, p, d, d, 0, 2, 0)
    want = port.pool(x, *pa)[: N * C * oh * ow]
    Y = kernels.PlaneImage(N, C, oh, ow, frame)
    kernels.PoolingKernelNhwcPlanes(dev(_nchw_to_nhwc(x, N, C, H, W)), Y, *pa[:15])
    assert_same(_identity_readback(kernels, Y, N, C, oh, ow), want, f"max pool nhwc -> planes {pa} frame {frame}")


@pytest.mark.parametrize("N,C,H,W,ptype,lp", [(256, 512, 7, 7, 1, 2), (5, 64, 7, 7, 0, 2), (3, 24, 9, 5, 2, 2),
                                                (2, 40, 3, 3, 2, 1), (4, 8, 1, 1, 1, 2), (2, 16, 30, 30, 1, 2)])
def test_global_pool_nhwc(cm, port, N, C, H, W, ptype, lp):
    """cm_pool_nhwc: a global pool of a channels-last tensor gives cm_pool's words on the NCHW
    tensor (AVG, MAX, LP2, LP1; pixel counts with and without a remainder of 7)."""
    from cormorant_b200 import kernels
    rng = np.random.default_rng(N + C + H + ptype)
    x = rand16(rng, N * C * H * W)
    pa = (N, C, H, W, 1, 1, H, W, 1, 1, 0, 0, 1, 1, ptype, lp, 0)
    want = port.pool(x, *pa)[: N * C]
    y = empty(N * C)
    kernels.PoolingKernelNhwc(dev(_nchw_to_nhwc(x, N, C, H, W)), y, *pa)
    assert_same(host(y), want, f"global pool nhwc {pa}")


def test_global_pool_nhwc_refusals(cm):
    """Only global pools, channels a multiple of 8."""
    from cormorant_b200 import kernels
    with pytest.raises(cm.CormorantError):      # not global: a 2 x 2 output
        kernels.PoolingKernelNhwc(dev(np.zeros(2 * 4 * 4 * 8, np.int16)), empty(2 * 8 * 4), 2, 8, 4, 4, 2, 2, 2, 2, 2, 2)
    with pytest.raises(cm.CormorantError):      # 12 channels
        kernels.PoolingKernelNhwc(dev(np.zeros(2 * 4 * 4 * 12, np.int16)), empty(2 * 12), 2, 12, 4, 4, 1, 1, 4, 4,
                                  pool_type=kernels.POOL_AVG)


def test_max_pool_nhwc_to_planes_refusals(cm):
    """Channel counts other than 16 x a power of two, and pool types other than MAX, are refused."""
    from cormorant_b200 import kernels
    Y = kernels.PlaneImage(2, 48, 4, 4)
    with pytest.raises(cm.CormorantError):
        kernels.PoolingKernelNhwcPlanes(dev(np.zeros(2 * 8 * 8 * 48, np.int16)), Y, 2, 48, 8, 8, 4, 4, 2, 2, 2, 2)
    Y2 = kernels.PlaneImage(2, 64, 4, 4)
    with pytest.raises(cm.CormorantError):
        kernels.PoolingKernelNhwcPlanes(dev(np.zeros(2 * 8 * 8 * 64, np.int16)), Y2, 2, 64, 8, 8, 4, 4, 2, 2, 2, 2,
                                        pool_type=kernels.POOL_AVG)


@pytest.mark.parametrize("g,epi", [(geo(2, 3, 64, 64, 64, 7, 2, 3), 1),       # space-to-depth stem form
                                   (geo(3, 64, 14, 14, 64, 3, 1, 1), 0),      # 64-column window form
                                   (geo(3, 64, 14, 14, 64, 3, 1, 1), 1),
                                   (geo(2, 64, 14, 14, 128, 3, 1, 1), 1)])    # 128-column tiles on CTA pairs
def test_conv_channels_last_output(cm, port, g, epi):
    """Epilogue bit 3 (EPI_NHWC): y is the same words as the NCHW output, channels-last."""
    from cormorant_b200 import kernels
    import torch
    rng = np.random.default_rng(sum(g) + epi)
    x = rand16(rng, g[0] * g[1] * g[2] * g[3])
    w, b = weights(rng, g)
    assert kernels.conv_writes_nhwc(*g)
    want = _nchw_to_nhwc(oracle(port, x, w, b, g, epi), g[0], g[4], g[5], g[6])
    y = empty(g[0] * g[4] * g[5] * g[6])
    kernels.ConvKernelPlanes(dev(x), None, dev(w), dev(b), y, None, *g, epilogue=epi | kernels.EPI_NHWC)
    torch.cuda.synchronize()
    assert_same(host(y), want, f"channels-last conv {g} epi {epi}")


def test_conv_channels_last_refused_off_gemm_paths(cm, port):
    """A conv on a CUDA-core path cannot write channels-last: CM_EUNSUPPORTED."""
    from cormorant_b200 import _lib, kernels
    g = geo(1, 4, 6, 6, 8, 3, 1, 1)
    L = _lib.lib()
    old = L.cm_set_direct_limit(1 << 26)                  # the direct path for this size
    try:
        assert not kernels.conv_writes_nhwc(*g)
        rng = np.random.default_rng(3)
        x = rand16(rng, 4 * 36)
        w, b = weights(rng, g)
        with pytest.raises(cm.CormorantError):
            kernels.ConvKernelPlanes(dev(x), None, dev(w), dev(b), empty(8 * 36), None, *g, epilogue=kernels.EPI_NHWC)
    finally:
        L.cm_set_direct_limit(old)
