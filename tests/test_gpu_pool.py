"""PoolingKernel parity on the GPU: cm_pool vs the C restatement, bit-exact.

Covers MAX / AVG (count_include_pad 0 and 1) / LP (p = 1, 2, and the
"any other order" branch) / an out-of-range pool_type, padding, dilation,
strides (including 0), asymmetric trailing padding, empty windows, global
pools on aligned and unaligned planes, full-range inputs that make the AVG
and LP sums wrap, and the BASELINE pool sweep at full size.
"""
import zlib

import numpy as np
import pytest

from tests._util import assert_same, dev, empty, host, rand16

pytestmark = pytest.mark.gpu


def out_size(n, k, s, p_begin, p_end, d):
    return (n + p_begin + p_end - d * (k - 1) - 1) // s + 1


# (N, C, H, W, ph, pw, sh, sw, pt, pl, dh, dw, extra_bottom_right)
GEOMS = [
    (2, 3, 11, 13, 3, 3, 2, 2, 1, 1, 1, 1, 0),
    (1, 4, 12, 12, 3, 3, 2, 2, 1, 1, 2, 2, 0),
    (2, 5, 8, 8, 2, 2, 2, 2, 0, 0, 1, 1, 0),
    (1, 3, 28, 28, 2, 2, 2, 2, 0, 0, 1, 1, 0),       # LeNet pools
    (1, 2, 7, 7, 7, 7, 1, 1, 0, 0, 1, 1, 0),          # global via the window kernel's caller rule
    (3, 2, 5, 6, 3, 3, 1, 1, 2, 2, 1, 1, 0),          # pad >= half window: all-pad corners
    (1, 2, 9, 9, 3, 2, 3, 2, 1, 0, 1, 1, 2),          # asymmetric trailing pad
    (1, 1, 6, 6, 4, 4, 2, 2, 3, 3, 1, 1, 0),          # windows entirely in padding
    (2, 3, 10, 1, 3, 1, 1, 1, 1, 0, 1, 1, 0),         # width 1
    (1, 2, 300, 500, 3, 3, 2, 2, 1, 1, 1, 1, 0),      # band split (plane > shared-memory budget)
    (1, 1, 40, 2000, 21, 3, 1, 1, 10, 1, 1, 1, 0),    # tall window, wide rows: direct kernel
    (1, 2, 9, 9, 3, 3, 0, 2, 1, 1, 1, 1, 0),          # stride 0
]

# (pool_type, lp_order, count_include_pad)
TYPES = [(0, 2, 0), (1, 2, 0), (1, 2, 1), (2, 1, 0), (2, 2, 0), (2, 3, 0), (5, 1, 0)]


def run_case(cm, port, x, N, C, H, W, ph, pw, sh, sw, pt, pl, dh, dw, extra, t, lp, cip):
    oh = out_size(H, ph, max(sh, 1), pt, pt + extra, dh) if sh else 3
    ow = out_size(W, pw, max(sw, 1), pl, pl + extra, dw) if sw else 3
    y = empty(N * C * oh * ow)
    cm.PoolingKernel(dev(x), y, N, C, H, W, oh, ow, ph, pw, sh, sw, pt, pl, dh, dw, t, lp, cip)
    want = port.pool(x, N, C, H, W, oh, ow, ph, pw, sh, sw, pt, pl, dh, dw, t, lp, cip)
    assert_same(host(y), want, f"geom={(N, C, H, W, ph, pw, sh, sw, pt, pl, dh, dw, extra)} type={(t, lp, cip)}")


@pytest.mark.parametrize("geom", GEOMS)
@pytest.mark.parametrize("typ", TYPES)
@pytest.mark.parametrize("rng_range", ["q8", "full"])
def test_window(cm, port, geom, typ, rng_range):
    N, C, H, W = geom[:4]
    rng = np.random.default_rng(zlib.crc32(repr((geom, typ, rng_range)).encode()))
    x = rand16(rng, N * C * H * W, *((-2048, 2048) if rng_range == "q8" else (-32768, 32768)))
    run_case(cm, port, x, *geom, *typ)


@pytest.mark.parametrize("hw", [(7, 7), (112, 112), (13, 11), (1, 1), (64, 300)])
@pytest.mark.parametrize("typ", TYPES)
def test_global(cm, port, hw, typ):
    H, W = hw
    N, C = 3, 5
    rng = np.random.default_rng(H * 1000 + W + typ[0])
    x = rand16(rng, N * C * H * W)
    run_case(cm, port, x, N, C, H, W, H, W, 1, 1, 0, 0, 1, 1, 0, *typ)


@pytest.mark.parametrize("hw", [(7, 7), (14, 14), (5, 3), (16, 32)])
@pytest.mark.parametrize("typ", TYPES)
def test_global_many_small_planes(cm, port, hw, typ):
    """Global pools of many small planes (the ResNet classifier's 7x7 input): several
    blocks of staged planes, a partial last block, odd word counts."""
    H, W = hw
    N, C = 3, 700
    rng = np.random.default_rng(H * 100 + W + typ[0])
    x = rand16(rng, N * C * H * W)
    run_case(cm, port, x, N, C, H, W, H, W, 1, 1, 0, 0, 1, 1, 0, *typ)


def test_empty_window(cm, port):
    x = rand16(np.random.default_rng(3), 2 * 3 * 4 * 4)
    for t in (0, 1, 2):
        y = empty(2 * 3 * 2 * 2)
        cm.PoolingKernel(dev(x), y, 2, 3, 4, 4, 2, 2, 0, 0, 1, 1, 0, 0, 1, 1, t, 2, 0)
        assert_same(host(y), port.pool(x, 2, 3, 4, 4, 2, 2, 0, 0, 1, 1, 0, 0, 1, 1, t, 2, 0), f"pool_h=0 type {t}")


SWEEP = [  # BASELINE pool sweep on [256, 64, 112, 112], raw uniform [-2048, 2048)
    ("max3x3s2p1d1", 3, 3, 2, 2, 1, 1, 1, 1, 0, 2, 0),
    ("max3x3s2p1d2", 3, 3, 2, 2, 1, 1, 2, 2, 0, 2, 0),
    ("avg3x3s2p1cip0", 3, 3, 2, 2, 1, 1, 1, 1, 1, 2, 0),
    ("avg3x3s2p1cip1", 3, 3, 2, 2, 1, 1, 1, 1, 1, 2, 1),
    ("lp2_2x2s2", 2, 2, 2, 2, 0, 0, 1, 1, 2, 2, 0),
    ("globalmax", 112, 112, 1, 1, 0, 0, 1, 1, 0, 2, 0),
    ("globalavg", 112, 112, 1, 1, 0, 0, 1, 1, 1, 2, 0),
]


@pytest.fixture(scope="module")
def sweep_input():
    rng = np.random.default_rng(42 + 5)
    return rand16(rng, 256 * 64 * 112 * 112, -2048, 2048)


@pytest.mark.parametrize("case", SWEEP, ids=[c[0] for c in SWEEP])
def test_sweep_full_size(cm, port, sweep_input, case):
    _, ph, pw, sh, sw, pt, pl, dh, dw, t, lp, cip = case
    N, C, H, W = 256, 64, 112, 112
    run_case(cm, port, sweep_input, N, C, H, W, ph, pw, sh, sw, pt, pl, dh, dw, 0, t, lp, cip)


# Layouts of the compile-time geometries with input width a multiple of 8 (one 8-column chunk
# per strip of outputs): planes of at most 32 KB go through the whole-plane kernel (several
# planes per CTA), larger ones through the row-streaming kernel (planes straddling warps).
ROWS = [
    (1, 3, 160, 128, 3, 3, 2, 2, 1, 1, 1, 1, 0),
    (1, 2, 150, 120, 3, 3, 2, 2, 1, 1, 2, 2, 0),
    (1, 2, 144, 120, 2, 2, 2, 2, 0, 0, 1, 1, 0),
    (5, 131, 12, 16, 3, 3, 2, 2, 1, 1, 1, 1, 0),
    (3, 5, 16, 16, 3, 3, 2, 2, 1, 1, 1, 1, 0),
    (2, 7, 40, 64, 3, 3, 2, 2, 1, 1, 1, 1, 0),
    (1, 9, 24, 112, 3, 3, 2, 2, 1, 1, 1, 1, 0),
    (2, 5, 30, 64, 3, 3, 2, 2, 1, 1, 2, 2, 0),
    (1, 11, 20, 112, 3, 3, 2, 2, 1, 1, 2, 2, 0),
    (2, 6, 18, 64, 2, 2, 2, 2, 0, 0, 1, 1, 0),
    (1, 13, 9, 40, 2, 2, 2, 2, 0, 0, 1, 1, 0),
]


@pytest.mark.parametrize("geom", ROWS)
@pytest.mark.parametrize("typ", TYPES)
def test_row_stream_layouts(cm, port, geom, typ):
    N, C, H, W = geom[:4]
    rng = np.random.default_rng(zlib.crc32(repr(("rows", geom, typ)).encode()))
    x = rand16(rng, N * C * H * W)
    run_case(cm, port, x, *geom, *typ)
