"""MatmulKernel parity on the GPU: cm_matmul (tcgen05 int8 byte-split) vs the oracle.

Bit-exact on raw int16 words.  Shapes follow the reference's own test matrix
(TestMatmulSim.cpp:276-349: unit dims, partial tiles in every dimension,
multi-tile, batch with A or B broadcast), its saturation KATs
(TestMatmulSim.cpp:364-367), accumulator wrap with full-range operands, the
K == 0 and overlapping-output edge cases, and every BASELINE sweep shape
(full compare at 256^3, sampled rows at the larger shapes).
"""
import numpy as np
import pytest

from tests._util import assert_same, dev, empty, host, rand16

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("mac_path")]

# (n, k, m, batch) -- TILE_N=4, TILE_K=256, TILE_M=16 in the reference; 128-tiles here
SHAPES = [(1, 1, 1, 1), (4, 256, 16, 1), (8, 256, 16, 1), (4, 512, 16, 1), (4, 256, 32, 1), (6, 256, 16, 1),
          (4, 261, 16, 1), (4, 256, 19, 1), (6, 261, 19, 1), (7, 13, 5, 1), (5, 1, 17, 1), (1, 256, 16, 1),
          (4, 256, 1, 1), (12, 519, 33, 1), (128, 128, 128, 1), (129, 130, 131, 2), (255, 257, 383, 3),
          (1, 400, 120, 1), (1, 120, 84, 1), (1, 84, 10, 1), (256, 512, 1000, 1), (300, 17, 200, 4),
          (64, 32, 64, 5), (33, 4096, 65, 1),
          # few-row direct form (lane = output column, warps split k): rows below the
          # template's width, exactly 8 rows, widths off a multiple of 32, k < 8 (idle
          # warps), a batch of 100 steps on the grid's y axis
          (3, 7, 70, 3), (8, 1000, 33, 2), (2, 5, 100, 100), (1, 3, 31, 1)]


@pytest.mark.parametrize("n,k,m,batch", SHAPES)
@pytest.mark.parametrize("dist", ["q8", "full"])
def test_shapes(cm, port, n, k, m, batch, dist):
    rng = np.random.default_rng(n * 7919 + k * 31 + m + batch)
    lo, hi = (-1024, 1024) if dist == "q8" else (-32768, 32768)
    a = rand16(rng, batch * n * k, lo, hi)
    b = rand16(rng, batch * k * m, lo, hi)
    c = empty(batch * n * m)
    cm.MatmulKernel(dev(a), dev(b), c, n, k, m, batch)
    assert_same(host(c), port.matmul(a, b, n, k, m, batch), f"{n}x{k}x{m} b{batch} {dist}")


@pytest.mark.parametrize("a_bs,b_bs", [(0, None), (None, 0), (0, 0)])
def test_broadcast(cm, port, a_bs, b_bs):
    n, k, m, batch = 5, 64, 19, 4
    rng = np.random.default_rng(11)
    a_bs = n * k if a_bs is None else a_bs
    b_bs = k * m if b_bs is None else b_bs
    a = rand16(rng, max((batch - 1) * a_bs + n * k, 1))
    b = rand16(rng, max((batch - 1) * b_bs + k * m, 1))
    c = empty(batch * n * m)
    cm.MatmulKernel(dev(a), dev(b), c, n, k, m, batch, a_bs, b_bs, n * m)
    assert_same(host(c), port.matmul(a, b, n, k, m, batch, a_bs, b_bs, n * m), f"strides {a_bs},{b_bs}")


@pytest.mark.parametrize("a_val,b_val,sat", [(25600, 25600, 32767), (25600, -25600, -32768)])
def test_saturation_kat(cm, port, a_val, b_val, sat):
    """a = 100.0, b = +-100.0, K = 3: 30000.0 saturates to AP_MAX / AP_MIN."""
    n, k, m = 4, 3, 16
    a = np.full(n * k, a_val, np.int16)
    b = np.full(k * m, b_val, np.int16)
    c = empty(n * m)
    cm.MatmulKernel(dev(a), dev(b), c, n, k, m)
    got = host(c)
    assert (got == sat).all()
    assert_same(got, port.matmul(a, b, n, k, m), "saturation")


def test_accumulator_wrap(cm, port):
    """Sums past +-2^31 at Q16.16 wrap (AP_WRAP) before the single saturating narrow."""
    n, k, m = 16, 4096, 48
    a = np.full(n * k, 32767, np.int16)
    b = np.full(k * m, 32767, np.int16)
    a[::2] = -32768
    c = empty(n * m)
    cm.MatmulKernel(dev(a), dev(b), c, n, k, m)
    assert_same(host(c), port.matmul(a, b, n, k, m), "wrap")


def test_k_zero_writes_zeros(cm, port):
    c = empty(3 * 5 * 2)
    cm.MatmulKernel(dev(np.zeros(1, np.int16)), dev(np.zeros(1, np.int16)), c, 3, 0, 5, 2, 0, 0, 15)
    assert (host(c) == 0).all()


def test_overlapping_output_batches(cm, port):
    """c_batch_stride < n*m: later batch steps overwrite earlier ones, as in the reference loop."""
    n, k, m, batch = 4, 40, 8, 3
    rng = np.random.default_rng(5)
    a = rand16(rng, batch * n * k)
    b = rand16(rng, batch * k * m)
    for c_bs in (0, 8, 20):
        c_len = (batch - 1) * c_bs + n * m
        init = np.full(c_len, -23131, np.int16)
        c = dev(init)
        cm.MatmulKernel(dev(a), dev(b), c, n, k, m, batch, n * k, k * m, c_bs)
        assert_same(host(c), port.matmul(a, b, n, k, m, batch, n * k, k * m, c_bs, c=init.copy()), f"c_bs={c_bs}")


def test_strided_offsets(cm, port):
    """run_matmul_at-style element offsets that break 16-byte alignment of every operand."""
    n, k, m, batch = 9, 37, 23, 2
    rng = np.random.default_rng(9)
    A = rand16(rng, batch * n * k + 3)
    B = rand16(rng, batch * k * m + 5)
    c = empty(batch * n * m + 7)
    ta, tb = dev(A), dev(B)
    cm.MatmulKernel(ta[3:], tb[5:], c[7:], n, k, m, batch)
    assert_same(host(c)[7:], port.matmul(A[3:], B[5:], n, k, m, batch), "offsets")


SWEEP = [(256, 256, 256, 64), (1024, 1024, 1024, 64), (4096, 4096, 4096, 64), (8192, 4096, 11008, 8)]


@pytest.mark.parametrize("n,k,m,batch", SWEEP)
@pytest.mark.big
def test_sweep_shapes(cm, port, n, k, m, batch):
    """BASELINE MatMul sweep: raw int16 uniform [-1024, 1024), seeded; sampled rows when large."""
    import torch
    rng = np.random.default_rng(42 + 2 + n)
    gen = torch.Generator(device="cpu").manual_seed(n * 31 + k)
    a = torch.randint(-1024, 1024, (batch * n * k,), dtype=torch.int16, generator=gen)
    b = torch.randint(-1024, 1024, (batch * k * m,), dtype=torch.int16, generator=gen)
    c = empty(batch * n * m)
    cm.MatmulKernel(a.cuda(), b.cuda(), c, n, k, m, batch)
    an, bn = a.numpy(), b.numpy()
    if n * k * m * batch <= (1 << 30):
        assert_same(host(c), port.matmul(an, bn, n, k, m, batch), "sweep full")
        return
    rows = 96
    bidx = rng.integers(0, batch, rows)
    ridx = rng.integers(0, n, rows)
    bidx[0], ridx[0] = batch - 1, n - 1
    want = port.matmul_rows(an, bn, n, k, m, n * k, k * m, bidx, ridx)
    got = host(c).reshape(batch, n, m)[bidx, ridx]
    assert_same(got, want, f"sweep {n}x{k}x{m} b{batch} sampled rows")


FUSED_SHAPES = [(1, 400, 120, 1), (1, 84, 10, 1), (7, 13, 5, 1), (129, 130, 131, 2), (256, 512, 1000, 1),
                (300, 17, 64, 3), (64, 0, 19, 2)]


@pytest.mark.parametrize("n,k,m,batch", FUSED_SHAPES)
@pytest.mark.parametrize("epi", [1, 2, 3])
def test_fused_bias_relu_epilogue(cm, port, n, k, m, batch, epi):
    """cm_matmul_fused == the reference sequence MatMul -> Add(bias row: size m, outer n,
    a_inc m, b_inc 0) -> Relu, word for word, per batch step; full-range words so the
    bias add saturates both ways."""
    rng = np.random.default_rng(n * 131 + k * 7 + m + 1000 * epi)
    a = rand16(rng, max(batch * n * k, 1))
    b = rand16(rng, max(batch * k * m, 1))
    bias = rand16(rng, m, -32768, 32768)
    c = empty(batch * n * m)
    cm.kernels.MatmulKernelFused(dev(a), dev(b), c, n, k, m, batch, epilogue=epi, bias=dev(bias))
    want = port.matmul(a, b, n, k, m, batch)[: batch * n * m] if k else np.zeros(batch * n * m, np.int16)
    for z in range(batch):
        t = want[z * n * m:(z + 1) * n * m]
        if epi & 2:
            t = port.vectorop(t, bias, m, 0, n, m, 0, c=t.copy())[: n * m]
        if epi & 1:
            t = port.vectorop(t, None, n * m, 4, 1, 0, 0)[: n * m]
        want[z * n * m:(z + 1) * n * m] = t
    assert_same(host(c), want, f"fused {n}x{k}x{m} b{batch} epi{epi}")


def test_fused_rejects_bad_epilogue(cm):
    from cormorant_b200 import CormorantError
    c = empty(16)
    with pytest.raises(CormorantError):
        cm.kernels.MatmulKernelFused(dev(np.ones(16, np.int16)), dev(np.ones(16, np.int16)), c, 4, 4, 4,
                                     epilogue=2, bias=None)
    with pytest.raises(CormorantError):
        cm.kernels.MatmulKernelFused(dev(np.ones(16, np.int16)), dev(np.ones(16, np.int16)), c, 4, 4, 4,
                                     epilogue=4, bias=dev(np.ones(4, np.int16)))


# Row-strided form (the reference scheduler's MatMul over gapped buffers, nodes.py:785-801):
# n = 1, B shared, `batch` rows of A a_bs apart, output rows c_bs apart.  Folded into one
# GEMM of `batch` rows on the tensor-core path.
ROW_STRIDED = [(84, 10, 3, 88, 16), (120, 84, 3, 120, 88), (13, 70, 300, 20, 72), (257, 64, 129, 264, 64),
               (40, 200, 517, 40, 203), (1000, 33, 260, 1001, 40)]


@pytest.mark.parametrize("k,m,rows,a_bs,c_bs", ROW_STRIDED)
@pytest.mark.parametrize("epi", [0, 3])
def test_row_strided_rows(cm, port, k, m, rows, a_bs, c_bs, epi):
    rng = np.random.default_rng(k * 7 + m + rows)
    a = rand16(rng, (rows - 1) * a_bs + k, -1024, 1024)
    b = rand16(rng, k * m, -1024, 1024)
    bias = rand16(rng, m, -4096, 4096)
    init = np.full((rows - 1) * c_bs + m, -23131, np.int16)
    c = dev(init)
    if epi:
        cm.kernels.MatmulKernelFused(dev(a), dev(b), c, 1, k, m, rows, a_bs, 0, c_bs, epilogue=epi, bias=dev(bias))
    else:
        cm.MatmulKernel(dev(a), dev(b), c, 1, k, m, rows, a_bs, 0, c_bs)
    want = port.matmul(a, b, 1, k, m, rows, a_bs, 0, c_bs, c=init.copy())
    if epi & 2:
        want = port.vectorop(want, bias, m, 0, rows, c_bs, 0, c=want.copy())
    if epi & 1:
        for r in range(rows):          # ReLU on the data words of each row; gap words untouched
            seg = want[r * c_bs:r * c_bs + m]
            want[r * c_bs:r * c_bs + m] = np.maximum(seg, 0)
    assert_same(host(c), want, f"row-strided k={k} m={m} rows={rows} a_bs={a_bs} c_bs={c_bs} epi={epi}")


@pytest.mark.big
def test_row_strided_full_size(cm, port):
    """4096 gapped rows x K = 512 x M = 1000 (rows 520 and 1008 words apart), whole output."""
    k, m, rows, a_bs, c_bs = 512, 1000, 4096, 520, 1008
    rng = np.random.default_rng(77)
    a = rand16(rng, (rows - 1) * a_bs + k, -1024, 1024)
    b = rand16(rng, k * m, -1024, 1024)
    init = np.full((rows - 1) * c_bs + m, -23131, np.int16)
    c = dev(init)
    cm.MatmulKernel(dev(a), dev(b), c, 1, k, m, rows, a_bs, 0, c_bs)
    assert_same(host(c), port.matmul(a, b, 1, k, m, rows, a_bs, 0, c_bs, c=init.copy()), "row-strided 4096x512x1000")


# Large calls run as batch chunks, each chunk's split overlapping the previous chunk's GEMM
# (at least 2^37 multiply-adds a chunk): broadcast operands, gapped outputs, the fused
# epilogue.  Checked on sampled rows, the last row of the last batch step included.
CHUNKED = [(2048, 2048, 2048, 48, "a"), (2048, 2048, 2048, 48, "b"), (4096, 2048, 1536, 24, None),
           (8192, 2048, 2048, 8, None)]


@pytest.mark.big
@pytest.mark.parametrize("n,k,m,batch,bcast", CHUNKED)
@pytest.mark.parametrize("epi", [0, 3])
def test_chunked_batches(cm, port, n, k, m, batch, bcast, epi):
    rng = np.random.default_rng(n + k + m + batch + epi)
    a_bs = 0 if bcast == "a" else n * k
    b_bs = 0 if bcast == "b" else k * m
    c_bs = n * m + 24                                   # a gap after every output slice
    a = rand16(rng, (batch - 1) * a_bs + n * k, -1024, 1024)
    b = rand16(rng, (batch - 1) * b_bs + k * m, -1024, 1024)
    bias = rand16(rng, m, -4096, 4096)
    init = np.full((batch - 1) * c_bs + n * m, -23131, np.int16)
    c = dev(init)
    if epi:
        cm.kernels.MatmulKernelFused(dev(a), dev(b), c, n, k, m, batch, a_bs, b_bs, c_bs, epilogue=epi,
                                     bias=dev(bias))
    else:
        cm.MatmulKernel(dev(a), dev(b), c, n, k, m, batch, a_bs, b_bs, c_bs)
    got = host(c)
    bidx = rng.integers(0, batch, 64)
    ridx = rng.integers(0, n, 64)
    bidx[0], ridx[0] = batch - 1, n - 1
    want = port.matmul_rows(a, b, n, k, m, a_bs, b_bs, bidx, ridx)
    if epi & 2:
        want = np.clip(want.astype(np.int32) + bias.astype(np.int32), -32768, 32767).astype(np.int16)
    if epi & 1:
        want = np.maximum(want, 0)
    rows = np.stack([got[z * c_bs + r * m: z * c_bs + (r + 1) * m] for z, r in zip(bidx, ridx)])
    assert_same(rows, want, f"chunked {n}x{k}x{m} b{batch} bcast={bcast} epi={epi}")
    gaps = np.concatenate([got[z * c_bs + n * m:(z + 1) * c_bs] for z in range(batch - 1)])
    assert (gaps == -23131).all()                       # the words between slices stay untouched


@pytest.mark.parametrize("n,k,m,batch", [(256, 4096, 384, 1), (129, 2048, 131, 2), (300, 1024, 64, 1)])
@pytest.mark.parametrize("splits", [0, 2, 3, 4])
def test_k_split_units(cm, port, n, k, m, batch, splits):
    """K-split MatMul GEMMs (a tile's K blocks over 2-4 units, int32 partial sums added
    with wrap before the narrowing) give the reference words; with the fused bias + Relu
    epilogue too.  Full-range words: the partial sums wrap."""
    from cormorant_b200 import _lib
    rng = np.random.default_rng(n + k + m + splits)
    a = rand16(rng, batch * n * k)
    b = rand16(rng, batch * k * m)
    bias = rand16(rng, m)
    want = port.matmul(a, b, n, k, m, batch)[: batch * n * m]
    L = _lib.lib()
    old = L.cm_set_gemm_split(splits)
    try:
        c = empty(batch * n * m)
        cm.MatmulKernel(dev(a), dev(b), c, n, k, m, batch)
        assert_same(host(c), want, f"K-split {splits}: {n}x{k}x{m} b{batch}")
        c = empty(batch * n * m)
        cm.kernels.MatmulKernelFused(dev(a), dev(b), c, n, k, m, batch, epilogue=3, bias=dev(bias))
    finally:
        L.cm_set_gemm_split(old)
    for z in range(batch):
        t = want[z * n * m:(z + 1) * n * m]
        t = port.vectorop(t, bias, m, 0, n, m, 0, c=t.copy())[: n * m]
        want[z * n * m:(z + 1) * n * m] = port.vectorop(t, None, n * m, 4, 1, 0, 0)[: n * m]
    assert_same(host(c), want, f"K-split {splits} fused: {n}x{k}x{m} b{batch}")


@pytest.mark.parametrize("n,k,m,batch,a_bcast", [(64, 512, 1000, 1, 0), (256, 512, 1000, 1, 0), (300, 261, 64, 3, 0),
                                                 (129, 130, 131, 2, 1), (7, 13, 5, 1, 0), (1, 400, 120, 5, 0)])
@pytest.mark.parametrize("epi", [0, 3])
def test_prepared_b_matches_fused(cm, port, n, k, m, batch, a_bcast, epi):
    """cm_matmul_prepared with B prepared once equals the reference MatMul (+ bias row Add +
    Relu) with B broadcast over the batch, word for word, over repeated calls -- on the
    one-GEMM form and on the paths that read B itself (launch-bound sizes, the row-strided
    form of n = 1)."""
    from cormorant_b200 import kernels
    rng = np.random.default_rng(n * 3 + k + m + batch + epi)
    a_bs = 0 if a_bcast else n * k
    a = rand16(rng, (1 if a_bcast else batch) * n * k)
    b = rand16(rng, k * m)
    bias = rand16(rng, m)
    want = port.matmul(a, b, n, k, m, batch, a_bs, 0, n * m)[: batch * n * m]
    for z in range(batch):
        t = want[z * n * m:(z + 1) * n * m]
        if epi & 2:
            t = port.vectorop(t, bias, m, 0, n, m, 0, c=t.copy())[: n * m]
        if epi & 1:
            t = port.vectorop(t, None, n * m, 4, 1, 0, 0)[: n * m]
        want[z * n * m:(z + 1) * n * m] = t
    bd = dev(b)
    w = kernels.MatmulWeights(bd, k, m)
    try:
        for rep in range(2):
            c = empty(batch * n * m)
            kernels.MatmulKernelPrepared(w, dev(a), c, n, batch, a_bs, n * m, epilogue=epi,
                                         bias=dev(bias) if epi & 2 else None)
            assert_same(host(c), want, f"prepared B {n}x{k}x{m} b{batch} epi {epi} call {rep}")
    finally:
        w.close()


def test_prepared_b_refusals(cm):
    from cormorant_b200 import CormorantError, _lib, kernels
    import ctypes as C
    L = _lib.lib()
    out = C.c_void_p(1)
    assert L.cm_matmul_weights_create(None, 16, 16, C.byref(out)) != 0 and not out.value
    w = kernels.MatmulWeights(dev(np.ones(64 * 32, np.int16)), 64, 32)
    try:
        with pytest.raises(CormorantError):          # bias row without a bias
            kernels.MatmulKernelPrepared(w, dev(np.ones(8 * 64, np.int16)), empty(8 * 32), 8, epilogue=2)
        with pytest.raises(CormorantError):          # epilogue out of range
            kernels.MatmulKernelPrepared(w, dev(np.ones(8 * 64, np.int16)), empty(8 * 32), 8, epilogue=4)
    finally:
        w.close()
    assert L.cm_matmul_prepared(None, None, None, 1, 1, 0, 0, 0, None) != 0


def test_k_split_launches_on_two_streams(cm, port):
    """K-split GEMMs queued on two unordered streams at once: each launch has its own slabs
    and arrival counters, so both give the reference words."""
    import torch
    from cormorant_b200 import _lib
    shapes = [(256, 4096, 384), (300, 2048, 200)]
    rng = np.random.default_rng(99)
    ops = []
    for (n, k, m) in shapes:
        a, b = rand16(rng, n * k), rand16(rng, k * m)
        ops.append((n, k, m, dev(a), dev(b), port.matmul(a, b, n, k, m)[: n * m]))
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    L = _lib.lib()
    old = L.cm_set_gemm_split(2)
    try:
        outs = [[empty(n * m) for (n, _, m, _, _, _) in ops] for _ in range(4)]
        torch.cuda.synchronize()                   # inputs and poisoned outputs are in place
        for rep in range(4):
            for (n, k, m, ad, bd, _), st, c in zip(ops, streams, outs[rep]):
                cm.MatmulKernel(ad, bd, c, n, k, m, 1, stream=st)
        torch.cuda.synchronize()
    finally:
        L.cm_set_gemm_split(old)
    for rep in range(4):
        for (n, k, m, _, _, want), c in zip(ops, outs[rep]):
            assert_same(host(c), want, f"two streams, call {rep}: {n}x{k}x{m}")
