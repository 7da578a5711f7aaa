"""VectorOPKernel parity on the GPU: cm_vectorop vs the C restatement (oracle/cm_oracle.c).

Bit-exact on raw int16 words.  Covers every op code (including the copy
default for unknown codes), flat and broadcast (outer/a_inc/b_inc) calls,
overlapping and gapped output rows, misaligned buffers, the exhaustive
int16 x int16 domain of every op, and the BASELINE sweep size 2^28.
"""
import numpy as np
import pytest

from tests._util import assert_same, dev, empty, host, rand16

pytestmark = pytest.mark.gpu

OPS = [0, 1, 2, 3, 4, 5, 6, 9]


@pytest.mark.parametrize("op", OPS)
@pytest.mark.parametrize("size", [1, 7, 8, 9, 1000, 4097, (1 << 20) + 3])
def test_flat(cm, port, op, size):
    rng = np.random.default_rng(1000 * op + size)
    a, b = rand16(rng, size), rand16(rng, size)
    if op == 3:
        b[rng.random(size) < 0.05] = 0
    c = empty(size)
    cm.VectorOPKernel(dev(a), dev(b), c, size, op, 1, 0, 0)
    assert_same(host(c), port.vectorop(a, b, size, op), f"op={op} size={size}")


@pytest.mark.parametrize("op", [0, 2, 3, 4, 5])
def test_unary_or_binary_with_null_b(cm, port, op):
    rng = np.random.default_rng(7)
    a = rand16(rng, 777)
    c = empty(777)
    if op >= 4:
        cm.VectorOPKernel(dev(a), None, c, 777, op)
        assert_same(host(c), port.vectorop(a, None, 777, op), "unary, b=NULL")
    else:
        with pytest.raises(cm.CormorantError):
            cm.VectorOPKernel(dev(a), None, c, 777, op)


# (outer, size, a_inc, b_inc): the reference's broadcast tests (TestSimulation.cpp:274-339),
# the scheduler's Gemm-bias Add (outer=batch, b_inc=0), depthwise MUL broadcast,
# plus overlapping (c_inc < size), gapped (c_inc > size) and c_inc = 0 layouts.
BCAST = [(2, 4, 4, 0), (3, 4, 0, 4), (256, 1000, 1000, 0), (12544, 16, 16, 0), (8, 16384, 16384, 0),
         (5, 8, 8, 8), (4, 7, 3, 2), (3, 5, 9, 0), (3, 16, 0, 0), (6, 24, 32, 8), (7, 64, 0, 64), (3, 9, 1, 1)]


@pytest.mark.parametrize("op", [0, 1, 2, 3, 4, 5])
@pytest.mark.parametrize("outer,size,a_inc,b_inc", BCAST)
def test_broadcast(cm, port, op, outer, size, a_inc, b_inc):
    rng = np.random.default_rng(outer * 131 + size * 7 + op)
    a = rand16(rng, (outer - 1) * a_inc + size)
    b = rand16(rng, (outer - 1) * b_inc + size)
    c_len = (outer - 1) * (a_inc + b_inc) + size
    init = np.full(c_len, -23131, np.int16)
    c = dev(init)
    cm.VectorOPKernel(dev(a), dev(b), c, size, op, outer, a_inc, b_inc)
    want = port.vectorop(a, b, size, op, outer, a_inc, b_inc, c=init.copy())
    assert_same(host(c), want, f"op={op} outer={outer} size={size} inc=({a_inc},{b_inc})")


@pytest.mark.parametrize("offs", [(1, 1, 1), (3, 3, 3), (1, 2, 3), (0, 5, 2), (7, 7, 7)])
@pytest.mark.parametrize("op", [0, 2, 3, 5])
def test_misaligned(cm, port, op, offs):
    rng = np.random.default_rng(sum(offs) * 17 + op)
    n = 10007
    big_a, big_b = rand16(rng, n + 16), rand16(rng, n + 16)
    A, B = dev(big_a), dev(big_b)
    C = empty(n + 16)
    oa, ob, oc = offs
    cm.VectorOPKernel(A[oa:oa + n], B[ob:ob + n], C[oc:oc + n], n, op)
    want = port.vectorop(big_a[oa:oa + n], big_b[ob:ob + n], n, op)
    got = host(C)
    assert_same(got[oc:oc + n], want, f"offsets {offs}")
    assert (got[:oc] == -23131).all() and (got[oc + n:] == -23131).all(), "wrote outside c"


@pytest.mark.parametrize("op", [0, 1, 2, 3, 4, 5])
def test_exhaustive_domain(cm, port, op):
    """Every (a, b) int16 pair: 2^32 evaluations per op, checked in chunks of 2^26."""
    import torch
    chunk = 1024
    bvals = torch.arange(-32768, 32768, dtype=torch.int32, device="cuda").to(torch.int16)
    b = bvals.repeat(chunk)
    c = torch.empty_like(b)
    for a0 in range(-32768, 32768, chunk):
        a = torch.arange(a0, a0 + chunk, dtype=torch.int32, device="cuda").to(torch.int16).repeat_interleave(65536)
        cm.VectorOPKernel(a, b, c, a.numel(), op)
        bad, first = port.check_pairs(op, a0, host(c))
        assert bad == 0, f"op {op}: {bad} mismatches in a-chunk {a0}, first index {first}"


@pytest.mark.parametrize("op", [0, 1, 2, 3, 4, 5])
def test_sweep_size(cm, port, op):
    """BASELINE config: 2^28 elements, full int16 range, DIV zeros replaced by 1."""
    n = 1 << 28
    rng = np.random.default_rng(42 + 3 + op)
    a, b = rand16(rng, n), rand16(rng, n)
    if op == 3:
        b[b == 0] = 1
    c = empty(n)
    cm.VectorOPKernel(dev(a), dev(b), c, n, op)
    assert_same(host(c), port.vectorop(a, b, n, op), f"sweep op={op}")


@pytest.mark.parametrize("op", [0, 1, 2, 4, 5, 7])
def test_one_launch_vectorop_matches_entry(cm, port, op):
    """cm_calls' VectorOP equals cm_vectorop (broadcast rows with gaps included)."""
    from cormorant_b200 import kernels
    rng = np.random.default_rng(op + 40)
    size, outer, a_inc, b_inc = 37, 5, 41, 3
    a = rand16(rng, outer * a_inc + size, -32768, 32768)
    b = rand16(rng, outer * b_inc + size, -32768, 32768)
    c1, c2 = empty(outer * (a_inc + b_inc) + size), empty(outer * (a_inc + b_inc) + size)
    c1.fill_(0)
    c2.fill_(0)
    cm.VectorOPKernel(dev(a), dev(b), c1, size, op, outer, a_inc, b_inc)
    kernels.RunCalls(kernels.call_array([(kernels.CALL_VECTOROP, 0, dev(a), dev(b), None, None, c2,
                                          (size, op, outer, a_inc, b_inc))]))
    assert_same(host(c2), host(c1), f"one-launch vectorop {op}")
