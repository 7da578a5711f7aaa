"""cm_matmul_noalloc: the MatMul entry point for callers that cannot allocate device
memory while running (a run loop that must not allocate after initialisation, or
code whose GPU memory is owned by another allocator).  It keeps its scratch in a
fixed device array inside the library instead of calling cudaMalloc.

Checked through the C ABI, bit-exact like every MatMul test, against the oracle's
MatMul and against the regular cm_matmul, on calls in a row with different shapes and
data (so a stale array from an earlier call would show): partial tiles, A broadcast,
outputs of at most 64 columns, overlapping output slices (c_batch_stride < n*m, later
batch steps win) and c_batch_stride = 0, a launch-bound call that needs no scratch at
all; plus the clear rejection of a call whose scratch need exceeds the array.  Named
test_zz_* so pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# (n, k, m, batch, a_batch_stride is zero, c_batch_stride or None for n*m)
CASES = [
    (300, 1000, 200, 3, False, None),     # partial tiles, both strides advance
    (257, 513, 129, 4, True, None),       # A broadcast
    (300, 257, 40, 3, False, None),       # m <= 64
    (129, 1000, 64, 2, False, None),      # m = 64
    (200, 300, 150, 3, False, 200 * 150 // 2),   # overlapping output slices
    (130, 140, 150, 3, False, 0),         # every batch step on the same output
    (7, 13, 5, 2, False, None),           # launch-bound: no scratch needed
]


def _p(t):
    return C.c_void_p(t.data_ptr())


def test_noalloc_matches_oracle_and_cm_matmul(port):
    import torch

    import cormorant_b200 as cm
    from cormorant_b200._lib import lib

    cm.init("0")
    L = lib()
    gen = torch.Generator().manual_seed(314)
    for (n, k, m, batch, a_bcast, c_bs) in CASES:
        c_bs = n * m if c_bs is None else c_bs
        a = torch.randint(-32768, 32768, ((1 if a_bcast else batch) * n * k,), dtype=torch.int32, generator=gen)
        b = torch.randint(-32768, 32768, (batch * k * m,), dtype=torch.int32, generator=gen)
        a16, b16 = a.to(torch.int16), b.to(torch.int16)
        a_bs = 0 if a_bcast else n * k
        out_words = (batch - 1) * c_bs + n * m
        want = torch.full((out_words,), -23131, dtype=torch.int16, device="cuda")
        got = torch.full((out_words,), -23131, dtype=torch.int16, device="cuda")
        ad, bd = a16.cuda(), b16.cuda()
        assert L.cm_matmul(_p(ad), _p(bd), _p(want), n, k, m, batch, a_bs, k * m, c_bs) == 0, L.cm_last_error()
        rc = L.cm_matmul_noalloc(_p(ad), _p(bd), _p(got), n, k, m, batch, a_bs, k * m, c_bs, None)
        assert rc == 0, L.cm_last_error()
        assert L.cm_synchronize(None) == 0, L.cm_last_error()
        g, w = got.cpu().numpy(), want.cpu().numpy()
        o = port.matmul(a16.numpy(), b16.numpy(), n, k, m, batch, a_bs, k * m, c_bs,
                        c=np.full(out_words, -23131, np.int16))
        case = (n, k, m, batch, a_bs, c_bs)
        assert np.array_equal(g, o), f"{int((g != o).sum())} words differ from the oracle for {case}"
        assert np.array_equal(g, w), f"{int((g != w).sum())} words differ from cm_matmul for {case}"


def test_noalloc_rejects_oversized_calls():
    import torch

    import cormorant_b200 as cm
    from cormorant_b200._lib import CM_EINVAL, lib

    cm.init("0")
    L = lib()
    n = k = m = 4096          # planes alone need 2 * 2 * 4096 * 4096 bytes = 64 MiB, plus terms
    a = torch.zeros(n * k, dtype=torch.int16, device="cuda")
    c = torch.zeros(n * m, dtype=torch.int16, device="cuda")
    rc = L.cm_matmul_noalloc(_p(a), _p(a), _p(c), n, k, m, 1, n * k, k * m, n * m, None)
    assert rc == CM_EINVAL
    assert b"scratch" in L.cm_last_error()


def test_noalloc_allocates_nothing_even_where_the_gemm_would_split(port):
    """A small grid is where the tensor-core GEMM may divide its tiles' K blocks among units,
    which needs slab memory from the stream-ordered pool; the allocation-free entry never
    does that.  With four-way splits forced, the device's default memory pool (the one the
    library's scratch comes from) must not grow during two cm_matmul_noalloc calls, while
    the same check around cm_matmul sees its scratch (so the check itself works)."""
    import torch
    from cuda.bindings import driver as drv

    import cormorant_b200 as cm
    from cormorant_b200._lib import lib

    cm.init("0")
    L = lib()
    n, k, m = 300, 1024, 200
    gen = torch.Generator().manual_seed(2718)
    a16 = torch.randint(-32768, 32768, (n * k,), dtype=torch.int32, generator=gen).to(torch.int16)
    b16 = torch.randint(-32768, 32768, (k * m,), dtype=torch.int32, generator=gen).to(torch.int16)
    ad, bd = a16.cuda(), b16.cuda()
    want = port.matmul(a16.numpy(), b16.numpy(), n, k, m)[: n * m]
    assert drv.cuInit(0)[0] == drv.CUresult.CUDA_SUCCESS
    err, dev = drv.cuDeviceGet(torch.cuda.current_device())
    assert err == drv.CUresult.CUDA_SUCCESS
    err, pool = drv.cuDeviceGetDefaultMemPool(dev)
    assert err == drv.CUresult.CUDA_SUCCESS
    attr_cur = drv.CUmemPool_attribute.CU_MEMPOOL_ATTR_USED_MEM_CURRENT
    attr_high = drv.CUmemPool_attribute.CU_MEMPOOL_ATTR_USED_MEM_HIGH

    def pool_growth(call):
        torch.cuda.synchronize()
        err, cur = drv.cuMemPoolGetAttribute(pool, attr_cur)
        assert err == drv.CUresult.CUDA_SUCCESS
        assert drv.cuMemPoolSetAttribute(pool, attr_high, drv.cuuint64_t(0))[0] == drv.CUresult.CUDA_SUCCESS
        call()
        torch.cuda.synchronize()
        err, high = drv.cuMemPoolGetAttribute(pool, attr_high)
        assert err == drv.CUresult.CUDA_SUCCESS
        return int(high) - int(cur)

    old = L.cm_set_gemm_split(4)
    try:
        c_ref = torch.zeros(n * m, dtype=torch.int16, device="cuda")
        assert pool_growth(lambda: L.cm_matmul(_p(ad), _p(bd), _p(c_ref), n, k, m, 1, n * k, k * m, n * m)) > 0
        outs = [torch.full((n * m,), -23131, dtype=torch.int16, device="cuda") for _ in range(2)]

        def two_calls():
            for c in outs:
                assert L.cm_matmul_noalloc(_p(ad), _p(bd), _p(c), n, k, m, 1, n * k, k * m, n * m, None) == 0, \
                    L.cm_last_error()
        assert pool_growth(two_calls) == 0
    finally:
        L.cm_set_gemm_split(old)
    for c in outs:
        assert np.array_equal(c.cpu().numpy(), want)
    assert np.array_equal(c_ref.cpu().numpy(), want)
