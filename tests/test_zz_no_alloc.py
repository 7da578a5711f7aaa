"""cm_matmul_noalloc: the MatMul entry point for callers that cannot allocate device
memory while running (a run loop that must not allocate after initialisation, or
code whose GPU memory is owned by another allocator).  It keeps its scratch in a
fixed device array inside the library instead of calling cudaMalloc.

Checked through the C ABI against the regular cm_matmul on two calls in a row
(different shapes and data, so a stale array from the first call would show),
bit-exact like every MatMul test, plus the clear rejection of a call whose
scratch need exceeds the array.  Named test_zz_* so pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_noalloc_matches_cm_matmul_twice():
    import torch

    import cormorant_b200 as cm
    from cormorant_b200._lib import lib

    cm.init("0")
    L = lib()
    gen = torch.Generator().manual_seed(314)
    # (n, k, m, batch, a_batch_stride-is-zero): partial tiles, both strides, A broadcast
    for (n, k, m, batch, a_bcast) in [(300, 1000, 200, 3, False), (257, 513, 129, 4, True)]:
        a = torch.randint(-32768, 32768, ((1 if a_bcast else batch) * n * k,), dtype=torch.int32, generator=gen)
        b = torch.randint(-32768, 32768, (batch * k * m,), dtype=torch.int32, generator=gen)
        a = a.to(torch.int16).cuda()
        b = b.to(torch.int16).cuda()
        a_bs = 0 if a_bcast else n * k
        want = torch.full((batch * n * m,), -23131, dtype=torch.int16, device="cuda")
        got = torch.full((batch * n * m,), -23131, dtype=torch.int16, device="cuda")
        assert L.cm_matmul(C.c_void_p(a.data_ptr()), C.c_void_p(b.data_ptr()), C.c_void_p(want.data_ptr()),
                           n, k, m, batch, a_bs, k * m, n * m) == 0, L.cm_last_error()
        rc = L.cm_matmul_noalloc(C.c_void_p(a.data_ptr()), C.c_void_p(b.data_ptr()), C.c_void_p(got.data_ptr()),
                                 n, k, m, batch, a_bs, k * m, n * m, None)
        assert rc == 0, L.cm_last_error()
        assert L.cm_synchronize(None) == 0, L.cm_last_error()
        g, w = got.cpu().numpy(), want.cpu().numpy()
        assert np.array_equal(g, w), f"{int((g != w).sum())} words differ for {(n, k, m, batch)}"


def test_noalloc_rejects_oversized_calls():
    import torch

    import cormorant_b200 as cm
    from cormorant_b200._lib import CM_EINVAL, lib

    cm.init("0")
    L = lib()
    n = k = m = 4096          # planes alone need 2 * 2 * 4096 * 4096 bytes = 64 MiB, plus terms
    a = torch.zeros(n * k, dtype=torch.int16, device="cuda")
    c = torch.zeros(n * m, dtype=torch.int16, device="cuda")
    rc = L.cm_matmul_noalloc(C.c_void_p(a.data_ptr()), C.c_void_p(a.data_ptr()), C.c_void_p(c.data_ptr()),
                             n, k, m, 1, n * k, k * m, n * m, None)
    assert rc == CM_EINVAL
    assert b"scratch" in L.cm_last_error()
