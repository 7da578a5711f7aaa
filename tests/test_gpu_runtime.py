"""The runtime mirror on the GPU: stream-ordered buffer syncs, run_* on a stream, the
overlapped-copy runner the bench's end-to-end figures use, and the int8 tensor-pipe
ceiling measurement.  Every result is checked bit-exact against the oracle."""
import ctypes as C

import numpy as np
import pytest

from tests._util import assert_same, rand16

pytestmark = pytest.mark.gpu


def test_async_syncs_and_run_on_stream(cm, port):
    """cm_buf_sync_to_device_async -> run_matmul(stream) -> cm_buf_sync_from_device_async."""
    import torch
    from cormorant_b200.runtime import InferenceBuf, run_matmul
    n, k, m, batch = 130, 257, 70, 2
    rng = np.random.default_rng(5)
    a, b = rand16(rng, batch * n * k, -1024, 1024), rand16(rng, batch * k * m, -1024, 1024)
    A, B, Cb = InferenceBuf.alloc(a.size), InferenceBuf.alloc(b.size), InferenceBuf.alloc(batch * n * m)
    try:
        A.ptr()[:] = a
        B.ptr()[:] = b
        Cb.ptr()[:] = -23131
        s = torch.cuda.Stream()
        A.sync_to_device(s)
        B.sync_to_device(s)
        run_matmul(A, B, Cb, n, k, m, batch, n * k, k * m, n * m, stream=s)
        Cb.sync_from_device(s)
        s.synchronize()
        assert_same(Cb.ptr().copy(), port.matmul(a, b, n, k, m, batch), "async syncs")
    finally:
        for x in (A, B, Cb):
            x.free()


def test_copy_overlap_sequence(cm, port):
    """Several calls through CopyOverlap, buffers reused across two steps: every output
    read back after the run equals the oracle (ordering of reuse is what is tested)."""
    import torch
    from cormorant_b200.runtime import CopyOverlap, InferenceBuf, run_op, run_pool
    rng = np.random.default_rng(17)
    n = 1 << 16
    sets = []
    for _ in range(2):
        A, B, Cc = (InferenceBuf.alloc(n) for _ in range(3))
        sets.append((A, B, Cc))
    X = InferenceBuf.alloc(2 * 6 * 28 * 28)
    Y = InferenceBuf.alloc(2 * 6 * 14 * 14)
    try:
        pipe = CopyOverlap()
        start = torch.cuda.Event()
        start.record()
        pipe.start(start)
        want, got = [], []
        for step in range(2):
            for i, op in enumerate((0, 2, 3, 4)):
                A, B, Cc = sets[i % 2]
                a, b = rand16(rng, n), rand16(rng, n, 1, 32768)
                # the host mirrors may only change once their last upload is done
                pipe.up.synchronize()
                A.ptr()[:] = a
                B.ptr()[:] = b
                pipe.call([A, B], [Cc], lambda s, A=A, B=B, Cc=Cc, op=op:
                          run_op(A, B if op < 4 else None, Cc, n, op, 1, 0, 0, stream=s))
                pipe.down.synchronize()
                got.append(Cc.ptr().copy())
                want.append(port.vectorop(a, b, n, op))
            x = rand16(rng, X.count(), -2048, 2048)
            pipe.up.synchronize()
            X.ptr()[:] = x
            pipe.call([X], [Y], lambda s: run_pool(X, Y, 2, 6, 28, 28, 14, 14, 2, 2, 2, 2, 0, 0, 1, 1, 1, 2, 0,
                                                   stream=s))
            pipe.join()
            torch.cuda.synchronize()
            got.append(Y.ptr().copy())
            want.append(port.pool(x, 2, 6, 28, 28, 14, 14, 2, 2, 2, 2, 0, 0, 1, 1, 1, 2, 0))
        for i, (g, w) in enumerate(zip(got, want)):
            assert_same(g, w, f"call {i}")
    finally:
        for t in sets:
            for x in t:
                x.free()
        X.free()
        Y.free()


def test_copy_overlap_views(cm, port):
    """A batched MatMul run as batch chunks through views of its owners (the bench's e2e
    form: disjoint views of one owner overlap each other), then, in the next step, once
    over the whole owners (a call on an owner is ordered after its views' copies and
    kernels), then chunked again; every read-back equals the oracle."""
    import torch
    from cormorant_b200.runtime import CopyOverlap, InferenceBuf, run_matmul
    n, k, m, batch, items = 96, 160, 72, 7, 2
    rng = np.random.default_rng(23)
    A, B, Cb = InferenceBuf.alloc(batch * n * k), InferenceBuf.alloc(batch * k * m), InferenceBuf.alloc(batch * n * m)
    chunks = []
    for i0 in range(0, batch, items):
        c = min(items, batch - i0)
        chunks.append((c, InferenceBuf.init_view(A, i0 * n * k, c * n * k), InferenceBuf.init_view(B, i0 * k * m, c * k * m),
                       InferenceBuf.init_view(Cb, i0 * n * m, c * n * m)))
    try:
        pipe = CopyOverlap()
        start = torch.cuda.Event()
        start.record()
        pipe.start(start)
        for step, whole in enumerate((False, True, False)):
            a, b = rand16(rng, A.count(), -1024, 1024), rand16(rng, B.count(), -1024, 1024)
            torch.cuda.synchronize()
            A.ptr()[:] = a
            B.ptr()[:] = b
            Cb.ptr()[:] = -23131
            if whole:
                pipe.call([A, B], [Cb], lambda s: run_matmul(A, B, Cb, n, k, m, batch, n * k, k * m, n * m, stream=s))
            else:
                for (c, Av, Bv, Cv) in chunks:
                    pipe.call([Av, Bv], [Cv], lambda s, c=c, Av=Av, Bv=Bv, Cv=Cv:
                              run_matmul(Av, Bv, Cv, n, k, m, c, n * k, k * m, n * m, stream=s))
            pipe.join()
            torch.cuda.synchronize()
            assert_same(Cb.ptr().copy(), port.matmul(a, b, n, k, m, batch), f"step {step} whole={whole}")
    finally:
        for x in (A, B, Cb):
            x.free()


@pytest.mark.parametrize("pairs", [0, 1])
def test_int8_mma_rate(cm, pairs):
    """The ceiling measurement runs, returns a plausible rate and leaves the library usable."""
    from cormorant_b200 import _lib
    L = _lib.lib()
    tops, ms, mhz = C.c_double(), C.c_double(), C.c_double()
    _lib.check(L.cm_int8_mma_rate(pairs, 2048, C.byref(tops), C.byref(ms), C.byref(mhz)))
    assert ms.value > 0.0
    # between a tenth of and twice the datasheet's dense int8 rate (4.5 POPS)
    assert 450.0 < tops.value < 9000.0, tops.value
    # an SM clock between 300 MHz and the B200's 1965 MHz maximum (plus measurement slack)
    assert 300.0 < mhz.value < 2100.0, mhz.value
    _lib.check(L.cm_int8_mma_rate(pairs, 16, C.byref(tops), C.byref(ms), None))
    assert L.cm_int8_mma_rate(pairs, 0, C.byref(tops), C.byref(ms), None) == _lib.CM_EINVAL
    assert L.cm_int8_mma_rate(2, 16, C.byref(tops), C.byref(ms), None) == _lib.CM_EINVAL


def test_profile_gemm_clock(cm):
    """While profiling, tensor-core GEMM launches record the SM clock they ran at; without a
    GEMM since cm_profile_begin the clock reads 0."""
    import torch
    from cormorant_b200 import _lib
    L = _lib.lib()
    mhz = C.c_double(-1.0)
    _lib.check(L.cm_profile_begin())
    _lib.check(L.cm_profile_end())
    _lib.check(L.cm_profile_gemm_clock(C.byref(mhz)))
    assert mhz.value == 0.0
    n = k = m = 1024
    a = torch.zeros(n * k, dtype=torch.int16, device="cuda")
    c = torch.empty(n * m, dtype=torch.int16, device="cuda")
    old = L.cm_set_direct_limit(0)                       # the tensor-core path
    try:
        _lib.check(L.cm_profile_begin())
        for _ in range(3):
            _lib.check(L.cm_matmul(C.c_void_p(a.data_ptr()), C.c_void_p(a.data_ptr()), C.c_void_p(c.data_ptr()),
                                   n, k, m, 1, n * k, k * m, n * m))
        _lib.check(L.cm_profile_end())
        _lib.check(L.cm_profile_gemm_clock(C.byref(mhz)))
    finally:
        L.cm_set_direct_limit(old)
    assert 300.0 < mhz.value < 2100.0, mhz.value
    assert L.cm_profile_gemm_clock(None) == _lib.CM_EINVAL
