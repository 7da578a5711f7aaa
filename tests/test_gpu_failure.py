"""Failure detection on the GPU without a fault: a device-side bounded wait that can
never be satisfied expires, the kernel reports CM_ETIMEOUT through the status word and
returns, and the library keeps working afterwards (the status word is cleared)."""
import numpy as np
import pytest

from cormorant_b200 import _lib
from tests._util import assert_same, dev, empty, host, rand16

pytestmark = pytest.mark.gpu


def test_wait_expiry_reports_timeout_and_context_survives(cm, port):
    L = _lib.lib()
    rc = L.cm_selftest_wait_timeout(50)
    assert rc == _lib.CM_ETIMEOUT, rc
    assert b"status" in L.cm_last_error()
    # the status word was cleared and the context is intact
    assert L.cm_synchronize(None) == _lib.CM_OK
    rng = np.random.default_rng(5)
    a, b = rand16(rng, 4096), rand16(rng, 4096)
    c = empty(4096)
    cm.VectorOPKernel(dev(a), dev(b), c, 4096, 0, 1, 0, 0)
    assert_same(host(c), port.vectorop(a, b, 4096, 0, 1, 0, 0), "vectorop after a timeout")


def test_wait_expiry_argument_checks(cm):
    L = _lib.lib()
    assert L.cm_selftest_wait_timeout(0) == _lib.CM_EINVAL
    assert L.cm_selftest_wait_timeout(20000) == _lib.CM_EINVAL
