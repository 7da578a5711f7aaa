"""CPU parity checkers for the Cormorant Q8.8 kernels.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline legs of ``bench.py`` may import this package, and only as the
checker or the timed CPU baseline -- the product (``cormorant_b200``) never
imports it and has no CPU fallback.

Two independent checkers share one numpy-facing interface:

* ``port()`` -- ``liboracle.so``, this repository's C restatement of the four
  kernels (``oracle/cm_oracle.c``);
* ``ref()``  -- ``_ref/libref_*.so``, the unmodified reference kernels
  (``kernels/*/kernel/*.cpp``) compiled in place against this directory's
  ``ap_fixed.h`` / ``hls_stream.h`` shims (``oracle/Makefile``).

``fast`` holds an exact numpy (float64 BLAS) restatement of MatMul for sizes
the C loops cannot finish quickly.
"""
from .api import build, have_ref, port, ref, ORACLE_DIR  # noqa: F401
