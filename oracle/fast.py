"""Exact numpy restatement of MatmulKernel for large shapes (test infrastructure only).

MatmulKernel (kernels/matmul/kernel/MatmulKernel.cpp:196-219) forms the exact
integer sum of int16 x int16 products in an int32 accumulator that wraps, then
narrows once: floor by 8 bits and clamp to int16.  Raw products are below
2^30 in magnitude, so any partial sum over K < 2^23 terms is an integer below
2^53 and a float64 GEMM (even with FMA and any summation order) is exact.
"""
from __future__ import annotations

import numpy as np


def narrow_acc(acc_int: np.ndarray) -> np.ndarray:
    """saturate_cast<ap_fixed<16,8>>(ap_fixed<32,16>): wrap to int32, floor >> 8, clamp."""
    wrapped = (acc_int.astype(np.int64) & 0xFFFFFFFF).astype(np.uint32).view(np.int32)
    return np.clip(wrapped.astype(np.int64) >> 8, -32768, 32767).astype(np.int16)


def matmul_2d(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """C[n][m] for one batch item; a is [n,k] int16, b is [k,m] int16."""
    k = a.shape[1]
    if k >= (1 << 23):
        raise ValueError("float64 exactness bound exceeded")
    acc = a.astype(np.float64) @ b.astype(np.float64)
    return narrow_acc(acc.astype(np.int64))
