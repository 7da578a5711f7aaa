"""cormorant_b200 -- B200 (sm_100a) implementation of Cormorant's Q8.8 kernels.

VectorOPKernel, MatmulKernel, ConvKernel and PoolingKernel run as hand-written
CUDA kernels in ``libcormorant_cuda.so`` behind a C ABI (include/cormorant_cuda.h);
this package is the Python host side: a ctypes binding, the kernel-call
mirror (``kernels``), the inference_buf / run_* mirror (``runtime``) and the
batch-sharded multi-GPU driver (``sharding``).
"""
from ._lib import CormorantError, lib  # noqa: F401
from .kernels import (  # noqa: F401
    OP_ADD, OP_DIV, OP_MUL, OP_RELU, OP_RELU6, OP_SUB, POOL_AVG, POOL_LP, POOL_MAX,
    ConvKernel, ConvKernelFused, MatmulKernel, MatmulKernelFused, PoolingKernel, VectorOPKernel, init,
    launch_count, release, synchronize,
)
