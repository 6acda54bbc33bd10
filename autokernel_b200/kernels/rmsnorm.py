"""Drop-in `rmsnorm` module for AutoKernel's kernel.py slot (replaces kernels/rmsnorm.py:45).

Copy or import as ``kernel.py``: AutoKernel's bench.py reads KERNEL_TYPE and
calls kernel_fn(**inputs); verify.py calls kernel_fn positionally.
"""
from autokernel_b200 import ops

KERNEL_TYPE = "rmsnorm"


def kernel_fn(x, weight, eps=1e-6):
    return ops.rmsnorm(x, weight, eps)
