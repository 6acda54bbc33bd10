"""Drop-in `reduce` module for AutoKernel's kernel.py slot (replaces kernels/reduce.py:51).

Copy or import as ``kernel.py``: AutoKernel's bench.py reads KERNEL_TYPE and
calls kernel_fn(**inputs); verify.py calls kernel_fn positionally.
"""
from autokernel_b200 import ops

KERNEL_TYPE = "reduce"


def kernel_fn(x, dim=-1):
    return ops.reduce(x, dim)
