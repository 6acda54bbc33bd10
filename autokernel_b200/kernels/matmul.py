"""Drop-in `matmul` module for AutoKernel's kernel.py slot (replaces kernels/matmul.py:62).

Copy or import as ``kernel.py``: AutoKernel's bench.py reads KERNEL_TYPE and
calls kernel_fn(**inputs); verify.py calls kernel_fn positionally.
"""
from autokernel_b200 import ops

KERNEL_TYPE = "matmul"


def kernel_fn(A, B):
    return ops.matmul(A, B)
