"""Drop-in `softmax` module for AutoKernel's kernel.py slot (replaces kernels/softmax.py:57).

Copy or import as ``kernel.py``: AutoKernel's bench.py reads KERNEL_TYPE and
calls kernel_fn(**inputs); verify.py calls kernel_fn positionally.
"""
from autokernel_b200 import ops

KERNEL_TYPE = "softmax"


def kernel_fn(x):
    return ops.softmax(x)
