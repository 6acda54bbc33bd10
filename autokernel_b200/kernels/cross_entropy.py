"""Drop-in `cross_entropy` module for AutoKernel's kernel.py slot (replaces kernels/cross_entropy.py:70).

Copy or import as ``kernel.py``: AutoKernel's bench.py reads KERNEL_TYPE and
calls kernel_fn(**inputs); verify.py calls kernel_fn positionally.
"""
from autokernel_b200 import ops

KERNEL_TYPE = "cross_entropy"


def kernel_fn(logits, targets):
    return ops.cross_entropy(logits, targets)
