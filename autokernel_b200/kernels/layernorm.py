"""Drop-in `layernorm` module for AutoKernel's kernel.py slot (replaces kernels/layernorm.py:65).

Copy or import as ``kernel.py``: AutoKernel's bench.py reads KERNEL_TYPE and
calls kernel_fn(**inputs); verify.py calls kernel_fn positionally.
"""
from autokernel_b200 import ops

KERNEL_TYPE = "layernorm"


def kernel_fn(x, weight, bias, eps=1e-5):
    return ops.layernorm(x, weight, bias, eps)
