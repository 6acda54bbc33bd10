"""Drop-in `rotary_embedding` module for AutoKernel's kernel.py slot (replaces kernels/rotary_embedding.py:75).

Copy or import as ``kernel.py``: AutoKernel's bench.py reads KERNEL_TYPE and
calls kernel_fn(**inputs); verify.py calls kernel_fn positionally.
"""
from autokernel_b200 import ops

KERNEL_TYPE = "rotary_embedding"


def kernel_fn(x, cos, sin):
    return ops.rotary_embedding(x, cos, sin)
