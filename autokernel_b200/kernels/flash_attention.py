"""Drop-in `flash_attention` module for AutoKernel's kernel.py slot (replaces kernels/flash_attention.py:130).

Copy or import as ``kernel.py``: AutoKernel's bench.py reads KERNEL_TYPE and
calls kernel_fn(**inputs); verify.py calls kernel_fn positionally.
"""
from autokernel_b200 import ops

KERNEL_TYPE = "flash_attention"


def kernel_fn(Q, K, V, causal=True, sm_scale=None):
    return ops.flash_attention(Q, K, V, causal, sm_scale)
