"""Drop-in `fused_mlp` module for AutoKernel's kernel.py slot (replaces kernels/fused_mlp.py:102).

Copy or import as ``kernel.py``: AutoKernel's bench.py reads KERNEL_TYPE and
calls kernel_fn(**inputs); verify.py calls kernel_fn positionally.
"""
from autokernel_b200 import ops

KERNEL_TYPE = "fused_mlp"


def kernel_fn(x, w_gate, w_up, w_down, activation="silu"):
    return ops.fused_mlp(x, w_gate, w_up, w_down, activation)
