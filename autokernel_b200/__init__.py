"""autokernel_b200: B200-native (sm_100a) implementation of AutoKernel's nine-operator
kernel_fn contract (rmsnorm, layernorm, softmax, rotary_embedding, reduce,
cross_entropy, matmul, fused_mlp, flash_attention) on hand-written CUDA kernels.

`autokernel_b200.ops` holds the operators with the reference signatures,
`autokernel_b200.kernels.<op>` the drop-in KERNEL_TYPE/kernel_fn modules and
`autokernel_b200.shard` the row/batch sharding over several GPUs.
"""
from . import ops  # noqa: F401
from ._lib import AkError, load  # noqa: F401

__version__ = "0.1.0"
