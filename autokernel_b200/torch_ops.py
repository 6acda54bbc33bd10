"""The nine operators as a PyTorch dispatcher op set: ``torch.ops.autokernel_b200.<op>``.

AutoKernel exports an optimized kernel to the Hugging Face kernels layout as a TORCH_LIBRARY
op set (export_hf.py:367-420; examples/hf_kernels_test/torch-ext/torch_binding.cpp:6-9:
``ops.def("matmul_cuda(Tensor A, Tensor B) -> Tensor")`` + a CUDA ``impl``).  Here the same
registration is made through ``torch.library`` from Python: each op gets a schema, a CUDA
implementation that calls the C ABI (libak_b200.so, through ``autokernel_b200.ops``), and a
fake (shape / dtype) implementation, so the ops can be traced by torch.compile / export
without running.  The C ABI stays free of torch types; this module is the only place the
kernels meet the dispatcher.

    import autokernel_b200.torch_ops            # registers the op set once
    y = torch.ops.autokernel_b200.softmax(x)

Schemas follow the reference's ``kernel_fn`` signatures (kernels/<op>.py), with defaults.
"""
from __future__ import annotations

import torch

from . import ops as _ops

NAMESPACE = "autokernel_b200"
_lib = torch.library.Library(NAMESPACE, "DEF")

_SCHEMAS = {
    "rmsnorm": "rmsnorm(Tensor x, Tensor weight, float eps=1e-06) -> Tensor",
    "layernorm": "layernorm(Tensor x, Tensor weight, Tensor bias, float eps=1e-05) -> Tensor",
    "softmax": "softmax(Tensor x) -> Tensor",
    "rotary_embedding": "rotary_embedding(Tensor x, Tensor cos, Tensor sin) -> Tensor",
    "reduce": "reduce(Tensor x, int dim=-1) -> Tensor",
    "cross_entropy": "cross_entropy(Tensor logits, Tensor targets) -> Tensor",
    "matmul": "matmul(Tensor A, Tensor B) -> Tensor",
    "fused_mlp": ("fused_mlp(Tensor x, Tensor w_gate, Tensor w_up, Tensor w_down, "
                  "str activation='silu') -> Tensor"),
    "flash_attention": ("flash_attention(Tensor Q, Tensor K, Tensor V, bool causal=True, "
                        "float? sm_scale=None) -> Tensor"),
}


def _fake_rows(x, *_, **__):
    return x.new_empty(x.shape)


def _fake_rope(x, cos, sin):
    dt = torch.promote_types(x.dtype, torch.promote_types(cos.dtype, sin.dtype))
    return x.new_empty(x.shape, dtype=dt)


def _fake_reduce(x, dim=-1):
    if x.dim() == 0:
        return x.new_empty(())
    d = dim % x.dim()
    return x.new_empty(x.shape[:d] + x.shape[d + 1:])


def _fake_cross_entropy(logits, targets):
    return logits.new_empty(())


def _fake_matmul(A, B):
    if A.dim() == 1:
        return A.new_empty((B.shape[1],))
    return A.new_empty((*A.shape[:-1], B.shape[1]))


def _fake_fused_mlp(x, w_gate, w_up, w_down, activation="silu"):
    return x.new_empty((*x.shape[:-1], w_down.shape[0]))


def _fake_attention(Q, K, V, causal=True, sm_scale=None):
    lead = torch.broadcast_shapes(Q.shape[:-2], K.shape[:-2], V.shape[:-2])
    return Q.new_empty((*lead, Q.shape[-2], Q.shape[-1]))


_IMPLS = {
    "rmsnorm": (_ops.rmsnorm, _fake_rows),
    "layernorm": (_ops.layernorm, _fake_rows),
    "softmax": (_ops.softmax, _fake_rows),
    "rotary_embedding": (_ops.rotary_embedding, _fake_rope),
    "reduce": (_ops.reduce, _fake_reduce),
    "cross_entropy": (_ops.cross_entropy, _fake_cross_entropy),
    "matmul": (_ops.matmul, _fake_matmul),
    "fused_mlp": (_ops.fused_mlp, _fake_fused_mlp),
    "flash_attention": (_ops.flash_attention, _fake_attention),
}

for _name, _schema in _SCHEMAS.items():
    _lib.define(_schema)
    _cuda, _fake = _IMPLS[_name]
    _lib.impl(_name, _cuda, "CUDA")
    torch.library.register_fake(f"{NAMESPACE}::{_name}", _fake, lib=_lib)


def op(name: str):
    """The registered overload packet ``torch.ops.autokernel_b200.<name>``."""
    return getattr(getattr(torch.ops, NAMESPACE), name)


__all__ = ["NAMESPACE", "op"]
