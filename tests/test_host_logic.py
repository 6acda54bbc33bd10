"""Host-side logic of autokernel_b200.ops that needs no GPU: broadcast decoding, operand
layout selection, and the no-CPU-fallback rule."""
from __future__ import annotations

import pytest
import torch

from autokernel_b200 import ops


@pytest.mark.parametrize("lead,cshape,expect", [
    ((2, 8, 64), (64, 32), (1, 64)),            # bench: x [B,H,S,D], cos [S,D/2]
    ((2, 64, 8), (64, 1, 32), (8, 64)),         # model: x [B,S,H,D], cos [S,1,D/2]
    ((2, 8, 64), (2, 8, 64, 32), (1, 1024)),    # full-size cos
    ((2, 8, 64), (32,), (1, 1)),                # one row for all
    ((2, 8, 64), (2, 1, 64, 32), None),         # non-contiguous broadcast block
    ((2, 8, 64), (8, 1, 32), (64, 8)),          # per-head
])
def test_rope_broadcast(lead, cshape, expect):
    got = ops._rope_broadcast(lead, torch.empty(cshape))
    assert got == expect


def _rows_for(lead, cshape):
    """Row r -> cos row via the (div, rows) rule, vs torch broadcasting of indices."""
    bc = ops._rope_broadcast(lead, torch.empty(cshape))
    cs_lead = cshape[:-1]
    idx = torch.arange(int(torch.tensor(cs_lead).prod()) if cs_lead else 1).reshape(cs_lead or (1,))
    want = idx.expand(*lead).reshape(-1) if cs_lead else torch.zeros(int(torch.tensor(lead).prod()), dtype=torch.long)
    r = torch.arange(want.numel())
    return (r // bc[0]) % bc[1], want


@pytest.mark.parametrize("lead,cshape", [((2, 8, 64), (64, 32)), ((2, 64, 8), (64, 1, 32)),
                                         ((3, 5, 7), (5, 1, 4)), ((3, 5, 7), (3, 5, 7, 4))])
def test_rope_broadcast_index_rule(lead, cshape):
    got, want = _rows_for(lead, cshape)
    assert torch.equal(got, want)


def test_b_operand_layouts():
    B = torch.empty(64, 32)
    t, ld, kmaj = ops._b_operand(B)
    assert (ld, kmaj) == (32, 0)
    W = torch.empty(32, 64)          # nn.Linear weight [N, K]; W.t() is [K, N]
    t, ld, kmaj = ops._b_operand(W.t())
    assert (ld, kmaj) == (64, 1) and t.data_ptr() == W.data_ptr()


@pytest.mark.parametrize("name", list(ops.OPS))
def test_cpu_tensors_are_rejected(name):
    x = torch.randn(4, 8)
    args = {
        "matmul": (x, torch.randn(8, 4)), "softmax": (x,), "layernorm": (x, torch.ones(8), torch.zeros(8)),
        "rmsnorm": (x, torch.ones(8)), "flash_attention": (x[None, None], x[None, None], x[None, None]),
        "fused_mlp": (x, torch.randn(16, 8), torch.randn(16, 8), torch.randn(8, 16)),
        "cross_entropy": (x, torch.zeros(4, dtype=torch.long)), "rotary_embedding": (x, torch.ones(4, 4), torch.ones(4, 4)),
        "reduce": (x,),
    }[name]
    with pytest.raises(ValueError, match="CUDA"):
        ops.OPS[name](*args)


# kernel_fn signatures of the reference starters (kernels/<op>.py), which AutoKernel's bench.py
# calls with keyword arguments named after its input generators (bench.py:203-276)
REFERENCE_SIGNATURES = {
    "matmul": [("A", None), ("B", None)],
    "softmax": [("x", None)],
    "layernorm": [("x", None), ("weight", None), ("bias", None), ("eps", 1e-5)],
    "rmsnorm": [("x", None), ("weight", None), ("eps", 1e-6)],
    "flash_attention": [("Q", None), ("K", None), ("V", None), ("causal", True), ("sm_scale", None)],
    "fused_mlp": [("x", None), ("w_gate", None), ("w_up", None), ("w_down", None),
                  ("activation", "silu")],
    "cross_entropy": [("logits", None), ("targets", None)],
    "rotary_embedding": [("x", None), ("cos", None), ("sin", None)],
    "reduce": [("x", None), ("dim", -1)],
}


@pytest.mark.parametrize("name", list(REFERENCE_SIGNATURES))
def test_drop_in_kernel_fn_signature(name):
    import inspect

    from autokernel_b200 import kernels
    mod = kernels.get(name)
    assert mod.KERNEL_TYPE == name
    params = list(inspect.signature(mod.kernel_fn).parameters.values())
    got = [(p.name, None if p.default is inspect.Parameter.empty else p.default) for p in params]
    assert got == REFERENCE_SIGNATURES[name]
    # the ops-level function takes the same arguments
    op_params = list(inspect.signature(ops.OPS[name]).parameters)
    assert op_params == [n for n, _ in REFERENCE_SIGNATURES[name]]
