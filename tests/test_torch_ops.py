"""The dispatcher op set (autokernel_b200.torch_ops): schemas and fake (shape / dtype) rules
checked on CPU against the reference formulas (oracle/ref_torch.py restates reference.py);
on a GPU, the registered ops return exactly what autokernel_b200.ops returns, pass
torch.library.opcheck, and trace whole under torch.compile."""
from __future__ import annotations

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import autokernel_b200.torch_ops  # noqa: F401  (registers torch.ops.autokernel_b200.*)
from autokernel_b200 import ops
from oracle import ref_torch

AK = torch.ops.autokernel_b200


def _cases(device="cpu", dt=torch.bfloat16):
    g = torch.Generator().manual_seed(0)

    def r(*s, dtype=dt):
        return torch.randn(*s, generator=g).to(dtype).to(device)
    x = r(3, 5, 64)
    cos, sin = r(5, 32, dtype=torch.float32), r(5, 32, dtype=torch.float32)
    q = r(2, 3, 40, 64)
    return {
        "rmsnorm": ((x, r(64)), ref_torch.rmsnorm),
        "layernorm": ((x, r(64), r(64)), ref_torch.layernorm),
        "softmax": ((x,), ref_torch.softmax),
        "rotary_embedding": ((r(2, 3, 5, 64), cos, sin), ref_torch.rotary_embedding),
        "reduce": ((r(3, 7, 5), 1), ref_torch.reduce_sum),
        "reduce_1d": ((r(100),), ref_torch.reduce_sum),
        "cross_entropy": ((r(6, 50), torch.randint(0, 50, (6,), generator=g).to(device)),
                          ref_torch.cross_entropy),
        "matmul": ((r(4, 6, 32), r(32, 16)), ref_torch.matmul),
        "fused_mlp": ((r(7, 32), r(48, 32), r(48, 32), r(32, 48)), ref_torch.fused_mlp),
        "flash_attention": ((q, q, q), ref_torch.attention),
    }


def _op(name):
    return getattr(AK, name.split("_1d")[0])


@pytest.mark.parametrize("name", list(_cases()))
def test_fake_shapes_match_reference(name):
    args, ref = _cases()[name]
    want = ref(*args)
    with FakeTensorMode() as mode:
        fargs = [mode.from_tensor(a) if isinstance(a, torch.Tensor) else a for a in args]
        got = _op(name)(*fargs)
    assert tuple(got.shape) == tuple(want.shape), (got.shape, want.shape)
    assert got.dtype == want.dtype, (got.dtype, want.dtype)


def test_schemas_follow_kernel_fn_signatures():
    for name, params in [("softmax", ["x"]), ("matmul", ["A", "B"]),
                         ("layernorm", ["x", "weight", "bias", "eps"]),
                         ("rmsnorm", ["x", "weight", "eps"]),
                         ("flash_attention", ["Q", "K", "V", "causal", "sm_scale"]),
                         ("fused_mlp", ["x", "w_gate", "w_up", "w_down", "activation"]),
                         ("cross_entropy", ["logits", "targets"]),
                         ("rotary_embedding", ["x", "cos", "sin"]), ("reduce", ["x", "dim"])]:
        schema = getattr(AK, name).default._schema
        assert [a.name for a in schema.arguments] == params, name


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(_cases()))
def test_registered_ops_equal_library_calls(name):
    args, _ = _cases("cuda")[name]
    got = _op(name)(*args)
    want = getattr(ops, name.split("_1d")[0])(*args)
    torch.cuda.synchronize()
    assert got.shape == want.shape and got.dtype == want.dtype
    assert torch.equal(got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["softmax", "layernorm", "matmul", "flash_attention", "reduce"])
def test_opcheck(name):
    args, _ = _cases("cuda")[name]
    torch.library.opcheck(_op(name), args, test_utils=("test_schema", "test_faketensor"))


@pytest.mark.gpu
def test_compiles_whole_graph():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(64, 128, generator=g).to(torch.bfloat16).cuda()
    w = torch.randn(128, 96, generator=g).to(torch.bfloat16).cuda()
    ln_w = torch.ones(96, dtype=torch.bfloat16, device="cuda")
    ln_b = torch.zeros(96, dtype=torch.bfloat16, device="cuda")

    def f(x):
        h = AK.matmul(x, w)
        h = AK.layernorm(h, ln_w, ln_b)
        return AK.softmax(h)

    eager = f(x)
    compiled = torch.compile(f, fullgraph=True, backend="eager")(x)
    torch.cuda.synchronize()
    assert torch.equal(eager, compiled)
