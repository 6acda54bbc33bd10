"""Pin the CPU oracles to the reference: every golden case in tests/golden/ was produced
by AutoKernel's reference.py (tests/golden/make_golden.py).

* oracle.ref_torch (the reference's CPU path, timed as the CPU baseline) must reproduce the
  reference's native-dtype outputs exactly.
* oracle.ref_f64 (the float64 precision oracle the GPU kernels are checked against) must
  agree with the reference evaluated on float32 copies of the inputs to float32 accuracy.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import ref_f64, ref_torch

OPS = ["rmsnorm", "layernorm", "softmax", "rotary_embedding", "reduce", "cross_entropy",
       "matmul", "fused_mlp", "flash_attention"]


def _f64_call(op, ins, kw):
    a = {k: (v.double().numpy() if v.is_floating_point() else v.numpy()) for k, v in ins.items()}
    if op == "rmsnorm":
        return ref_f64.rmsnorm(a["x"], a["weight"], kw.get("eps", 1e-6))
    if op == "layernorm":
        return ref_f64.layernorm(a["x"], a["weight"], a["bias"], kw.get("eps", 1e-5))
    if op == "softmax":
        return ref_f64.softmax(a["x"])
    if op == "rotary_embedding":
        return ref_f64.rotary_embedding(a["x"], a["cos"], a["sin"])
    if op == "reduce":
        return ref_f64.reduce_sum(a["x"], kw.get("dim", -1))
    if op == "cross_entropy":
        return ref_f64.cross_entropy(a["logits"], a["targets"])
    if op == "matmul":
        return ref_f64.matmul(a["A"], a["B"])
    if op == "fused_mlp":
        return ref_f64.fused_mlp(a["x"], a["w_gate"], a["w_up"], a["w_down"], kw.get("activation", "silu"))
    if op == "flash_attention":
        return ref_f64.attention(a["Q"], a["K"], a["V"], kw.get("causal", True))
    raise KeyError(op)


def _torch_call(op, ins, kw):
    f = ref_torch.OPS[op]
    if op == "rmsnorm":
        return f(ins["x"], ins["weight"], **kw)
    if op == "layernorm":
        return f(ins["x"], ins["weight"], ins["bias"], **kw)
    if op == "softmax":
        return f(ins["x"])
    if op == "rotary_embedding":
        return f(ins["x"], ins["cos"], ins["sin"])
    if op == "reduce":
        return f(ins["x"], **kw)
    if op == "cross_entropy":
        return f(ins["logits"], ins["targets"])
    if op == "matmul":
        return f(ins["A"], ins["B"])
    if op == "fused_mlp":
        return f(ins["x"], ins["w_gate"], ins["w_up"], ins["w_down"], **kw)
    if op == "flash_attention":
        return f(ins["Q"], ins["K"], ins["V"], **kw)
    raise KeyError(op)


@pytest.mark.parametrize("op", OPS)
def test_torch_port_matches_reference_bitwise(op):
    for case in load_golden(op):
        got = _torch_call(op, case["inputs"], case["kwargs"])
        assert got.dtype == case["out"].dtype and got.shape == case["out"].shape, case["name"]
        assert torch.equal(got, case["out"]) or (
            torch.isnan(case["out"]).any() and torch.allclose(got, case["out"], equal_nan=True)), case["name"]


@pytest.mark.parametrize("op", OPS)
def test_f64_oracle_matches_reference_fp32(op):
    for case in load_golden(op):
        got = np.asarray(_f64_call(op, case["inputs"], case["kwargs"]))
        ref = case["out_f32"].double().numpy()
        assert got.shape == ref.shape, case["name"]
        finite = np.isfinite(ref)
        assert (np.isfinite(got) == finite).all(), case["name"]
        # fp32 evaluation of the reference vs exact: relative error ~1e-6 of the value scale
        scale = max(1.0, float(np.abs(ref[finite]).max()) if finite.any() else 1.0)
        tol = 2e-5 if op in ("flash_attention", "fused_mlp", "matmul") else 1e-5
        err = np.abs(got[finite] - ref[finite]).max() if finite.any() else 0.0
        assert err <= tol * scale, f"{case['name']}: max err {err:.3e}"


def test_llama_oracle_matches_reference_model():
    """oracle/llama_f64.py reproduces the reference LlamaModel's fp32 logits (golden fixture)."""
    from conftest import GOLDEN
    from oracle import llama_f64
    g = torch.load(GOLDEN / "llama_tiny.pt", weights_only=False)
    cfg = g["cfg"]
    sd = {k: v.double().numpy() for k, v in g["state_dict"].items()}
    got = llama_f64.forward(sd, g["tokens"].numpy(), cfg["n_heads"], cfg["n_kv_heads"])
    ref = g["logits"].double().numpy()
    assert np.abs(got - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max())
