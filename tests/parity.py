"""Comparison rules shared by the GPU parity tests.

A GPU result y is accepted against the float64 oracle value e when, elementwise,

    |y - e| <= atol + rtol * |e| + q(e)

where (atol, rtol) is the operator's tolerance -- 1e-2 for GEMM / MLP /
attention and 1e-3 for norms, softmax and RoPE (fp32-accumulated), as the
BASELINE north star states, tightened to 1e-5 / 1e-4 for fp32 outputs as in the
reference's bench.py tables -- and q(e) is one quantum (ulp) of the output dtype
at |e|: a bf16 output carries a relative rounding step of 2^-8, which is larger
than a 1e-3 relative tolerance, so an exactly-rounded kernel could otherwise
fail by the rounding of its own output.  For fp32 outputs q is 0.
"""
from __future__ import annotations

import numpy as np
import torch

# (atol, rtol) per operator class and output dtype
TOL = {
    "gemm": {torch.float16: (1e-2, 1e-2), torch.bfloat16: (1e-2, 1e-2), torch.float32: (1e-4, 1e-4)},
    "norm": {torch.float16: (1e-3, 1e-3), torch.bfloat16: (1e-3, 1e-3), torch.float32: (1e-5, 1e-5)},
    "loss": {torch.float16: (1e-2, 1e-2), torch.bfloat16: (2e-2, 2e-2), torch.float32: (1e-5, 1e-5)},
    "sum": {torch.float16: (1e-2, 1e-2), torch.bfloat16: (5e-2, 5e-2), torch.float32: (1e-4, 1e-5)},
}
OP_CLASS = {
    "matmul": "gemm", "fused_mlp": "gemm", "flash_attention": "gemm",
    "rmsnorm": "norm", "layernorm": "norm", "softmax": "norm", "rotary_embedding": "norm",
    "cross_entropy": "loss", "reduce": "sum",
}
MANT_BITS = {torch.float16: 10, torch.bfloat16: 7, torch.float32: 23}


def quantum(e: np.ndarray, dtype: torch.dtype) -> np.ndarray:
    if dtype == torch.float32:
        return np.zeros_like(e)
    mb = MANT_BITS[dtype]
    a = np.maximum(np.abs(e), 2.0 ** -14 if dtype == torch.float16 else 2.0 ** -126)
    return 2.0 ** (np.floor(np.log2(a)) - mb)


def check(y: torch.Tensor, exact, op: str, name: str = "", scale_tol: float = 1.0,
          reduce_n: int | None = None) -> dict:
    """Assert y (GPU tensor) matches the float64 oracle `exact`; returns error stats.

    For sums the absolute tolerance grows with sqrt(n) of the summed elements
    (fp32 accumulation of n terms of unit scale), given by reduce_n."""
    atol, rtol = TOL[OP_CLASS[op]][y.dtype]
    atol, rtol = atol * scale_tol, rtol * scale_tol
    if reduce_n:
        atol = atol * max(1.0, np.sqrt(reduce_n) / 32)
    got = y.detach().float().cpu().double().numpy()
    e = np.asarray(exact, dtype=np.float64)
    assert got.shape == e.shape, f"{name}: shape {got.shape} vs {e.shape}"
    fin = np.isfinite(e)
    assert (np.isfinite(got) == fin).all(), f"{name}: non-finite mismatch"
    if np.isnan(e).any():
        assert (np.isnan(got) == np.isnan(e)).all(), f"{name}: NaN mismatch"
    err = np.abs(got[fin] - e[fin])
    bound = atol + rtol * np.abs(e[fin]) + quantum(e[fin], y.dtype)
    bad = err > bound
    stats = {"max_abs": float(err.max()) if err.size else 0.0,
             "frac_bad": float(bad.mean()) if err.size else 0.0}
    assert not bad.any(), (f"{name}: {int(bad.sum())}/{bad.size} elements out of tolerance, "
                           f"max abs err {stats['max_abs']:.3e} (atol {atol}, rtol {rtol})")
    return stats


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().double().numpy() if t.is_floating_point() else t.detach().cpu().numpy()
