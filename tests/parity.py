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


def check_like_reference(y: torch.Tensor, ref_native: torch.Tensor, exact, op: str,
                         name: str = "", max_ulps: float = 1.0, abs_floor: float = 0.0) -> None:
    """For kernels that follow reference.py's own per-operator rounding in 16-bit dtypes
    (RMSNorm, RoPE with tables in x's dtype, the SwiGLU hidden): y must be within `max_ulps`
    output quanta of reference.py's output on the same inputs (0: bit-identical) or, where
    given, within `abs_floor` of it, and within the operator's tolerance of the float64 value
    once the reference's own rounding error |ref_native - exact| is allowed for."""
    got = y.detach().float().cpu().double().numpy()
    r = ref_native.detach().float().double().numpy()
    assert got.shape == r.shape, f"{name}: shape {got.shape} vs {r.shape}"
    both_nan = np.isnan(got) & np.isnan(r)
    d = np.where(both_nan, 0.0, np.abs(got - r))
    lim = max_ulps * quantum(r, y.dtype) if y.dtype != torch.float32 else 1e-6 * (1 + np.abs(r))
    lim = np.maximum(lim, abs_floor)
    bad = ~(d <= lim)
    assert not bad.any(), (f"{name}: {int(bad.sum())}/{bad.size} elements more than {max_ulps} "
                           f"ulp from reference.py's output, max diff {np.nanmax(d):.3e}")
    e = np.asarray(exact, dtype=np.float64)
    atol, rtol = TOL[OP_CLASS[op]][y.dtype]
    fin = np.isfinite(e) & np.isfinite(r)
    bound = atol + rtol * np.abs(e[fin]) + quantum(e[fin], y.dtype) + np.abs(r[fin] - e[fin])
    err = np.abs(got[fin] - e[fin])
    assert (err <= bound).all(), (f"{name}: {int((err > bound).sum())} elements beyond the f64 "
                                  f"tolerance widened by the reference's own rounding")


def reference_mlp_hidden(x, w_gate, w_up, activation: str = "silu", dtype=torch.bfloat16):
    """reference.py's SwiGLU hidden (reference.py:45-55) on float64 projections: the gate and
    up projections stored in `dtype`, the activation applied to the stored gate and stored, the
    product stored -- the rounding points of the reference's own 16-bit path, without the
    rounding noise of any particular GEMM.  Returns a CPU tensor of `dtype`."""
    import torch.nn.functional as F
    xf = np.asarray(to_np(x) if isinstance(x, torch.Tensor) else x, dtype=np.float64)
    g = torch.from_numpy(xf @ to_np(w_gate).T).to(dtype)
    u = torch.from_numpy(xf @ to_np(w_up).T).to(dtype)
    if activation == "silu":
        g = F.silu(g)
    elif activation == "gelu":
        g = F.gelu(g)
    elif activation == "relu2":
        g = F.relu(g) ** 2
    return g * u
