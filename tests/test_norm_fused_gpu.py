"""RMSNorm folded into the projections that read it (ak_row_sumsq, ak_linear_rms,
ak_mlp_gate_up_rms): RMSNorm(x) @ W^T computed as (x @ (W diag(w_norm))^T) scaled per row by
1 / rms, against the float64 oracle of the unfused norm + projection (models/llama_7b.py:22-30
then the q/k/v or feed-forward projections), and the sums of squares a residual GEMM writes
for the next norm."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import ref_f64
from parity import check, to_np

pytestmark = pytest.mark.gpu

DEV = "cuda"
DTS = {"f16": torch.float16, "bf16": torch.bfloat16}


def ops():
    from autokernel_b200 import ops as _ops
    return _ops


def _r(shape, seed, scale=1.0, dt="bf16"):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*shape, device=DEV, generator=g) * scale).to(DTS[dt])


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("M,K,N", [(300, 512, 384), (4096, 4096, 4096), (129, 4096, 11008)])
def test_linear_rms_matches_norm_then_projection(dt, M, K, N):
    x = _r((M, K), 1, 1.0, dt)
    wn = (1 + 0.1 * _r((K,), 2, 1.0, "bf16").float()).to(DTS[dt])
    W = _r((N, K), 3, 0.02, dt)
    ss = ops().row_sumsq(x)
    assert ss.shape == ((K + 255) // 256, M)
    np.testing.assert_allclose(to_np(ss).sum(0), (to_np(x) ** 2).sum(1), rtol=1e-5)
    Wf = ops().fold_norm_weight(W, wn)
    y = ops().linear_rms(x, Wf, ss, 1e-6)
    # the kernel's arithmetic: the unweighted norm of x times the folded (once-rounded) weight
    ones = np.ones(K)
    check(y, ref_f64.rmsnorm(to_np(x), ones, 1e-6) @ to_np(Wf).T, "matmul",
          f"linear_rms {M}x{K}x{N}")
    # and the unfused math: folding rounds each weight once, as the unfused path rounds each
    # normalised activation once, so it sits within twice the tolerance
    e = ref_f64.rmsnorm(to_np(x), to_np(wn), 1e-6) @ to_np(W).T
    check(y, e, "matmul", f"linear_rms {M}x{K}x{N} vs unfused math", scale_tol=2.0)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_residual_gemm_writes_next_norm_sums(dt):
    """h += o @ Wo^T in place, with the sums of squares of the new h for the next norm."""
    M, K, N = 1000, 1024, 2048
    o = _r((M, K), 4, 1.0, dt)
    Wo = _r((N, K), 5, 0.02, dt)
    h = _r((M, N), 6, 1.0, dt)
    h_ref = to_np(h) + to_np(o) @ to_np(Wo).T
    _, ss = ops().linear_rms(o, Wo, residual=h, out=h, want_ss=True)
    torch.cuda.synchronize()
    check(h, h_ref, "matmul", "residual")
    np.testing.assert_allclose(to_np(ss).sum(0), (to_np(h) ** 2).sum(1), rtol=1e-4)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_mlp_hidden_rms(dt):
    M, D, H = 512, 1024, 2816
    x = _r((M, D), 7, 1.0, dt)
    wn = (1 + 0.1 * _r((D,), 8, 1.0, "bf16").float()).to(DTS[dt])
    wg, wu = _r((H, D), 9, 0.02, dt), _r((H, D), 10, 0.02, dt)
    hid = ops().mlp_hidden_rms(x, ops().fold_norm_weight(wg, wn), ops().fold_norm_weight(wu, wn),
                               ops().row_sumsq(x), 1e-6)
    xn = ref_f64.rmsnorm(to_np(x), to_np(wn), 1e-6)
    check(hid, ref_f64.mlp_hidden(xn, to_np(wg), to_np(wu)), "fused_mlp", "mlp_hidden_rms")


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_linear_rms_with_rope_epilogue(dt):
    """q = RoPE(RMSNorm(h) @ Wq^T) in one GEMM: against the f64 oracle of the norm, projection
    and interleaved rotation (models/llama_7b.py:40-48), position = row % T."""
    B, T, D, hd = 2, 256, 512, 128
    h = _r((B, T, D), 11, 1.0, dt)
    wn = (1 + 0.1 * _r((D,), 12, 1.0, "bf16").float()).to(DTS[dt])
    Wq = _r((D, D), 13, 0.05, dt)
    c, s = ref_f64.cos_sin_table(T, hd // 2)
    ct, st = torch.tensor(c, dtype=torch.float32, device=DEV), torch.tensor(s, dtype=torch.float32, device=DEV)
    Wf = ops().fold_norm_weight(Wq, wn)
    q = ops().linear_rms(h, Wf, ops().row_sumsq(h), 1e-6, rope=(ct, st, T, hd))
    proj = (ref_f64.rmsnorm(to_np(h), np.ones(D), 1e-6) @ to_np(Wf).T).reshape(B, T, D // hd, hd)
    e = ref_f64.rotary_embedding(proj, c[:, None, :], s[:, None, :]).reshape(B, T, D)
    check(q, e, "matmul", "linear_rms + rope")
