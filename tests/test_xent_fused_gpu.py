"""LM head fused with cross entropy (ak_linear_cross_entropy_rows): the per-row losses of the
logits x @ W^T without storing them, against the float64 oracle on the logits rounded to the
dtype (what the LM head of models/llama_7b.py stores before reference.py:58-60 reads them),
and the exact fields -- row max and target logit -- bitwise against the unfused path
(ops.linear then ops.cross_entropy_rows)."""
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


def _inputs(n, dim, vocab, dt, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(n, dim, device=DEV, generator=g).to(DTS[dt])
    w = (torch.randn(vocab, dim, device=DEV, generator=g) * 0.02).to(DTS[dt])
    t = torch.randint(0, vocab, (n,), device=DEV, generator=g)
    t[::7] = -100  # ignored rows
    t[1] = vocab - 1
    t[2] = 0
    return x, w, t


def _close(loss, e, name, tol=2e-3):
    """Per-row losses (fp32) against the f64 oracle: the logits are 16-bit, so a logit that the
    fp32 accumulation rounds to the other neighbour moves a loss by up to ~1 logit ulp."""
    got = to_np(loss)
    err = np.abs(got - e)
    assert (err <= tol * (1 + np.abs(e))).all(), f"{name}: max err {err.max():.3e}"


def _oracle_rows(x, w, t, dtype):
    """float64 cross entropy of the float64 logits rounded to the dtype."""
    z = torch.from_numpy(to_np(x) @ to_np(w).T).to(dtype).double().numpy()
    return ref_f64.cross_entropy_rows(z, t.cpu().numpy())


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("n,dim,vocab", [(300, 256, 1000), (1024, 512, 32000), (129, 64, 50257),
                                         (4096, 4096, 32000)])
def test_linear_cross_entropy_matches_oracle_and_unfused(dt, n, dim, vocab):
    x, w, t = _inputs(n, dim, vocab, dt, n + vocab)
    loss, tt, mx, tl = ops().linear_cross_entropy_rows(x, w, t, with_stats=True)
    loss_u, _, mx_u, tl_u = ops().cross_entropy_rows(ops().linear(x, w), t, with_stats=True)
    torch.cuda.synchronize()
    # exact fields: bitwise the unfused LM head + loss
    keep = t != -100
    assert torch.equal(mx, mx_u)
    assert torch.equal(tl[keep], tl_u[keep])
    # losses within tolerance of the f64 oracle and of the unfused path
    e_loss, e_max, _, e_keep = _oracle_rows(x, w, t, DTS[dt])
    _close(loss, np.where(e_keep, e_loss, 0.0), f"{n}x{dim}x{vocab}")
    check(loss, to_np(loss_u), "cross_entropy", "vs unfused")
    # the mean, through the finalize kernel
    m = ops().linear_cross_entropy(x, w, t)
    assert m.dtype == x.dtype and m.dim() == 0
    e_mean = e_loss[e_keep].sum() / e_keep.sum()
    assert abs(float(m.float()) - e_mean) <= 1e-2 * (1 + abs(e_mean))


def test_linear_cross_entropy_llama_head_sampled_rows():
    """The LLaMA LM head at one GPU micro-batch: [16384, 4096] x [32000, 4096] fp16, checked on
    one seeded row of every 128-row tile."""
    n, dim, vocab = 16384, 4096, 32000
    x, w, t = _inputs(n, dim, vocab, "f16", 3)
    loss, _, mx, tl = ops().linear_cross_entropy_rows(x, w, t, with_stats=True)
    torch.cuda.synchronize()
    rng = np.random.default_rng(0)
    rows = np.arange(0, n, 128) + rng.integers(0, 128, n // 128)
    ri = torch.as_tensor(rows, device=DEV)
    e_loss, e_max, e_tl, e_keep = _oracle_rows(x[ri], w, t[ri], torch.float16)
    _close(loss[ri], np.where(e_keep, e_loss, 0.0), "llama head sampled")
    assert np.abs(to_np(mx[ri]) - e_max).max() < 1e-2


def test_linear_cross_entropy_fp32_uses_unfused_kernels():
    x, w, t = _inputs(200, 128, 3000, "bf16", 9)
    x, w = x.float(), w.float()
    loss, _ = ops().linear_cross_entropy_rows(x, w, t)
    e_loss, _, _, e_keep = _oracle_rows(x, w, t, torch.float32)
    _close(loss, np.where(e_keep, e_loss, 0.0), "fp32", tol=1e-5)


def test_linear_cross_entropy_bad_target_and_determinism():
    x, w, t = _inputs(256, 256, 1000, "bf16", 5)
    a = ops().linear_cross_entropy_rows(x, w, t)[0]
    b = ops().linear_cross_entropy_rows(x, w, t)[0]
    assert torch.equal(a, b)
    t2 = t.clone()
    t2[3] = 1000  # out of range, not ignore_index
    loss, _ = ops().linear_cross_entropy_rows(x, w, t2)
    torch.cuda.synchronize()
    assert torch.isnan(loss[3]) and torch.isfinite(loss[4])
    from autokernel_b200 import _lib
    assert _lib.device_status() == 0
