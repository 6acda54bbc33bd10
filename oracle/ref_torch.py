"""PyTorch-on-CPU restatement of the reference's oracle -- TEST INFRASTRUCTURE ONLY.

This is what AutoKernel's reference.py computes when its tensors live on the
CPU: the same ATen operators applied in the input dtype, with the same
intermediate roundings.  It exists for two jobs, both outside the product:
  * bench.py's cpu_baseline leg and `bench.py --impl reference`, which time
    the reference's PyTorch CPU path on the GPU box's host cores (the
    reference tree itself is not present there), and
  * tests/test_oracle_pinned.py, which checks it bit-for-bit against outputs
    produced by the real reference.py (tests/golden/).
The operator sequence of each function has to match the reference's to give
the same bits, so each one names the reference line it restates.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def matmul(A, B):
    """reference.py:10-12."""
    return A @ B


def softmax(x, dim: int = -1):
    """reference.py:15-17."""
    return torch.softmax(x, dim)


def layernorm(x, weight, bias, eps: float = 1e-5):
    """reference.py:20-23: layer norm over the last dim."""
    return F.layer_norm(x, (x.shape[-1],), weight, bias, eps)


def rmsnorm(x, weight, eps: float = 1e-6):
    """reference.py:26-29: x / sqrt(mean(x**2) + eps) * w, each step in x's dtype."""
    ms = x.pow(2).mean(-1, keepdim=True)
    return x.div(ms.add(eps).sqrt()).mul(weight)


def attention(Q, K, V, causal: bool = True, sm_scale=None):
    """reference.py:32-42: scores, -inf above the diagonal, softmax, @ V."""
    scale = Q.shape[-1] ** -0.5 if sm_scale is None else sm_scale
    s = (Q @ K.transpose(-2, -1)) * scale
    if causal:
        hide = torch.ones(Q.shape[-2], K.shape[-2], dtype=torch.bool, device=Q.device).triu(1)
        s = s.masked_fill(hide, float("-inf"))
    return torch.softmax(s, -1) @ V


def fused_mlp(x, w_gate, w_up, w_down, activation: str = "silu"):
    """reference.py:45-55."""
    g = x @ w_gate.T
    u = x @ w_up.T
    if activation == "silu":
        g = F.silu(g)
    elif activation == "gelu":
        g = F.gelu(g)
    elif activation == "relu2":
        g = F.relu(g).pow(2)
    return (g * u) @ w_down.T


def cross_entropy(logits, targets):
    """reference.py:58-60: mean over rows (ignore_index -100)."""
    return F.cross_entropy(logits.reshape(-1, logits.shape[-1]), targets.reshape(-1))


def rotary_embedding(x, cos, sin):
    """reference.py:63-69: rotate interleaved (even, odd) pairs."""
    ev, od = x[..., 0::2], x[..., 1::2]
    a = ev * cos - od * sin
    b = ev * sin + od * cos
    return torch.stack((a, b), dim=-1).flatten(-2)


def reduce_sum(x, dim: int = -1):
    """reference.py:72-74."""
    return x.sum(dim=dim)


OPS = {
    "matmul": matmul,
    "softmax": softmax,
    "layernorm": layernorm,
    "rmsnorm": rmsnorm,
    "flash_attention": attention,
    "fused_mlp": fused_mlp,
    "cross_entropy": cross_entropy,
    "rotary_embedding": rotary_embedding,
    "reduce": reduce_sum,
}
