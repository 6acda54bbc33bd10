"""float64 restatement of AutoKernel's LLaMA forward -- TEST INFRASTRUCTURE ONLY.

Follows models/llama_7b.py: RMSNorm x * rsqrt(mean(x^2) + eps) * w (:22-30), rotary
embedding on interleaved (even, odd) pairs with angles t * theta^(-2i/d) (:33-48), causal
scaled-dot-product attention with key/value heads repeated n_rep times (:63-85), SwiGLU
feed-forward w2(silu(w1 x) * w3 x) (:88-98), residual blocks (:109-112), final norm and LM
head (:199-209).  Weights are the reference module's state_dict (numpy arrays).  Pinned to
the reference model itself by tests/test_oracle_pinned.py (tests/golden/llama_tiny.pt).
"""
from __future__ import annotations

import numpy as np

from . import ref_f64


def _rms(x, w, eps):
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * w


def forward(w: dict, tokens: np.ndarray, n_heads: int, n_kv_heads: int, eps: float = 1e-6,
            theta: float = 10000.0) -> np.ndarray:
    w = {k: np.asarray(v, dtype=np.float64) for k, v in w.items()}
    B, T = tokens.shape
    h = w["tok_embeddings.weight"][tokens]
    D = h.shape[-1]
    hd = D // n_heads
    rep = n_heads // n_kv_heads
    cos, sin = ref_f64.cos_sin_table(T, hd // 2, theta)
    cs, sn = cos[:, None, :], sin[:, None, :]
    n_layers = len({k.split(".")[1] for k in w if k.startswith("layers.")})
    for i in range(n_layers):
        p = f"layers.{i}."
        x = _rms(h, w[p + "attention_norm.weight"], eps)
        q = (x @ w[p + "attention.wq.weight"].T).reshape(B, T, n_heads, hd)
        k = (x @ w[p + "attention.wk.weight"].T).reshape(B, T, n_kv_heads, hd)
        v = (x @ w[p + "attention.wv.weight"].T).reshape(B, T, n_kv_heads, hd)
        q = ref_f64.rotary_embedding(q, cs, sn)
        k = ref_f64.rotary_embedding(k, cs, sn)
        q, k, v = (a.transpose(0, 2, 1, 3) for a in (q, k, v))
        k = np.repeat(k, rep, axis=1)
        v = np.repeat(v, rep, axis=1)
        o = ref_f64.attention(q, k, v, causal=True).transpose(0, 2, 1, 3).reshape(B, T, D)
        h = h + o @ w[p + "attention.wo.weight"].T
        x = _rms(h, w[p + "ffn_norm.weight"], eps)
        h = h + ref_f64.fused_mlp(x, w[p + "feed_forward.w1.weight"], w[p + "feed_forward.w3.weight"],
                                  w[p + "feed_forward.w2.weight"], "silu")
    h = _rms(h, w["norm.weight"], eps)
    return h @ w["output.weight"].T


def next_token_loss(logits: np.ndarray, tokens: np.ndarray) -> float:
    """Mean cross entropy of logits[:, t] against tokens[:, t + 1]."""
    V = logits.shape[-1]
    return float(ref_f64.cross_entropy(logits[:, :-1].reshape(-1, V), tokens[:, 1:].reshape(-1)))
