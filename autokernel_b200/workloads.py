"""BASELINE configurations of the nine operators: synthetic inputs and algorithmic work.

Inputs are seeded and generated on the device for the benchmark (torch RNG, not
timed).  The algorithmic byte / FLOP counts are the per-call figures the
roofline uses: for memory-bound operators every input read once plus every
output written once; for contractions 2*M*N*K (causal attention counts only
the unmasked half: 2*B*H*D*S*(S+1)).
"""
from __future__ import annotations

import math

import torch


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def rope_table(S: int, half: int, theta: float = 10000.0, device="cuda",
               dtype=torch.bfloat16):
    """cos/sin [S, half] of angle pos * theta^(-2i/(2*half)), positions 0..S-1."""
    inv = 1.0 / theta ** (torch.arange(0, 2 * half, 2, device=device, dtype=torch.float32) / (2 * half))
    ang = torch.outer(torch.arange(S, device=device, dtype=torch.float32), inv)
    return ang.cos().to(dtype), ang.sin().to(dtype)


# ---------------------------------------------------------------- memory-bound sweep

SWEEP = {
    "softmax": {"rows": 8192, "cols": 32768},
    "layernorm": {"rows": 16384, "cols": 4096},
    "rope": {"B": 8, "H": 32, "S": 4096, "D": 128},
    "reduce": {"n": 1 << 30},
}


def sweep_inputs(device, seed: int = 0, scale: float = 1.0) -> dict:
    """softmax x~N(0, sd 2) [8192, 32768]; LayerNorm x~N(0,1) [16384, 4096] with
    w = 1 + 0.1N, b = 0.1N, eps 1e-5; RoPE q, k ~N(0,1) [8, 32, 4096, 128] with theta 10000;
    reduce x~U(-1,1) fp32 [2^30].  bf16 except reduce.  `scale` < 1 shrinks the leading dims
    (used for small profiling captures)."""
    g = _gen(device, seed)
    bf = torch.bfloat16
    s, l, r, rd = SWEEP["softmax"], SWEEP["layernorm"], SWEEP["rope"], SWEEP["reduce"]
    sr = max(1, int(s["rows"] * scale))
    lr = max(1, int(l["rows"] * scale))
    rb = max(1, int(r["B"] * scale))
    n = max(1024, int(rd["n"] * scale))
    d = {
        "sm_x": (torch.randn(sr, s["cols"], device=device, generator=g) * 2.0).to(bf),
        "ln_x": torch.randn(lr, l["cols"], device=device, generator=g).to(bf),
        "ln_w": (1 + 0.1 * torch.randn(l["cols"], device=device, generator=g)).to(bf),
        "ln_b": (0.1 * torch.randn(l["cols"], device=device, generator=g)).to(bf),
        "q": torch.randn(rb, r["H"], r["S"], r["D"], device=device, generator=g).to(bf),
        "k": torch.randn(rb, r["H"], r["S"], r["D"], device=device, generator=g).to(bf),
        "red_x": torch.rand(n, device=device, generator=g) * 2 - 1,
    }
    d["cos"], d["sin"] = rope_table(r["S"], r["D"] // 2, device=device)
    return d


def sweep_bytes(d: dict) -> dict:
    """Algorithmic bytes per call of each sweep kernel (read inputs once, write outputs once)."""
    e = lambda t: t.numel() * t.element_size()  # noqa: E731
    return {
        "softmax": 2 * e(d["sm_x"]),
        "layernorm": 2 * e(d["ln_x"]) + e(d["ln_w"]) + e(d["ln_b"]),
        "rope": 2 * (2 * e(d["q"])) + e(d["cos"]) + e(d["sin"]),  # q and k, read + write
        "reduce": e(d["red_x"]),
    }


# ---------------------------------------------------------------- contraction configs

GEMM_SHAPES = [(4096, 4096, 4096), (8192, 8192, 8192), (16384, 16384, 16384),
               (16384, 4096, 4096), (16384, 11008, 4096), (16384, 4096, 11008)]  # (M, N, K)
ATTN = {"B": 8, "H": 32, "S": 4096, "D": 128}
MLP = {"M": 16384, "D": 4096, "H": 11008}
XENT = {"rows": 65536 // 8, "vocab": 32000}   # per GPU at 8 GPUs (e2e LM head shard)
RMS = {"M": 4096, "N": 4096}


def gemm_inputs(M, N, K, device, seed=0, dtype=torch.bfloat16):
    g = _gen(device, seed)
    A = (torch.randn(M, K, device=device, generator=g) / math.sqrt(K)).to(dtype)
    B = (torch.randn(K, N, device=device, generator=g) / math.sqrt(K)).to(dtype)
    return A, B


def attn_flops(B, H, S, D, causal=True) -> float:
    return 2.0 * B * H * D * S * (S + 1) if causal else 4.0 * B * H * S * S * D
