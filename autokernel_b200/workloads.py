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


SWEEP_BLOCKS = 8  # configs[1] is cut into 8 equal blocks along its sharded (row / batch) dim


def sweep_inputs(device, blocks=range(SWEEP_BLOCKS), seed: int = 0, scale: float = 1.0) -> dict:
    """softmax x~N(0, sd 2) [8192, 32768]; LayerNorm x~N(0,1) [16384, 4096] with
    w = 1 + 0.1N, b = 0.1N, eps 1e-5; RoPE q, k ~N(0,1) [8, 32, 4096, 128] with theta 10000;
    reduce x~U(-1,1) fp32 [2^30].  bf16 except reduce.

    The full configuration is SWEEP_BLOCKS blocks of rows (softmax 1024 rows, LayerNorm 2048
    rows, RoPE one batch entry, reduce 2^27 elements); block b is drawn from its own generator
    seeded with seed + b, so a rank that owns blocks [b0, b1) holds exactly rows [b0, b1) of
    the one global tensor whatever the number of GPUs.  Blocks past SWEEP_BLOCKS continue the
    same sequence (a weak-scaled run gives rank r the blocks [8r, 8r + 8)).  `scale` < 1
    shrinks every block (small profiling captures only)."""
    blocks = list(blocks)
    nb = len(blocks)
    bf = torch.bfloat16
    s, l, r, rd = SWEEP["softmax"], SWEEP["layernorm"], SWEEP["rope"], SWEEP["reduce"]
    per = lambda n: max(1, int(n // SWEEP_BLOCKS * scale))  # noqa: E731
    sr, lr, rb, n = per(s["rows"]), per(l["rows"]), per(r["B"]), max(1024, per(rd["n"]))
    d = {
        "sm_x": torch.empty(nb * sr, s["cols"], device=device, dtype=bf),
        "ln_x": torch.empty(nb * lr, l["cols"], device=device, dtype=bf),
        "q": torch.empty(nb * rb, r["H"], r["S"], r["D"], device=device, dtype=bf),
        "k": torch.empty(nb * rb, r["H"], r["S"], r["D"], device=device, dtype=bf),
        "red_x": torch.empty(nb * n, device=device, dtype=torch.float32),
    }
    for i, b in enumerate(blocks):
        g = _gen(device, seed + b)
        d["sm_x"][i * sr:(i + 1) * sr] = torch.randn(sr, s["cols"], device=device, generator=g) * 2.0
        d["ln_x"][i * lr:(i + 1) * lr] = torch.randn(lr, l["cols"], device=device, generator=g)
        d["q"][i * rb:(i + 1) * rb] = torch.randn(rb, r["H"], r["S"], r["D"], device=device, generator=g)
        d["k"][i * rb:(i + 1) * rb] = torch.randn(rb, r["H"], r["S"], r["D"], device=device, generator=g)
        d["red_x"][i * n:(i + 1) * n] = torch.rand(n, device=device, generator=g) * 2 - 1
    g = _gen(device, seed + 1_000_003)  # parameters shared by every block
    d["ln_w"] = (1 + 0.1 * torch.randn(l["cols"], device=device, generator=g)).to(bf)
    d["ln_b"] = (0.1 * torch.randn(l["cols"], device=device, generator=g)).to(bf)
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
