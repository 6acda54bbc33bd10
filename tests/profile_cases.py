"""Small, fixed workloads for profiling one kernel at a time under ncu.

Each case calls one operator twice on seeded inputs (the first call warms the kernel up,
the second is the one to capture: ``ncu -k regex:<kernel> -s 1 -c 1``), keeps the device
footprint to a few GB and exits non-zero if the device status word reports a timeout.

    python tests/profile_cases.py attn        # attn_kernel: causal 2x32x4096x128 bf16
    python tests/profile_cases.py gemm_mn     # gemm_kernel: 4096^3 bf16, B row-major
    python tests/profile_cases.py gemm_k      # gemm_kernel: x[16384,4096] @ W[11008,4096]^T
    python tests/profile_cases.py layernorm   # row_reg_kernel: LayerNorm 16384x4096 bf16 (full size)

These are the workloads behind the summaries in profiles/; they are test-side recipes, not
part of the library.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
from autokernel_b200 import _lib, ops  # noqa: E402


def _attn():
    g = torch.Generator(device="cuda").manual_seed(0)
    q, k, v = (torch.randn(2, 32, 4096, 128, device="cuda", generator=g, dtype=torch.bfloat16)
               for _ in range(3))
    return lambda: ops.flash_attention(q, k, v, causal=True)


def _gemm_mn():
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(4096, 4096, device="cuda", generator=g, dtype=torch.bfloat16) / 64
    b = torch.randn(4096, 4096, device="cuda", generator=g, dtype=torch.bfloat16)
    return lambda: ops.matmul(a, b)


def _gemm_k():
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(16384, 4096, device="cuda", generator=g, dtype=torch.bfloat16)
    w = torch.randn(11008, 4096, device="cuda", generator=g, dtype=torch.bfloat16) * 0.02
    return lambda: ops.linear(x, w)


def _layernorm():
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(16384, 4096, device="cuda", generator=g, dtype=torch.bfloat16)
    w = 1 + 0.1 * torch.randn(4096, device="cuda", generator=g, dtype=torch.bfloat16)
    b = 0.1 * torch.randn(4096, device="cuda", generator=g, dtype=torch.bfloat16)
    return lambda: ops.layernorm(x, w, b)


CASES = {"attn": _attn, "gemm_mn": _gemm_mn, "gemm_k": _gemm_k, "layernorm": _layernorm}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("case", choices=sorted(CASES))
    a = ap.parse_args(argv)
    fn = CASES[a.case]()
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    st = _lib.device_status()
    print(f"{a.case}: device status {st}")
    return 0 if st == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
