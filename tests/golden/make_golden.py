"""Generate tests/golden/*.pt from the reference's own oracle (AutoKernel reference.py).

Run in a container that has the reference tree (read-only) at REF_DIR:

    python tests/golden/make_golden.py [REF_DIR]

For every case it stores the seeded inputs (CPU torch.Generator), the output of
reference.<op>_ref on those inputs in their own dtype ("out"), and on float32
copies ("out_f32").  The fixtures are small (a few hundred KB in total) and
are committed; the GPU box never needs the reference tree.
"""
from __future__ import annotations

import importlib.util
import math
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REF_DIR = Path(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")

spec = importlib.util.spec_from_file_location("ak_reference", REF_DIR / "reference.py")
ref = importlib.util.module_from_spec(spec)
spec.loader.exec_module(ref)

DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def gen(seed):
    g = torch.Generator().manual_seed(seed)
    return lambda *shape, scale=1.0: torch.randn(*shape, generator=g) * scale


def cos_sin(S, half, theta=10000.0):
    inv = 1.0 / theta ** (torch.arange(0, 2 * half, 2).float() / (2 * half))
    ang = torch.outer(torch.arange(S).float(), inv)
    return ang.cos(), ang.sin()


def cases():
    out = []
    # rmsnorm: bench sizes scaled down, an odd width, weights 1 + 0.1 N(0,1)
    for dt in ("f16", "bf16", "f32"):
        for (M, N) in ((16, 768), (7, 1023), (2, 4096)):
            r = gen(1)
            out.append(("rmsnorm", dt, f"{M}x{N}", {"x": r(M, N), "weight": 1 + 0.1 * r(N)}, {"eps": 1e-6}))
    for dt in ("f16", "bf16", "f32"):
        for (M, N) in ((16, 512), (3, 4097), (2, 4096)):
            r = gen(2)
            out.append(("layernorm", dt, f"{M}x{N}",
                        {"x": r(M, N), "weight": 1 + 0.1 * r(N), "bias": 0.1 * r(N)}, {"eps": 1e-5}))
    for dt in ("f16", "bf16", "f32"):
        for (M, N) in ((32, 128), (4, 1023)) + (((1, 50257), (1, 32768)) if dt == "bf16" else ()):
            r = gen(3)
            x = r(M, N, scale=2.0)
            out.append(("softmax", dt, f"{M}x{N}", {"x": x}, {}))
    # special rows: zeros, constant, huge magnitudes, -inf entries
    sp = torch.zeros(4, 256)
    sp[1] = 0.5
    sp[2] = gen(4)(256) * 1e4
    sp[3] = gen(5)(256)
    sp[3, ::3] = float("-inf")
    for dt in ("f16", "bf16", "f32"):
        out.append(("softmax", dt, "special", {"x": sp.clone()}, {}))
    for dt in ("f16", "bf16", "f32"):
        r = gen(6)
        c, s = cos_sin(64, 32)
        out.append(("rotary_embedding", dt, "1x2x64x64", {"x": r(1, 2, 64, 64), "cos": c, "sin": s}, {}))
        c, s = cos_sin(127, 32)
        out.append(("rotary_embedding", dt, "1x2x127x64", {"x": r(1, 2, 127, 64), "cos": c, "sin": s}, {}))
        c, s = cos_sin(16, 64)
        out.append(("rotary_embedding", dt, "bshd_1x16x4x128",
                    {"x": r(1, 16, 4, 128), "cos": c[:, None, :], "sin": s[:, None, :]}, {}))
        out.append(("rotary_embedding", dt, "randcs_2x3x10x16",
                    {"x": r(2, 3, 10, 16), "cos": r(10, 8), "sin": r(10, 8)}, {}))
    for dt in ("f16", "bf16", "f32"):
        r = gen(7)
        out.append(("reduce", dt, "16x1024", {"x": r(16, 1024)}, {"dim": -1}))
        out.append(("reduce", dt, "33x1023", {"x": r(33, 1023)}, {"dim": -1}))
        out.append(("reduce", dt, "8x300x5_dim1", {"x": r(8, 300, 5)}, {"dim": 1}))
        out.append(("reduce", dt, "flat_20011", {"x": torch.rand(20011, generator=torch.Generator().manual_seed(8)) * 2 - 1}, {"dim": -1}))
    for dt in ("f16", "bf16", "f32"):
        g = torch.Generator().manual_seed(9)
        for (N, V) in ((32, 256), (7, 1000)) + (((2, 32000), (1, 50257)) if dt == "f16" else ()):
            logits = torch.randn(N, V, generator=g)
            t = torch.randint(0, V, (N,), generator=g)
            if N == 7:
                t[2] = -100  # ignore_index row
            out.append(("cross_entropy", dt, f"{N}x{V}", {"logits": logits, "targets": t}, {}))
    for dt in ("f16", "bf16", "f32"):
        for (M, N, K) in ((64, 96, 128), (127, 33, 65), (128, 64, 256)):
            r = gen(10)
            out.append(("matmul", dt, f"{M}x{N}x{K}",
                        {"A": r(M, K, scale=1 / math.sqrt(K)), "B": r(K, N)}, {}))
    for dt in ("f16", "bf16", "f32"):
        for act in ("silu", "gelu", "relu2"):
            r = gen(11)
            out.append(("fused_mlp", dt, f"32x64x128_{act}",
                        {"x": r(32, 64), "w_gate": r(128, 64, scale=0.02),
                         "w_up": r(128, 64, scale=0.02), "w_down": r(64, 128, scale=0.02)},
                        {"activation": act}))
        r = gen(12)
        out.append(("fused_mlp", dt, "130x64x72_silu",
                    {"x": r(130, 64), "w_gate": r(72, 64, scale=0.05),
                     "w_up": r(72, 64, scale=0.05), "w_down": r(64, 72, scale=0.05)},
                    {"activation": "silu"}))
    for dt in ("f16", "bf16"):
        r = gen(13)
        for (B, H, S, D) in ((1, 2, 64, 64), (1, 1, 127, 64), (1, 1, 192, 128)):
            for causal in (True, False):
                out.append(("flash_attention", dt, f"{B}x{H}x{S}x{D}_{'c' if causal else 'nc'}",
                            {"Q": r(B, H, S, D), "K": r(B, H, S, D), "V": r(B, H, S, D)},
                            {"causal": causal}))
        out.append(("flash_attention", dt, "q64_k96_c",
                    {"Q": r(1, 1, 64, 64), "K": r(1, 1, 96, 64), "V": r(1, 1, 96, 64)}, {"causal": True}))
    return out


REF_FN = {
    "rmsnorm": lambda i, k: ref.rmsnorm_ref(i["x"], i["weight"], **k),
    "layernorm": lambda i, k: ref.layernorm_ref(i["x"], i["weight"], i["bias"], **k),
    "softmax": lambda i, k: ref.softmax_ref(i["x"], **k),
    "rotary_embedding": lambda i, k: ref.rotary_embedding_ref(i["x"], i["cos"], i["sin"]),
    "reduce": lambda i, k: ref.reduce_sum_ref(i["x"], **k),
    "cross_entropy": lambda i, k: ref.cross_entropy_ref(i["logits"], i["targets"]),
    "matmul": lambda i, k: ref.matmul_ref(i["A"], i["B"]),
    "fused_mlp": lambda i, k: ref.fused_mlp_ref(i["x"], i["w_gate"], i["w_up"], i["w_down"], **k),
    "flash_attention": lambda i, k: ref.flash_attention_ref(i["Q"], i["K"], i["V"], **k),
}


def main():
    by_op: dict[str, list] = {}
    for op, dt, name, inputs, kw in cases():
        dtype = DT[dt]
        ins = {k: (v.to(dtype) if v.is_floating_point() else v) for k, v in inputs.items()}
        ins32 = {k: (v.float() if v.is_floating_point() else v) for k, v in ins.items()}
        o = REF_FN[op](ins, kw)
        o32 = REF_FN[op](ins32, kw)
        by_op.setdefault(op, []).append(
            {"name": f"{name}_{dt}", "dtype": dt, "inputs": ins, "kwargs": kw,
             "out": o, "out_f32": o32})
    total = 0
    for op, cs in by_op.items():
        p = HERE / f"{op}.pt"
        torch.save(cs, p)
        total += p.stat().st_size
        print(f"{p.name}: {len(cs)} cases, {p.stat().st_size / 1e3:.0f} KB")
    print(f"total {total / 1e6:.2f} MB")


if __name__ == "__main__":
    main()
