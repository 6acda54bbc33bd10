"""B200 row and roofline helpers for AutoKernel's bench.py (autokernel_b200.gpuspec), checked
against a stand-in bench module with the same table / config structure (bench.py:103-122,
330-597) and the clock-based fallback it replaces (bench.py:167-175)."""
from __future__ import annotations

import json
import types

import torch

from autokernel_b200 import gpuspec


def _fake_bench():
    return types.SimpleNamespace(
        _KNOWN_GPUS={"H100 SXM": (989.5, 3352.0, 50.0), "A100": (312.0, 2039.0, 40.0)},
        KERNEL_CONFIGS={
            "flash_attention": {"flops_fn": lambda s: 4 * s["batch"] * s["heads"] * s["seq_len"] ** 2 * s["head_dim"]},
            "cross_entropy": {"bytes_fn": lambda s, dt: (s["batch"] * s["vocab"] + s["batch"]) * 2},
        })


def _match(table, name):
    """bench.py's lookup: the first fragment contained in the device name."""
    for frag, spec in table.items():
        if frag in name:
            return spec
    return None


def test_install_adds_b200_row_first():
    b = _fake_bench()
    peaks = gpuspec.install(b)
    assert next(iter(b._KNOWN_GPUS)) == "B200"
    assert _match(b._KNOWN_GPUS, "NVIDIA B200") == (2250.0, 7700.0, 126.0) == peaks.known_gpus_row()
    assert _match(b._KNOWN_GPUS, "NVIDIA H100 SXM") == (989.5, 3352.0, 50.0)
    gpuspec.install(b)  # idempotent
    assert list(b._KNOWN_GPUS).count("B200") == 1


def test_nominal_row_vs_clock_fallback():
    """Without the row, bench.py estimates 148 SMs x 256 ops x 1.965 GHz x 2 = 149 TFLOP/s and
    max(1.965 x 32 x 2, 500) = 500 GB/s: 15x and 15x too low."""
    fallback_tf = 148 * 256 * 1.965 * 2 / 1e3
    assert abs(fallback_tf - 149.0) < 0.5
    assert gpuspec.B200_NOMINAL.fp16_tflops / fallback_tf > 14
    assert gpuspec.B200_NOMINAL.hbm_gb_s / 500.0 > 14


def test_measured_peaks(tmp_path):
    p = tmp_path / "peaks.json"
    p.write_text(json.dumps({"hbm_gbs": 6540.5, "bf16_tflops": 1650.2}))
    b = _fake_bench()
    peaks = gpuspec.install(b, measured_path=p)
    assert b._KNOWN_GPUS["B200"] == (1650.2, 6540.5, 126.0) == peaks.known_gpus_row()


def test_causal_flops_and_int64_targets():
    b = _fake_bench()
    s = {"batch": 8, "heads": 32, "seq_len": 4096, "head_dim": 128}
    full = b.KERNEL_CONFIGS["flash_attention"]["flops_fn"](s)
    gpuspec.install(b)
    causal = b.KERNEL_CONFIGS["flash_attention"]["flops_fn"](s)
    assert causal == 2 * 8 * 32 * 128 * 4096 * 4097  # 1.0998e12, the causal count
    assert abs(causal / full - 4097 / 8192) < 1e-12
    ce = {"batch": 4096, "vocab": 32000}
    assert b.KERNEL_CONFIGS["cross_entropy"]["bytes_fn"](ce, torch.float16) == 4096 * 32000 * 2 + 4096 * 8
    assert b.KERNEL_CONFIGS["cross_entropy"]["bytes_fn"](ce, torch.float32) == 4096 * 32000 * 4 + 4096 * 8
