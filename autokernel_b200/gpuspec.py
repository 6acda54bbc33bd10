"""B200 awareness for AutoKernel's benchmark harness (bench.py).

AutoKernel's bench.py rates every kernel against a GPU table (`_KNOWN_GPUS`,
bench.py:103-122: name fragment -> (peak fp16 TFLOP/s, peak HBM GB/s, L2 MB)) that has no
Blackwell row; a B200 falls through to the clock-based estimate (bench.py:167-175), which
assumes 256 fp16 ops/clk/SM and a 256-bit bus -> ~150 TFLOP/s and ~500 GB/s, so every
roofline percentage it prints on a B200 is wrong by an order of magnitude.  The ridge point
uses the fp16 peak (bench.py:1073), which on B200 equals the dense bf16 peak, and the
flash-attention FLOP count is 4*B*H*S^2*D (bench.py:446) although the kernel contract is
causal by default (half the work).

This module supplies the B200 row (nominal datasheet figures, or the peaks measured on the
machine when a MEASURED_PEAKS.json is given), a causal FLOP count, and `install()`, which
adds both to an imported bench module without editing its source:

    import bench                                  # AutoKernel's bench.py
    from autokernel_b200 import gpuspec
    gpuspec.install(bench)                        # or install(bench, measured="MEASURED_PEAKS.json")
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path


@dataclass(frozen=True)
class Peaks:
    name: str
    fp16_tflops: float   # dense tensor-core fp16 (= bf16 on B200)
    hbm_gb_s: float
    l2_mb: float

    def known_gpus_row(self) -> tuple[float, float, float]:
        """The (peak fp16 TFLOP/s, peak GB/s, L2 MB) tuple bench.py's table holds."""
        return (self.fp16_tflops, self.hbm_gb_s, self.l2_mb)


# Datasheet: 2.25 PFLOP/s dense bf16/fp16 (the 4.5 figure is 2:4 sparse), HBM3e 7.7 TB/s
# (HGX), 126 MB L2 (nvidia-smi / cudaDeviceProp on the part).
B200_NOMINAL = Peaks("B200", 2250.0, 7700.0, 126.0)
NAME_FRAGMENT = "B200"  # matched as a substring of torch.cuda.get_device_properties().name


def measured(path: str | Path) -> Peaks:
    """Peaks measured on the machine: a copy bandwidth and a cuBLAS bf16 GEMM rate
    (keys hbm_gbs and bf16_tflops), with the nominal L2 size."""
    d = json.loads(Path(path).read_text())
    return Peaks("B200 (measured)", float(d["bf16_tflops"]), float(d["hbm_gbs"]), B200_NOMINAL.l2_mb)


def causal_attention_flops(s: dict) -> float:
    """FLOPs of causal attention for bench.py's flash_attention shape dict
    (batch, heads, seq_len, head_dim): Q K^T and P V over the S(S+1)/2 visible pairs."""
    return 2.0 * s["batch"] * s["heads"] * s["head_dim"] * s["seq_len"] * (s["seq_len"] + 1)


def cross_entropy_bytes(s: dict, dt) -> float:
    """Bytes cross entropy moves, as a bench.py bytes_fn (shape dict with batch and vocab,
    logits dtype): the logits once plus int64 targets at 8 bytes each (bench.py:508 counts
    them at the logits' width)."""
    import torch
    esz = torch.empty((), dtype=dt).element_size()
    return s["batch"] * s["vocab"] * esz + s["batch"] * 8


def install(bench, measured_path: str | Path | None = None, causal_flops: bool = True,
            int64_targets: bool = True) -> Peaks:
    """Register the B200 row in `bench._KNOWN_GPUS` (first, so it wins the substring match);
    with causal_flops count flash-attention work as causal, with int64_targets count cross
    entropy's targets at 8 bytes.  Returns the row used."""
    peaks = measured(measured_path) if measured_path else B200_NOMINAL
    table = dict(getattr(bench, "_KNOWN_GPUS", {}))
    table.pop(NAME_FRAGMENT, None)
    bench._KNOWN_GPUS = {NAME_FRAGMENT: peaks.known_gpus_row(), **table}
    cfgs = getattr(bench, "KERNEL_CONFIGS", None)
    if causal_flops and cfgs and "flash_attention" in cfgs:
        cfgs["flash_attention"]["flops_fn"] = causal_attention_flops
    if int64_targets and cfgs and "cross_entropy" in cfgs:
        cfgs["cross_entropy"]["bytes_fn"] = cross_entropy_bytes
    return peaks


__all__ = ["Peaks", "B200_NOMINAL", "NAME_FRAGMENT", "measured", "causal_attention_flops",
           "cross_entropy_bytes", "install"]
