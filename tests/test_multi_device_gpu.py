"""One process, two GPUs: every kernel that opts into more than 48 KB of shared memory (the
tcgen05 GEMM in its plain, dual and cross-entropy modes, the attention kernel and the softmax
ring) must run on cuda:1 after it has run on cuda:0.  The opt-in attribute belongs to each
device's context, so it is set once per (kernel, device).  Skipped with fewer than 2 GPUs."""
from __future__ import annotations

import pytest
import torch

from oracle import ref_f64
from parity import check, reference_mlp_hidden, to_np

pytestmark = pytest.mark.gpu


def _run_all(dev):
    from autokernel_b200 import _lib, ops
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    bf = torch.bfloat16
    A = (torch.randn(512, 256, device=dev, generator=g) / 16).to(bf)
    B = torch.randn(256, 384, device=dev, generator=g).to(bf)
    check(ops.matmul(A, B), ref_f64.matmul(to_np(A), to_np(B)), "matmul", f"{dev} matmul")
    wg, wu = ((torch.randn(512, 256, device=dev, generator=g) * 0.05).to(bf) for _ in range(2))
    wd = (torch.randn(256, 512, device=dev, generator=g) * 0.05).to(bf)
    y = ops.fused_mlp(A, wg, wu, wd)
    check(y, to_np(reference_mlp_hidden(A, wg, wu, "silu", bf)) @ to_np(wd).T, "fused_mlp",
          f"{dev} mlp")
    Q, K, V = (torch.randn(1, 2, 256, 128, device=dev, generator=g).to(bf) for _ in range(3))
    check(ops.flash_attention(Q, K, V), ref_f64.attention(to_np(Q), to_np(K), to_np(V), True),
          "flash_attention", f"{dev} attention")
    x = torch.randn(64, 16384, device=dev, generator=g).to(bf)  # 32 KiB rows: the TMA ring
    check(ops.softmax(x), ref_f64.softmax(to_np(x)), "softmax", f"{dev} softmax")
    t = torch.randint(0, 1000, (300,), device=dev, generator=g)
    h = torch.randn(300, 256, device=dev, generator=g).to(bf)
    W = (torch.randn(1000, 256, device=dev, generator=g) * 0.02).to(bf)
    loss, _ = ops.linear_cross_entropy_rows(h, W, t)
    loss_u, _ = ops.cross_entropy_rows(ops.linear(h, W), t)
    check(loss, to_np(loss_u), "cross_entropy", f"{dev} fused LM head")
    torch.cuda.synchronize(dev)
    assert _lib.device_status() == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_kernels_on_second_device_after_first():
    _run_all(torch.device("cuda", 0))
    _run_all(torch.device("cuda", 1))
    _run_all(torch.device("cuda", 0))
