"""Row-sharded reduce and cross entropy over 2 GPUs with NCCL: the all-reduced results equal the
single-GPU ones (fp64 partials) and the float64 oracle.  Skipped with fewer than 2 GPUs."""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        from autokernel_b200 import ops, shard
        g = torch.Generator().manual_seed(0)
        x = torch.rand(1 << 22, generator=g) * 2 - 1
        logits = torch.randn(1024, 32000, generator=g).half()
        t = torch.randint(0, 32000, (1024,), generator=g)
        s = shard.reduce_sum_sharded(shard.shard_rows(x, rank, world).to(dev), finalize=False)
        ce = shard.cross_entropy_sharded(shard.shard_rows(logits, rank, world).to(dev),
                                         shard.shard_rows(t, rank, world).to(dev))
        single_s = float(ops.reduce(x.to(dev)).double())  # fp32 output
        single_ce = float(ops.cross_entropy(logits.to(dev), t.to(dev)).float())
        q.put((rank, float(s.item()), float(ce.float()), single_s, single_ce))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_reduce_and_cross_entropy_nccl():
    from oracle import ref_f64
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=180) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
    g = torch.Generator().manual_seed(0)
    x = torch.rand(1 << 22, generator=g) * 2 - 1
    logits = torch.randn(1024, 32000, generator=g).half()
    t = torch.randint(0, 32000, (1024,), generator=g)
    want_s = ref_f64.reduce_sum(x.double().numpy(), 0)
    want_ce = ref_f64.cross_entropy(logits.float().numpy(), t.numpy())
    for _, s, ce, single_s, single_ce in res:
        assert abs(s - want_s) <= 1e-6 * max(1.0, abs(want_s)) + 1e-3
        assert abs(ce - want_ce) <= 1e-2 * max(1.0, abs(want_ce))
        assert abs(s - single_s) <= 1e-2  # single-GPU result is rounded to fp32
        assert abs(ce - single_ce) <= 1e-2
