"""Multi-rank host logic of autokernel_b200.shard on CPU (gloo, world_size 2).

The per-rank partials come from the CPU oracle here (no GPU in these tests); on a GPU box
they come from the CUDA kernels and the process group is NCCL, with the same host code."""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from autokernel_b200.shard import (cross_entropy_sharded, max_over_ranks, reduce_sum_sharded,
                                   row_range, shard_rows)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _partial_sum(x):
    from oracle import ref_f64
    return torch.tensor([ref_f64.reduce_sum(x.double().numpy().reshape(-1), 0)], dtype=torch.float64)


def _partial_ce(logits, targets):
    from oracle import ref_f64
    loss, _, _, keep = ref_f64.cross_entropy_rows(logits.double().numpy(), targets.numpy())
    return torch.tensor([loss.sum(), float(keep.sum())], dtype=torch.float64)


def _worker(rank, world, port, q, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        g = torch.Generator().manual_seed(0)
        x = torch.rand(1001, 37, generator=g) * 2 - 1
        logits = torch.randn(203, 50, generator=g)
        t = torch.randint(0, 50, (203,), generator=g)
        t[5] = -100
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected rank failure before the collective")
        s = reduce_sum_sharded(shard_rows(x, rank, world), partial_fn=_partial_sum,
                               out_dtype=torch.float64)
        ce = cross_entropy_sharded(shard_rows(logits, rank, world).double(),
                                   shard_rows(t, rank, world), partial_fn=_partial_ce)
        m = max_over_ranks(float(rank) + 0.5)
        q.put((rank, "ok", float(s), float(ce), m))
    except Exception as e:  # reported to the parent, never hangs the test
        q.put((rank, "err", repr(e), None, None))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _launch(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(res)


@pytest.mark.parametrize("n,world", [(10, 3), (1001, 2), (7, 8), (0, 4), (8192, 8)])
def test_row_range_partitions(n, world):
    spans = [row_range(n, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1


def test_sharded_sum_and_cross_entropy_match_single_process():
    from oracle import ref_f64
    res = _launch("ok")
    g = torch.Generator().manual_seed(0)
    x = torch.rand(1001, 37, generator=g) * 2 - 1
    logits = torch.randn(203, 50, generator=g)
    t = torch.randint(0, 50, (203,), generator=g)
    t[5] = -100
    want_s = ref_f64.reduce_sum(x.double().numpy().reshape(-1), 0)
    want_ce = ref_f64.cross_entropy(logits.double().numpy(), t.numpy())
    for rank, status, s, ce, m in res:
        assert status == "ok", s
        assert abs(s - want_s) <= 1e-9 * max(1.0, abs(want_s))
        assert abs(ce - want_ce) <= 1e-12 * max(1.0, abs(want_ce))
        assert m == 1.5  # max over ranks of rank + 0.5


def test_rank_failure_surfaces_as_error_not_hang():
    """A rank that dies before the collective makes the survivor's collective fail within
    the process-group timeout; both outcomes are reported to the parent."""
    res = _launch("fail")
    status = {r: s for r, s, *_ in res}
    assert status[1] == "err"
    assert status[0] == "err"
