"""Row / batch sharding of the operators across the GPUs of one node.

One process per GPU (torchrun); each rank owns a contiguous block of rows (or of
the batch for attention / RoPE).  Row-wise operators need no communication.
The two operators whose result couples all rows do one fp64 all-reduce of a
per-rank partial, over NCCL on NVLink when the process group is NCCL:

    reduce        partial = fp64 sum of the local elements   -> SUM -> cast
    cross_entropy partial = fp64 (sum of row losses, rows)    -> SUM -> sum / rows

The reference has no distributed code; this module is the build's own
(row/batch data parallelism of the same arithmetic).  Partials are fp64, so
the result differs from the single-GPU one only by fp64 rounding.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def row_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, stop) block of n rows for `rank`; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_rows(t: torch.Tensor, rank: int, world: int, dim: int = 0) -> torch.Tensor:
    """This rank's contiguous block of t along dim (a view)."""
    a, b = row_range(t.shape[dim], rank, world)
    return t.narrow(dim, a, b - a)


def _default_partial_sum(x: torch.Tensor) -> torch.Tensor:
    from . import ops
    return ops.reduce_partial(x)


def _default_partial_ce(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    from . import ops
    return ops.cross_entropy_partial(logits, targets)


def reduce_sum_sharded(x_local: torch.Tensor, group=None, out_dtype: torch.dtype | None = None,
                       partial_fn: Callable[[torch.Tensor], torch.Tensor] = _default_partial_sum,
                       finalize: bool = True) -> torch.Tensor:
    """Global sum of all ranks' elements.  Returns a 0-d tensor of out_dtype (x's dtype by
    default), or the all-reduced fp64 1-element total when finalize is False."""
    total = partial_fn(x_local)
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(total, op=dist.ReduceOp.SUM, group=group)
    if not finalize:
        return total
    dtype = out_dtype or x_local.dtype
    if total.is_cuda:
        from . import ops
        return ops.scalar_from_total(total, dtype)
    return total.reshape(()).to(dtype)


def cross_entropy_sharded(logits_local: torch.Tensor, targets_local: torch.Tensor, group=None,
                          partial_fn: Callable = _default_partial_ce,
                          out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Mean cross entropy over all ranks' rows (rows with target -100 are not counted).
    `partial_fn(x, targets)` gives the shard's fp64 (sum, count); with a fused LM head x is
    the hidden state rather than the logits."""
    sc = partial_fn(logits_local, targets_local)
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(sc, op=dist.ReduceOp.SUM, group=group)
    dtype = out_dtype or logits_local.dtype
    if sc.is_cuda:
        from . import ops
        return ops.mean_from_sum_count(sc, dtype)
    return (sc[0] / sc[1]).to(dtype)


def max_over_ranks(value: float, device=None, group=None) -> float:
    """Maximum of a host float over all ranks (timing: the slowest rank defines a step)."""
    if not (dist.is_available() and dist.is_initialized()):
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
