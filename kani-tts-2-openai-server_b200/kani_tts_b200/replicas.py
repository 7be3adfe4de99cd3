"""Data-parallel replicas: independent speech streams sharded over GPUs.

The decode path has no exchange step: each GPU owns a contiguous shard of
the streams, with its own weight replica, static caches and CUDA graph
(one process per GPU).  The only cross-rank traffic is the bookkeeping
below: a barrier around timed regions and max / sum reductions of scalars
(timings, token counts) over ``torch.distributed``.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def stream_shard(total_streams: int, world: int, rank: int) -> range:
    """Contiguous, balanced shard of stream ids owned by `rank` (sizes differ by <= 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(total_streams, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def _reduce(x: float, op, device) -> float:
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=op)
    return float(t.item())


def max_over_ranks(x: float, device="cpu") -> float:
    """Max of a per-rank scalar (used for wall times: the job ends with its slowest rank)."""
    return _reduce(x, dist.ReduceOp.MAX if dist.is_available() else None, device)


def sum_over_ranks(x: float, device="cpu") -> float:
    """Sum of a per-rank scalar (units of work processed)."""
    return _reduce(x, dist.ReduceOp.SUM if dist.is_available() else None, device)


def aggregate_throughput(units: float, seconds: float, device="cpu") -> tuple[float, float, float]:
    """(total units, slowest rank's seconds, units per second for the whole job)."""
    total = sum_over_ranks(units, device)
    slowest = max_over_ranks(seconds, device)
    return total, slowest, (total / slowest if slowest > 0 else 0.0)


def barrier() -> None:
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()
