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


def gather_over_ranks(x: float, device="cpu") -> list[float]:
    """Every rank's value of a per-rank scalar, in rank order (one all-gather)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [float(x)]
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    out = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [float(v.item()) for v in out]


def aggregate_throughput(units: float, seconds: float, device="cpu") -> tuple[float, float, float]:
    """(total units, slowest rank's seconds, units per second for the whole job)."""
    total = sum_over_ranks(units, device)
    slowest = max_over_ranks(seconds, device)
    return total, slowest, (total / slowest if slowest > 0 else 0.0)


def barrier() -> None:
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


# ----------------------------------------------------------- failed replicas
#
# The collectives above assume every replica finishes.  For serving, a replica
# that dies (its process killed, an exception) must not stall the others: each
# rank posts its outcome to the process group's key-value store, and rank 0
# collects with a deadline instead of a collective, so a silent rank is
# reported as failed and the finished replicas' work still counts.

def report_outcome(store, rank: int, units: float = 0.0, seconds: float = 0.0, error: str | None = None,
                   prefix: str = "replica") -> None:
    """Post this rank's result (or its error) under ``prefix/rank`` in a
    ``torch.distributed`` Store (TCPStore / FileStore / HashStore)."""
    msg = f"error:{error}" if error is not None else f"ok:{float(units)!r}:{float(seconds)!r}"
    store.set(f"{prefix}/{rank}", msg)


def collect_outcomes(store, world: int, timeout_s: float = 30.0, poll_s: float = 0.05,
                     prefix: str = "replica") -> dict:
    """Wait (at most ``timeout_s``) for every rank's report and summarise:
    ``{"ok": [ranks], "failed": {rank: reason}, "units": sum over ok ranks,
    "seconds": slowest ok rank, "rate": units / seconds}``.  A rank that never
    reports within the deadline is listed as failed; the call never blocks on a
    collective, so it returns even when a replica process has died."""
    import time
    keys = {r: f"{prefix}/{r}" for r in range(world)}
    pending = set(keys)
    results: dict[int, str] = {}
    deadline = time.monotonic() + timeout_s
    while pending:
        for r in sorted(pending):
            if store.check([keys[r]]):
                results[r] = store.get(keys[r]).decode()
                pending.discard(r)
        if not pending or time.monotonic() > deadline:
            break
        time.sleep(poll_s)
    ok, failed, units, seconds = [], {}, 0.0, 0.0
    for r in range(world):
        msg = results.get(r)
        if msg is None:
            failed[r] = f"no report within {timeout_s:g} s"
        elif msg.startswith("error:"):
            failed[r] = msg[len("error:"):]
        else:
            _, u, s = msg.split(":")
            ok.append(r)
            units += float(u)
            seconds = max(seconds, float(s))
    return {"ok": ok, "failed": failed, "units": units, "seconds": seconds,
            "rate": units / seconds if seconds > 0 else 0.0}
