"""The multi-GPU path is independent replicas; its host-side pieces (stream
sharding, max / sum aggregation of timings and work) run here as two gloo
ranks on the CPU."""
from __future__ import annotations

import os
import socket

import pytest
import torch.multiprocessing as mp

from kani_tts_b200.replicas import aggregate_throughput, gather_over_ranks, max_over_ranks, stream_shard


def test_stream_shard_partitions_all_streams():
    for total in (0, 1, 63, 64, 128, 512, 513):
        for world in (1, 2, 3, 4, 8):
            shards = [stream_shard(total, world, r) for r in range(world)]
            ids = [i for s in shards for i in s]
            assert ids == list(range(total))
            sizes = [len(s) for s in shards]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        stream_shard(8, 2, 2)


def test_single_process_aggregation_is_identity():
    assert max_over_ranks(3.5) == 3.5
    assert gather_over_ranks(3.5) == [3.5]
    assert aggregate_throughput(64 * 1500, 2.0) == (96000.0, 2.0, 48000.0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shard = stream_shard(64 * world, world, rank)
        # rank r "processes" its shard in (r + 1) seconds
        total, slowest, rate = aggregate_throughput(len(shard) * 1500, float(rank + 1))
        per_rank = gather_over_ranks(7.5 + rank)   # the bench's per-rank times, in rank order
        q.put((rank, list(shard)[:1], len(shard), total, slowest, rate, per_rank))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_aggregate_like_the_bench():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    assert [r[1] for r in res] == [[0], [64]]           # disjoint shards of 64 streams
    for _, _, n, total, slowest, rate, per_rank in res:
        assert n == 64
        assert total == 2 * 64 * 1500
        assert slowest == 2.0                            # max over ranks
        assert rate == total / 2.0
        assert per_rank == [7.5, 8.5]                    # every rank's value, in rank order


def _replica_worker(rank, world, port, mode, q):
    """rank 0 hosts the store and collects; the others report, raise or die."""
    import os
    import torch.distributed as dist
    from kani_tts_b200 import replicas as R
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=__import__("datetime").timedelta(seconds=20))
    if rank == 1 and mode == "killed":
        os._exit(3)                                   # the process dies without a word
    if rank == 1 and mode == "raised":
        try:
            raise RuntimeError("replica 1: CUDA error 700")
        except RuntimeError as e:
            R.report_outcome(store, rank, error=str(e))
    else:
        R.report_outcome(store, rank, units=1000.0 * (rank + 1), seconds=0.5 + 0.1 * rank)
    if rank == 0:
        q.put(R.collect_outcomes(store, world, timeout_s=3.0))
        # keep the store alive until the others are done with it
        import time
        time.sleep(0.5)


@pytest.mark.parametrize("mode", ["killed", "raised"])
def test_failed_replica_is_reported_and_the_others_count(mode):
    """Three replica processes; replica 1 dies (or reports an exception).  The
    collector returns within its deadline, names replica 1 as failed and adds up
    the work of replicas 0 and 2 (slowest ok time 0.7 s)."""
    import multiprocessing as mp
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_replica_worker, args=(r, 3, port, mode, q)) for r in range(3)]
    for p in procs:
        p.start()
    summary = q.get(timeout=60)
    for p in procs:
        p.join(timeout=30)
    assert summary["ok"] == [0, 2]
    assert list(summary["failed"]) == [1]
    if mode == "raised":
        assert "CUDA error 700" in summary["failed"][1]
    else:
        assert "no report" in summary["failed"][1]
    assert summary["units"] == 4000.0 and abs(summary["seconds"] - 0.7) < 1e-9
    assert procs[1].exitcode == (3 if mode == "killed" else 0)
