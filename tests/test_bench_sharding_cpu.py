"""bench.py's multi-GPU plumbing on the CPU: two gloo ranks (world size 2,
127.0.0.1) check that the per-rank image shards are disjoint and together
cover 0 .. world*batch-1, and that the timing reduction returns the maximum
over ranks (the slowest rank defines the job's time)."""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, batch, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      GLOO_SOCKET_IFNAME="lo")
    sys.path.insert(0, str(ROOT))
    import datetime

    import torch
    import torch.distributed as dist

    import bench

    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    try:
        seeds = list(bench.shard_seeds(rank, batch))
        gathered = [None] * world
        dist.all_gather_object(gathered, seeds)
        elapsed = 10.0 + 5.0 * rank  # rank 1 is the slow one
        q.put((rank, gathered, bench.max_over_ranks(elapsed, dist)))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharding_and_max_timing():
    world, batch = 2, 5
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, batch, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, gathered, tmax in results:
        flat = [s for shard in gathered for s in shard]
        assert sorted(flat) == list(range(world * batch))  # disjoint and complete
        assert len(set(flat)) == len(flat)
        assert gathered[rank] == list(range(rank * batch, (rank + 1) * batch))
        assert tmax == pytest.approx(15.0)  # max over ranks, on every rank


def test_single_process_reduction_is_identity():
    sys.path.insert(0, str(ROOT))
    import bench

    assert bench.max_over_ranks(3.5, None) == 3.5
    assert list(bench.shard_seeds(0, 4)) == [0, 1, 2, 3]
