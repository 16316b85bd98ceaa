"""Multi-rank bookkeeping on CPU with world-size-2 gloo process groups: the
shard split covers every (batch, head) unit exactly once, and the job value
is computed from the slowest rank's time (max over ranks)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from neurodsl_b200 import ranks


def test_shard_range_covers_units_once():
    for n in (0, 1, 7, 128, 768):
        for world in (1, 2, 3, 4, 8):
            covered = []
            for r in range(world):
                a, b = ranks.shard_range(n, r, world)
                covered.extend(range(a, b))
                assert b - a in (n // world, n // world + 1)
            assert covered == list(range(n))
    with pytest.raises(ValueError):
        ranks.shard_range(4, 2, 2)


def test_job_throughput():
    assert ranks.job_throughput(10.0, 4, 2.0) == 20.0
    with pytest.raises(ValueError):
        ranks.job_throughput(1.0, 1, 0.0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        r, w, lr = ranks.dist_env()
        assert (r, w, lr) == (rank, world, rank)
        ms = 10.0 + 5.0 * rank           # rank 1 is the slow one
        mx = ranks.max_over_ranks(ms)
        # every rank holds the units of its shard of 128 (batch, head) pairs
        a, b = ranks.shard_range(128, rank, world)
        t = torch.tensor([b - a], dtype=torch.int64)
        dist.all_reduce(t)
        dist.barrier()
        q.put((rank, mx, int(t.item()), ranks.job_throughput(1.0, world, mx / 1e3)))
    finally:
        dist.destroy_process_group()


def test_gloo_world_size_2_max_over_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = sorted(q.get(timeout=10) for _ in range(2))
    for rank, mx, total, thr in got:
        assert mx == 15.0            # both ranks see the slowest rank's time
        assert total == 128          # shards cover every unit once
        assert abs(thr - 2 / 0.015) < 1e-6


def test_max_over_ranks_without_process_group():
    assert ranks.max_over_ranks(3.5) == 3.5
