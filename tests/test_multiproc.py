"""Replica aggregation of bench.py across ranks, on 2 gloo processes (CPU)."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import datetime
    import sys
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    local_ms = 100.0 * (rank + 1)  # rank 1 is the slow one
    value, max_ms = bench.aggregate(local_ms, 50, dist)
    q.put((rank, value, max_ms, bench.replica_streams(64, rank, world)))
    dist.barrier()
    dist.destroy_process_group()


def test_aggregate_takes_max_over_ranks():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, value, max_ms, streams in res:
        assert max_ms == 200.0
        assert value == pytest.approx(2 * 50 / 0.2)  # whole-job tokens / slowest rank's time
    assert res[0][3] == list(range(0, 64, 2)) and res[1][3] == list(range(1, 64, 2))


def test_single_process_aggregate():
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    v, m = bench.aggregate(250.0, 100)
    assert m == 250.0 and v == pytest.approx(400.0)
