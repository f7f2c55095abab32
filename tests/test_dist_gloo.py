"""Multi-process host logic on CPU ranks (gloo, world size 2): request sharding,
the final gather of committed tokens, and a rank that fails between steps."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from yapd_b200.shard import gather_committed, shard_range


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_range_partitions():
    for total in (0, 1, 7, 64, 2048):
        for world in (1, 2, 3, 8):
            spans = [shard_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [h - l for l, h in spans]
            assert max(sizes) - min(sizes) <= 1


def _gather_worker(rank, world, port, total, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lo, hi = shard_range(total, world, rank)
    xt = torch.arange(lo * 4, hi * 4, dtype=torch.int64).view(hi - lo, 4)
    full = gather_committed(xt, total, dist)
    q.put((rank, full.tolist()))
    dist.destroy_process_group()


def test_gather_committed_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    total = 5
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, total, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=60) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = torch.arange(total * 4).view(total, 4).tolist()
    assert res[0] == want and res[1] == want


def _failing_worker(rank, world, port, q):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        # a rank that dies between steps, with no collective in flight
        os._exit(3)
    try:
        gather_committed(torch.zeros(1, 4, dtype=torch.int64), 2, dist)
        q.put("no error")
    except Exception as e:  # the survivor's collective ends with an error, not a hang
        q.put(type(e).__name__)


def test_rank_failure_is_reported_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    msg = q.get(timeout=90)
    for p in procs:
        p.join(timeout=90)
    assert msg != "no error"
    assert procs[1].exitcode == 3
