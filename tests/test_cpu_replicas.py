"""The multi-GPU replica plumbing (voxgen_b200/replicas.py) with two gloo ranks on the CPU: the
start barrier, the max over ranks of the device-timed duration, the whole-job rate, and the
partition of independent streams over ranks. The data path has no collective, so this is all
the N > 1 host logic there is."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from voxgen_b200 import replicas


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    r, w, local = replicas.env()
    pg = replicas.init("gloo", w, timeout_s=60)
    replicas.barrier(pg)
    ms = 10.0 + 5.0 * r                      # rank 1 is the slow replica
    mx = replicas.max_over_ranks(ms, pg)
    mine = replicas.shard(list(range(16)), r, w)
    replicas.barrier(pg)
    replicas.shutdown(pg)
    q.put((r, w, local, mx, mine))


def test_two_gloo_ranks():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [o[0] for o in out] == [0, 1] and all(o[1] == 2 for o in out)
    assert all(o[3] == 15.0 for o in out), "every rank sees the slowest rank's time"
    shards = [o[4] for o in out]
    assert sorted(shards[0] + shards[1]) == list(range(16)) and not set(shards[0]) & set(shards[1])


def test_single_process_and_rate():
    assert replicas.init("gloo", 1) is None
    assert replicas.max_over_ranks(3.5, None) == 3.5
    # 8 replicas of 1000 steps each, slowest took 1.25 s: 6400 steps per second for the job
    assert replicas.aggregate_rate(1000, 8, 1250.0) == pytest.approx(6400.0)
    assert replicas.shard(list(range(5)), 1, 2) == [1, 3]
