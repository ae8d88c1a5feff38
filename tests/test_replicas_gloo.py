"""Replica sharding and the max/sum-over-ranks aggregation of bench.py, run as two gloo
ranks on CPU (the GPU run uses the same functions over NCCL)."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from speech_serving import replicas


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    try:
        mine = replicas.shard(list(range(10)), world, rank)
        lo, hi = replicas.shard_range(10, world, rank)
        ms = 5.0 + 3.0 * rank  # rank 1 is the slower one
        ms_max = replicas.max_over_ranks(ms)
        units = replicas.sum_over_ranks(len(mine))
        every = replicas.gather_over_ranks(ms)
        q.put((rank, mine, (lo, hi), ms_max, units, replicas.whole_job_rate(units, ms_max), every))
    finally:
        dist.destroy_process_group()


def test_two_rank_replicas_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (_, m0, r0, t0, u0, v0, e0), (_, m1, r1, t1, u1, v1, e1) = res
    assert m0 == [0, 2, 4, 6, 8] and m1 == [1, 3, 5, 7, 9]
    assert r0 == (0, 5) and r1 == (5, 10)
    assert t0 == t1 == 8.0  # every rank reports the slowest rank's time
    assert u0 == u1 == 10
    assert v0 == pytest.approx(10 / 8e-3)
    assert e0 == e1 == [5.0, 8.0]  # per-rank values in rank order


def test_single_process_fallbacks():
    assert replicas.max_over_ranks(3.5) == 3.5
    assert replicas.gather_over_ranks(2.0) == [2.0]
    assert replicas.shard([1, 2, 3], 1, 0) == [1, 2, 3]
    with pytest.raises(ValueError):
        replicas.shard([1], 2, 2)
    with pytest.raises(ValueError):
        replicas.whole_job_rate(1, 0)


def _dying_worker(rank, world, port, q):
    """Rank 1 dies after joining the group (a replica whose serving loop crashed); rank 0
    then aggregates as bench.py does and must get an error, not hang."""
    import time
    from datetime import timedelta

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(3)
    t0 = time.monotonic()
    try:
        replicas.max_over_ranks(1.0)
        q.put(("returned", time.monotonic() - t0))
    except Exception as e:  # the collective's error on a lost peer or its timeout
        q.put(("raised", type(e).__name__, time.monotonic() - t0))
    os._exit(0)  # the group is broken: leave without a collective teardown


def test_lost_rank_ends_the_aggregation_with_an_error():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert res[0] == "raised", res
    assert res[-1] < 60.0  # bounded by the group's timeout, not a hang
    assert procs[1].exitcode == 3 and procs[0].exitcode == 0
