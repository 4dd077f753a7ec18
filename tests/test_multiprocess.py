"""Multi-process host logic on CPU (gloo, world size 2).

The paged-KV path shards whole sequences across ranks with no collective on
the hot path; the only cross-rank steps are the start barrier and the
max-over-ranks timing reduction of bench.py. This test runs those steps on
two gloo ranks: every rank must compute the same LPT assignment
independently, the shards must partition the job, and the timing reduction
must return the slowest rank's time on every rank. A second test makes one
rank fail before joining and checks that the other sees an error within its
process-group timeout instead of hanging.
"""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        import random

        from grpo_training_engine_b200.sharding import lpt_assign

        rng = random.Random(1234)
        costs = [rng.randint(1024, 8192) for _ in range(256)]
        parts = lpt_assign(costs, world)
        gathered = [None] * world
        dist.all_gather_object(gathered, parts[rank])
        t = torch.tensor([float(rank + 1) * 0.5])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        q.put((rank, gathered, parts, float(t)))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharding_and_max_timing():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, gathered, parts, tmax in results:
        assert gathered == parts  # every rank derived the same assignment
        assert sorted(i for part in gathered for i in part) == list(range(256))
        assert tmax == 1.0  # slowest rank's time


def _worker_fail(rank: int, world: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if rank == 1:
        raise SystemExit(3)  # never joins the group
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        dist.barrier()
        q.put("joined")
    except Exception as exc:  # the store / barrier times out
        q.put(f"error:{type(exc).__name__}")


@pytest.mark.timeout(120)
def test_missing_rank_is_detected_not_hung():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_fail, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    msg = q.get(timeout=100)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert msg.startswith("error:")
    assert procs[1].exitcode == 3
