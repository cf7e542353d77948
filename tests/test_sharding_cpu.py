"""Multi-rank host logic on CPU: sequence sharding, the optional output gather over gloo ranks,
and failure detection when a rank dies between steps (injected on the host, no GPU)."""

from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from miniserve_b200.sharding import gather_rows, shard_by_tokens, shard_loads
from miniserve_b200.workloads import config5_contexts


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_config5_shards_cover_every_sequence_once_and_balance(world: int) -> None:
    ctx = config5_contexts(seed=0)
    shards = shard_by_tokens(ctx.tolist(), world)
    flat = sorted(i for s in shards for i in s)
    assert flat == list(range(len(ctx)))
    loads = shard_loads(ctx.tolist(), shards)
    # Greedy LPT keeps every rank within one (the largest) sequence of the others.
    assert max(loads) - min(loads) <= int(ctx.max())
    assert max(loads) / (sum(loads) / world) < 1.001


def test_shards_are_deterministic_and_sorted() -> None:
    ctx = [5, 9, 9, 1, 30, 2]
    a = shard_by_tokens(ctx, 3)
    assert a == shard_by_tokens(ctx, 3)
    assert all(s == sorted(s) for s in a)


def _gather_worker(rank: int, world: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=30))
    try:
        ctx = list(np.random.default_rng(1).integers(1, 100, size=11))
        shards = shard_by_tokens(ctx, world)
        # Each rank "computes" one row per sequence it owns: a row that encodes the global index.
        local = torch.tensor([[i, 10 * i] for i in shards[rank]], dtype=torch.float32)
        out = gather_rows(local, shards, rank)
        expect = torch.tensor([[i, 10 * i] for i in range(len(ctx))], dtype=torch.float32)
        q.put((rank, bool(torch.equal(out, expect))))
    finally:
        torch.distributed.destroy_process_group()


def test_gather_rows_over_two_gloo_ranks() -> None:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    results = dict(q.get(timeout=5) for _ in range(2))
    assert results == {0: True, 1: True}
    assert all(p.exitcode == 0 for p in procs)


def _failing_worker(rank: int, world: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=10))
    torch.distributed.barrier()  # step 1 completes on both ranks
    if rank == 1:
        os._exit(3)  # rank 1 dies between steps, with nothing in flight
    try:
        local = torch.zeros(1, 2)
        gather_rows(local, [[0], [1]], rank)
        q.put((rank, "no error"))
    except Exception as exc:  # the survivor learns of it from the collective, not by hanging
        q.put((rank, type(exc).__name__))


def test_rank_dying_between_steps_is_reported_not_hung() -> None:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    assert procs[1].exitcode == 3
    rank, what = q.get(timeout=5)
    assert rank == 0 and what != "no error"
