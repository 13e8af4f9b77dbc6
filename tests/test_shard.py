"""Multi-process host logic of the sharded step (gloo, world size 2, CPU)."""

from __future__ import annotations

import os
import socket

import torch
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out) -> None:
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from bpdecode_b200 import shard
    from bpdecode_b200.workloads import row_patterns

    assert shard.init("gloo", timeout_s=60)
    rows = shard.shard_rows(10, world, rank)
    # per-rank work is independent: each rank draws its own rows' grammars
    pats = row_patterns(len(rows), seed=rank)
    elapsed = [1.5 + rank, 10.0 * rank]
    mx = shard.max_over_ranks(elapsed)
    tot = shard.sum_over_ranks([float(len(rows))])
    per = shard.gather_over_ranks(3.0 + rank)
    shard.barrier()
    out.put((rank, list(rows), len(pats), mx, tot, per))
    shard.finish()


def test_two_ranks_shard_rows_and_reduce_timings() -> None:
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    mp.start_processes(_worker, args=(world, _free_port(), q), nprocs=world, join=True,
                       start_method="spawn")
    got = sorted(q.get() for _ in range(world))
    assert got[0][1] == [0, 1, 2, 3, 4] and got[1][1] == [5, 6, 7, 8, 9]
    for _, _, n, mx, tot, per in got:
        assert n == 5
        assert mx == [2.5, 10.0]  # max over ranks of every entry
        assert tot == [10.0]
        assert per == [3.0, 4.0]  # every rank's value, in rank order


def test_single_process_is_identity() -> None:
    from bpdecode_b200 import shard

    assert shard.shard_rows(7, 1, 0) == range(0, 7)
    assert shard.shard_rows(7, 3, 2) == range(5, 7)
    assert shard.max_over_ranks([1.0, 2.0]) == [1.0, 2.0]
    assert torch.distributed.is_available()


def _lost_rank_worker(rank: int, world: int, port: int, out) -> None:
    """Rank 1 leaves between steps (before the barrier that closes the timed
    region); rank 0 must get an error from its next collective, not hang."""
    import time

    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from bpdecode_b200 import shard

    assert shard.init("gloo", timeout_s=5)
    shard.barrier()  # both ranks are up
    if rank == 1:
        os._exit(0)  # leaves without the group's next collective
    t0 = time.monotonic()
    try:
        shard.max_over_ranks([1.0])
        out.put((rank, "no error", time.monotonic() - t0))
    except Exception as exc:  # noqa: BLE001 -- any collective error is the signal
        out.put((rank, type(exc).__name__, time.monotonic() - t0))
    os._exit(0)


def test_lost_rank_ends_the_others_collective_with_an_error() -> None:
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    ctx_procs = mp.start_processes(_lost_rank_worker, args=(world, _free_port(), q),
                                   nprocs=world, join=False, start_method="spawn")
    rank, err, waited = q.get()
    for p in ctx_procs.processes:
        p.join(timeout=60)
    assert rank == 0 and err != "no error"
    assert waited < 30  # the short process-group timeout, not a hang
