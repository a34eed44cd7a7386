"""Request-level sharding host logic on two gloo ranks (CPU): each rank owns
its own utterance, the timed value is the maximum over ranks and the job
rate counts every rank's frames.  No GPU and no data-path collective."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import shard


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    r, w, local = shard.dist_env()
    shard.init("gloo", local, timeout_s=60)
    try:
        utt = shard.utterance_for_rank(r)
        ms = 100.0 + 50.0 * r  # rank 1 is the slow one
        dist.barrier()
        mx = shard.max_over_ranks(ms, "cpu")
        rate = shard.aggregate_rate(w, 2, 200, mx)
        q.put((r, w, utt, mx, rate))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_sharding_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    seeds = {r[2]["prompt_seed"] for r in res}
    seq_ids = {r[2]["seq_id"] for r in res}
    assert len(seeds) == world and seq_ids == {0, 1}  # distinct utterances
    for r, w, utt, mx, rate in res:
        assert w == world
        assert mx == 150.0  # the slowest rank's time
        assert rate == pytest.approx(world * 2 * 200 / 0.150)


def test_single_process_identity():
    assert shard.max_over_ranks(3.5) == 3.5
    assert shard.aggregate_rate(1, 5, 200, 1000.0) == pytest.approx(1000.0)


def _leaver(rank: int, world: int, port: int, q) -> None:
    """Rank 1 takes part in step 1 and then leaves between steps (exits
    without joining step 2's barrier); rank 0 must learn of it from the
    process group's short timeout instead of waiting for good."""
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    shard.init("gloo", rank, timeout_s=3)
    dist.barrier()
    shard.max_over_ranks(1.0, "cpu")  # step 1: both ranks
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()  # the message is out before the process goes
        os._exit(0)  # no destroy_process_group: the rank is simply gone
    t0 = time.monotonic()
    try:
        dist.barrier()  # step 2: its peer never comes
        q.put((rank, "no error"))
    except Exception as e:  # the timeout (or the peer's closed connection) ends the wait
        q.put((rank, f"error after {time.monotonic() - t0:.1f} s: {type(e).__name__}"))
    q.close()
    q.join_thread()
    os._exit(0)


def test_rank_leaving_between_steps_is_detected():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaver, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res = dict(q.get(timeout=10) for _ in range(world))
    assert res[1] == "left"
    assert res[0].startswith("error after"), res[0]
    assert float(res[0].split()[2]) < 30.0
