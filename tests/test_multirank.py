"""World-size-2 `gloo` test of the multi-GPU host logic on CPU: every rank
derives its utterance shard independently (no data-path collective) and the
shards partition the job; the timing reduction is a max over ranks."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_pkg


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        load_pkg()
        import irodori_b200.synth as synth
        from irodori_b200 import sharding
        utts = synth.throughput_utterances(64, seed=4)
        costs = [sharding.utterance_cost(S, tl, rf) for tl, S, rf, _ in utts]
        mine = sharding.shard_for_rank(costs, rank, world)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        # bench.py's timing reduction: max over ranks
        t = torch.tensor([float(10 + rank)])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            q.put((gathered, float(t.item())))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_rank_sharding_and_max_timing():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()  # both ranks rendezvous on the same port
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    gathered, tmax = q.get(timeout=90)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    flat = sorted(i for shard in gathered for i in shard)
    assert flat == list(range(64))
    assert set(gathered[0]).isdisjoint(gathered[1])
    assert tmax == 11.0


def _failing_worker(rank, world, port, q):
    """Rank 1 raises right after joining (before the timing barrier); rank 0
    enters the bench's timing reduction and must get an error, not hang."""
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["RANK"] = str(rank)
    os.environ["WORLD_SIZE"] = str(world)
    load_pkg()
    from irodori_b200 import sharding
    d = sharding.init_rank_group("gloo", 5.0)
    if rank == 1:
        raise RuntimeError("injected worker failure before the timing barrier")
    t0 = time.monotonic()
    try:
        sharding.max_over_ranks(d, 12.5)
        q.put(("no error", time.monotonic() - t0))
    except Exception as e:  # the collective fails: the dead rank never joins
        q.put((type(e).__name__, time.monotonic() - t0))


@pytest.mark.timeout(120)
def test_rank_failure_before_barrier_does_not_hang():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    what, elapsed = q.get(timeout=90)
    for p in procs:
        p.join(timeout=60)
    assert what != "no error"
    assert elapsed < 30.0, elapsed
    assert procs[1].exitcode != 0  # the injected failure
    assert procs[0].exitcode == 0  # the survivor reported the error and left
