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
