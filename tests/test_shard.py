"""Multi-rank host logic of the bench on CPU (gloo, world size 2): the
round-robin shards and the max-over-ranks timing reduction."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kokopop_b200.shard import period, rank_batch, rank_batches


def test_single_rank_covers_pool_in_batches():
    bs = rank_batches(256, 0, 1, 64)
    assert len(bs) == 4
    assert sorted(i for b in bs for i in b) == list(range(256))


def test_eight_ranks_keep_batch_64_and_are_disjoint_per_step():
    for step in range(3):
        seen = []
        for r in range(8):
            b = rank_batch(256, r, 8, 64, step)
            assert len(b) == 64 and len(set(b)) == 64
            seen += b
        # 8 x 64 = 512 = every utterance exactly twice per step
        assert sorted(seen) == sorted(list(range(256)) * 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = rank_batches(256, rank, world, 64)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        elapsed = torch.tensor([1.0 + rank], dtype=torch.float64)
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
        q.put((rank, gathered, float(elapsed)))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_shards_and_max_time():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, gathered, mx in res:
        assert mx == 2.0
        assert period(256, 2, 64) == len(gathered[0]) == 2
        all_idx = sorted(i for per_rank in gathered for b in per_rank for i in b)
        assert all_idx == list(range(256))
