"""World-size-2 gloo test of the replica layout's host logic (batch sharding,
MAX-over-ranks timing, SUM of processed units), run as two CPU processes."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from torchplusplus_b200 import replicas


def test_shard_covers_batch_exactly():
    for total in (0, 1, 7, 32, 33, 64):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                s, n = replicas.shard(total, r, world)
                seen.extend(range(s, s + n))
            assert seen == list(range(total))
    with pytest.raises(ValueError):
        replicas.shard(4, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        start, count = replicas.shard(33, rank, world)
        # each rank "times" its slice; the job time is the slowest rank's
        t = replicas.max_over_ranks(0.5 + rank, world)
        units = replicas.sum_over_ranks(count, world)
        out[rank] = torch.tensor([start, count, t, units], dtype=torch.float64)
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_timing_and_units():
    world = 2
    out = torch.zeros(world, 4, dtype=torch.float64).share_memory_()
    mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    (s0, c0, t0, u0), (s1, c1, t1, u1) = out.tolist()
    assert (s0, c0, s1, c1) == (0, 17, 17, 16)
    assert t0 == t1 == 1.5          # MAX over ranks
    assert u0 == u1 == 33           # every sequence counted once
