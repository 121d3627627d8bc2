"""Multi-GPU layout of the decode path: independent replicas, one process
per GPU, the global batch sharded across ranks.

A decode step has no exchange between sequences (each sequence reads only its
own KV cache), so the path shards with no data-path collective: every rank
runs the whole model on its slice of the batch, and the only communication is
host-side bookkeeping (a barrier around timed regions and a MAX of the
per-rank device times).  The reference serves one process on one GPU
(torchpp/llmops/llm.py:20-40); scaling by replicas is this package's own
layout, not a reference feature.
"""
from __future__ import annotations

import torch


def shard(total: int, rank: int, world: int) -> tuple[int, int]:
    """(start, count) of rank's contiguous slice of `total` sequences; the
    first total % world ranks take one extra."""
    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError("need 0 <= rank < world and total >= 0")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def max_over_ranks(x: float, world: int, device: torch.device | str = "cpu") -> float:
    """MAX of a per-rank scalar (e.g. seconds of device time) over the
    default process group; `device` must suit the group's backend (cuda for
    NCCL, cpu for gloo)."""
    if world == 1:
        return float(x)
    import torch.distributed as dist
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int, device: torch.device | str = "cpu") -> float:
    """SUM of a per-rank scalar (e.g. tokens processed)."""
    if world == 1:
        return float(x)
    import torch.distributed as dist
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())
