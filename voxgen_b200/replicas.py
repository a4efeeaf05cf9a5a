"""Replica plumbing for multi-GPU decode: one process per GPU, each holding a full copy of the
weights and decoding its own streams. A batch-1 BaseLM decode step does not shard, so there is no
collective on the data path; the process group carries only a start barrier and the max over
ranks of each rank's device-timed duration (the job's wall time is the slowest replica's).

The functions take the process group (None for a single process) and work with either backend:
NCCL with CUDA tensors on a GPU box, gloo with CPU tensors in tests.
"""
from __future__ import annotations

import os
from datetime import timedelta
from typing import List, Optional, Sequence, Tuple


def env() -> Tuple[int, int, int]:
    """(rank, world size, local rank) from the torchrun environment; (0, 1, 0) without it."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def init(backend: str, world: int, timeout_s: float = 600.0, device=None):
    """Joins the default process group when world > 1 and returns it (None otherwise). The
    rendezvous comes from MASTER_ADDR / MASTER_PORT (use 127.0.0.1 on one node)."""
    if world <= 1:
        return None
    import torch.distributed as dist
    kw = {"timeout": timedelta(seconds=timeout_s)}
    if device is not None and backend == "nccl":
        kw["device_id"] = device
    dist.init_process_group(backend, **kw)
    return dist.group.WORLD


def barrier(pg) -> None:
    if pg is not None:
        import torch.distributed as dist
        dist.barrier(group=pg)


def max_over_ranks(value: float, pg, device=None) -> float:
    """The largest `value` over all ranks (every rank gets it)."""
    if pg is None:
        return float(value)
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=pg)
    return float(t.item())


def aggregate_rate(units_per_rank: int, world: int, max_ms: float) -> float:
    """Whole-job units per second: every rank processed units_per_rank units, and the job took
    as long as the slowest rank (max_ms)."""
    return world * units_per_rank / (max_ms / 1e3)


def shard(items: Sequence, rank: int, world: int) -> List:
    """This rank's share of independent work items (streams): items[rank::world]."""
    return list(items[rank::world])


def shutdown(pg) -> None:
    if pg is not None:
        import torch.distributed as dist
        dist.destroy_process_group()
