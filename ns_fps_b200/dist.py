"""Whole-cloud sharding across ranks (one process per GPU).

Farthest-point iterations are sequential inside a cloud, so a batch shards
only by cloud: rank r of W takes clouds r, r + W, r + 2W, ...  No collective
touches the sampling path; torch.distributed is used only to agree on timings
(max over ranks) and to line ranks up before and after a timed region.
"""
from __future__ import annotations

import os
from datetime import timedelta
from typing import List, Sequence


def shard_indices(count: int, rank: int, world: int) -> List[int]:
    """Cloud indices owned by `rank` (round-robin, whole clouds)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    return list(range(rank, count, world))


def env_rank():
    """(rank, local_rank, world) from the torchrun environment (0, 0, 1 alone)."""
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def init(backend: str, timeout_s: float = 120.0):
    """Initialise the default process group when WORLD_SIZE > 1."""
    import torch.distributed as dist
    _, _, world = env_rank()
    if world > 1 and not dist.is_initialized():
        dist.init_process_group(backend=backend, timeout=timedelta(seconds=timeout_s))
    return world


def max_over_ranks(values: Sequence[float], device=None) -> List[float]:
    """Element-wise max of `values` over all ranks (identity when alone)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return [float(v) for v in values]
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.cpu().tolist()]


def sum_over_ranks(values: Sequence[float], device=None) -> List[float]:
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return [float(v) for v in values]
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return [float(v) for v in t.cpu().tolist()]


def barrier(device=None):
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        if device is not None and dist.get_backend() == "nccl":
            dist.barrier(device_ids=[device])
        else:
            dist.barrier()


def finalize():
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()
