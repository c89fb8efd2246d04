"""Expert-parallel helpers with the reference's signatures (spider_moe/expert_parallel.py:19-37).

Ownership is round-robin: rank ``r`` of ``world`` owns experts ``e`` with
``e % world == r`` (expert_parallel.py:29-30).  ``all_reduce_sum_`` is the
reference's in-place SUM all-reduce (a no-op without an initialised
multi-rank process group).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def ep_enabled() -> bool:
    return dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1


def get_rank_world() -> tuple[int, int]:
    if not ep_enabled():
        return 0, 1
    return dist.get_rank(), dist.get_world_size()


def owns_expert(expert_id: int, rank: int, world: int) -> bool:
    return expert_id % world == rank


def local_experts(num_experts: int, rank: int, world: int) -> list[int]:
    return [e for e in range(num_experts) if owns_expert(e, rank, world)]


def all_reduce_sum_(tensor: torch.Tensor) -> torch.Tensor:
    """In-place SUM all-reduce when EP is active; no-op otherwise."""
    if ep_enabled() and tensor.numel() > 0:
        dist.all_reduce(tensor, op=dist.ReduceOp.SUM)
    return tensor
