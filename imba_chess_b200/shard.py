"""Partitioning independent games across GPUs (one process per GPU).

Games never interact, so the multi-GPU path has no data-path collective:
game ``i`` belongs to rank ``i % world_size`` - the same rule as the
reference's file/row sharding (src/imba_chess/data/sharding.py:8-17) and its
round-robin worker assignment (scripts/eval_vs_stockfish.py:1178).  Each rank
owns one model copy, one KV pool and one stream.  ``torch.distributed`` is
used only around measurements: a barrier, and reductions of counts and
elapsed times (max over ranks).
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist


def dist_env() -> tuple[int, int, int]:
    """(world_size, rank, local_rank) from the torchrun environment."""
    return int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0"))


def shard_games(num_games: int, rank: int, world_size: int) -> list[int]:
    """Game indices owned by ``rank``: i with i % world_size == rank."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"bad rank {rank} for world size {world_size}")
    return list(range(rank, num_games, world_size))


def reduce_max(value: float, device: torch.device | None = None) -> float:
    """Max of a per-rank scalar over all ranks (identity without a process group)."""
    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def reduce_sum(value: float, device: torch.device | None = None) -> float:
    """Sum of a per-rank scalar over all ranks (identity without a process group)."""
    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())
