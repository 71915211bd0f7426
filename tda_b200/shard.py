"""(batch x head) sharding of the TDA forward across the GPUs of one node.

Every (batch, head) slice is independent (triton_threshold_attention.py:40,374:
one program per flattened b*H + h), and tau depends only on the query position
inside the full sequence, so a rank that owns a contiguous block of flattened
heads computes its rows of the output with no communication.  The only
collectives are host-side plumbing: a barrier around timed regions and a MAX
reduction of per-rank times.
"""
from __future__ import annotations

import os
from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    start: int  # first flattened batch*head index owned by this rank
    stop: int   # one past the last

    @property
    def size(self) -> int:
        return self.stop - self.start


def shard_range(total: int, world: int, rank: int) -> Shard:
    """Contiguous, balanced split of ``total`` units over ``world`` ranks (the
    first ``total % world`` ranks get one extra unit)."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return Shard(rank, world, start, stop)


def env_rank_world() -> tuple[int, int, int]:
    """(rank, local_rank, world_size) from the torchrun environment (1 process
    = rank 0 of 1 when unset)."""
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    return rank, local, world


def max_over_ranks(value: float, device=None) -> float:
    """MAX of a per-rank float over the default process group (identity when
    torch.distributed is not initialised)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, device=None) -> float:
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())
