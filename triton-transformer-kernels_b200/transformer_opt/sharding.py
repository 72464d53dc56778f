"""Batch sharding across GPUs (one process per GPU, no collective on the hot path).

Every operation of the inference forward is independent across sequences,
so a batch splits into contiguous per-rank slices with replicated weights.
NCCL (or gloo on CPU) is used only after the forward, to bring per-rank
validation results to rank 0.
"""

from __future__ import annotations

from typing import List, Tuple

import torch
import torch.distributed as dist


def shard_range(total: int, world_size: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, stop) slice of `total` items for `rank`; sizes differ by at most 1."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError("rank must be in [0, world_size)")
    base, extra = divmod(total, world_size)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather_stats(values: List[float], device: torch.device) -> List[List[float]]:
    """All-gather a short list of floats from every rank (validation only)."""
    local = torch.tensor(values, dtype=torch.float64, device=device)
    if not dist.is_available() or not dist.is_initialized():
        return [local.tolist()]
    out = [torch.empty_like(local) for _ in range(dist.get_world_size())]
    dist.all_gather(out, local)
    return [t.tolist() for t in out]


def max_over_ranks(value: float, device: torch.device) -> float:
    """Maximum of a scalar over all ranks (identity without a process group)."""
    if not dist.is_available() or not dist.is_initialized():
        return float(value)
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
