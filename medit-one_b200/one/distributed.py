"""Sequence-sharded data parallelism for decode.

Sequences are independent (no op of One.forward mixes sequences, one/modeling_one.py:
325-590), so a global batch is split into contiguous per-rank shards; each rank runs its own
engine on its shard with no collective on the step path. Collectives appear only outside the
step loop: the max of the ranks' step times (timing) and the gather of generated tokens.
One process per GPU; the process group is torch.distributed (NCCL on GPUs, gloo on CPU).
"""
from __future__ import annotations

from typing import Tuple

import torch
import torch.distributed as dist


def shard(global_batch: int, world: int, rank: int) -> Tuple[int, int]:
    """(first sequence, count) of this rank's contiguous shard; the first
    `global_batch % world` ranks take one extra sequence."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world / rank")
    base, extra = divmod(global_batch, world)
    count = base + (1 if rank < extra else 0)
    start = rank * base + min(rank, extra)
    return start, count


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank scalar (the slowest rank's time)."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_tokens(local: torch.Tensor, global_batch: int) -> torch.Tensor:
    """Concatenate every rank's [count, steps] token block along the batch (rank order) on
    every rank. Shards may differ by one sequence: blocks are padded to the largest shard
    for the collective and trimmed after."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return local
    world = dist.get_world_size()
    counts = [shard(global_batch, world, r)[1] for r in range(world)]
    width = local.shape[1]
    padded = torch.zeros((max(counts), width), dtype=local.dtype, device=local.device)
    padded[: local.shape[0]] = local
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded)
    return torch.cat([p[:c] for p, c in zip(parts, counts)], dim=0)
