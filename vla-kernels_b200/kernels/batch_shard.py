"""Batch sharding of independent policy queries over the ranks of one node.

The attention and softmax ops have no cross-sample dependency, so a batch of
B queries is split into contiguous shards, one per rank (one process per GPU),
each rank runs the op on its shard, and the outputs are gathered once. This is
the only multi-GPU component of the hot path; the reference runs on a single
device and has none.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard(B: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous shard [lo, hi) of rank `rank`; the first B % world ranks
    take one extra element, so shards differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    if B < 0:
        raise ValueError(f"negative batch {B}")
    base, rem = divmod(B, world)
    lo = rank * base + min(rank, rem)
    return lo, lo + base + (1 if rank < rem else 0)


def gather(local: torch.Tensor, total: int, group=None) -> torch.Tensor:
    """All-gather of the per-rank shards (dim 0) into the full batch, in rank
    order. Equal shards on NCCL go through one all_gather_into_tensor; uneven
    shards (or gloo) are padded to the largest shard and trimmed."""
    world = dist.get_world_size(group)
    sizes = [shard(total, r, world) for r in range(world)]
    rank = dist.get_rank(group)
    lo, hi = sizes[rank]
    if local.shape[0] != hi - lo:
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, its shard is {hi - lo}")
    largest = max(h - l for l, h in sizes)
    equal = all(h - l == largest for l, h in sizes)
    if equal and dist.get_backend(group) == "nccl":
        out = local.new_empty((total,) + tuple(local.shape[1:]))
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
        return out
    padded = local.new_zeros((largest,) + tuple(local.shape[1:]))
    padded[: local.shape[0]] = local
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    return torch.cat([p[: h - l] for p, (l, h) in zip(parts, sizes)], dim=0)
