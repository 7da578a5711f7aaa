"""Batch sharding across GPUs of one node (one process per GPU, torch.distributed).

Every Cormorant kernel call is independent per batch item (per image, per
batched-GEMM slice; VectorOP per element range), so ranks take contiguous
shards and run with no communication.  Only when a caller needs the whole
output on every rank is it gathered, over NCCL (NVLink/NVSwitch) on GPUs or
gloo on CPU.
"""
from __future__ import annotations


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """(start, count) of rank's contiguous share of `total` items; shares differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    lo = total * rank // world
    hi = total * (rank + 1) // world
    return lo, hi - lo


def gather_batches(local, total: int, per_item: int, group=None):
    """All-gather rank shards of a [count * per_item] tensor into the full [total * per_item] tensor.

    Shards may differ in length by one item; they are padded to the largest shard for the
    collective and trimmed afterwards.  Returns the full tensor on every rank.
    """
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    counts = [shard_range(total, r, world)[1] for r in range(world)]
    cmax = max(counts)
    rank = dist.get_rank(group)
    if local.numel() != counts[rank] * per_item:
        raise ValueError(f"rank {rank}: expected {counts[rank] * per_item} words, got {local.numel()}")
    padded = torch.zeros(cmax * per_item, dtype=local.dtype, device=local.device)
    padded[: local.numel()] = local.reshape(-1)
    # neither NCCL nor gloo has an int16 type; an all-gather only moves bytes
    wire = padded.view(torch.uint8)
    parts = [torch.empty_like(wire) for _ in range(world)]
    dist.all_gather(parts, wire, group=group)
    return torch.cat([p.view(local.dtype)[: c * per_item] for p, c in zip(parts, counts)])
