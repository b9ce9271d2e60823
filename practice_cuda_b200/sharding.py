"""Work partitioning for the multi-GPU configs.

BASELINE cfg3 shards the 32 BMM batches and cfg4 the activation rows across
ranks; each shard is independent, so the data path has no collective.  The
reference has no sharded BMM; these helpers define the split every rank
computes locally (balanced contiguous ranges), and an optional gather used
only to validate results.
"""

from __future__ import annotations

import torch


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, end) of ``total`` items for ``rank`` of ``world``;
    the first ``total % world`` ranks take one extra item."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank/world: {rank}/{world}")
    if total < 0:
        raise ValueError(f"total must be >= 0, got {total}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_sizes(total: int, world: int) -> list[int]:
    return [shard_range(total, r, world)[1] - shard_range(total, r, world)[0] for r in range(world)]


def gather_shards(local: torch.Tensor, total: int, group=None) -> torch.Tensor:
    """All-gather dim-0 shards produced with ``shard_range`` (validation only).

    Shards may differ in length by one; each is padded to the largest before
    ``all_gather_into_tensor`` and the padding is dropped afterwards.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    sizes = shard_sizes(total, world)
    cap = max(sizes)
    padded = torch.zeros((cap,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    padded[: local.shape[0]].copy_(local)
    full = torch.empty((cap * world,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(full, padded, group=group)
    parts = [full[r * cap: r * cap + sizes[r]] for r in range(world)]
    return torch.cat(parts, dim=0)
