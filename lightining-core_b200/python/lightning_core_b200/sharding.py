"""Sharding of the hot path across ranks (one process per GPU).

Attention shards by independent (batch, head) units, the GEMM by row-blocks of A (B replicated),
the conv->attention pipeline by image: no rank needs another rank's data while computing, so
the only collective is the all-gather that assembles the outputs (NCCL over NVLink on GPUs,
gloo in the CPU tests).  Shards are contiguous and balanced (sizes differ by at most one unit).
"""
from __future__ import annotations


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [lo, hi) of `total` units owned by `rank` out of `world` (balanced)."""
    if world < 1 or not 0 <= rank < world or total < 0:
        raise ValueError("bad shard request")
    base, extra = divmod(total, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def assemble(local, total: int, rank: int, world: int, group=None):
    """All-gather the per-rank shards (leading dim) into the full [total, ...] tensor on every rank.

    Shards may be uneven, so each is padded to the largest shard before the collective and the
    padding is dropped afterwards.  `local` is a torch tensor on the process group's device.
    """
    import torch
    import torch.distributed as dist

    lo, hi = shard_range(total, rank, world)
    if local.shape[0] != hi - lo:
        raise ValueError(f"rank {rank}: shard has {local.shape[0]} rows, expected {hi - lo}")
    if world == 1:
        return local
    most = shard_range(total, 0, world)[1]  # rank 0 always holds a largest shard
    padded = local
    if local.shape[0] < most:
        pad = torch.zeros((most - local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
        padded = torch.cat([local, pad])
    gathered = torch.empty((world * most,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    if hasattr(dist, "all_gather_into_tensor") and local.device.type == "cuda":
        dist.all_gather_into_tensor(gathered, padded.contiguous(), group=group)
    else:
        parts = list(gathered.chunk(world))
        dist.all_gather(parts, padded.contiguous(), group=group)
        gathered = torch.cat(parts)
    pieces = []
    for r in range(world):
        a, b = shard_range(total, r, world)
        pieces.append(gathered[r * most: r * most + (b - a)])
    return torch.cat(pieces)
