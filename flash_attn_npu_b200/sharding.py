"""(batch, head) sharding for multi-GPU runs.

Attention is independent per (b, h) slice, so a multi-GPU run partitions the flattened index
`b * H + h` into contiguous, near-equal ranges, one per rank, and runs the kernel on each
range with no communication on the hot path.  Outputs are gathered to rank 0 only after the
timed region, for verification.
"""
from __future__ import annotations

import torch


def shard_range(n_slices: int, world_size: int, rank: int) -> tuple[int, int]:
    """[start, stop) of the flattened (b*H + h) slices owned by `rank`.

    The first `n_slices % world_size` ranks get one extra slice.
    """
    if world_size <= 0 or not (0 <= rank < world_size):
        raise ValueError("bad rank / world size")
    base, extra = divmod(n_slices, world_size)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return start, stop


def shard_counts(n_slices: int, world_size: int) -> list[int]:
    return [b - a for a, b in (shard_range(n_slices, world_size, r) for r in range(world_size))]


def take_shard(t: torch.Tensor, world_size: int, rank: int) -> torch.Tensor:
    """Rank's slices of a [B, H, S, ...] tensor, as [n_local, 1, S, ...] (a view when possible)."""
    b, h = t.shape[0], t.shape[1]
    start, stop = shard_range(b * h, world_size, rank)
    flat = t.reshape(b * h, 1, *t.shape[2:])
    return flat[start:stop]


def gather_shards(local: torch.Tensor, n_slices: int, world_size: int, rank: int, group=None,
                  dst: int = 0):
    """Collect every rank's [n_local, ...] shard on `dst`; returns the [n_slices, ...] tensor
    there and None elsewhere.  Uses point-to-point sends, so unequal shard sizes are fine.
    """
    import torch.distributed as dist

    counts = shard_counts(n_slices, world_size)
    if rank != dst:
        if local.shape[0] > 0:
            dist.send(local.contiguous(), dst=dst, group=group)
        return None
    out = torch.empty((n_slices, *local.shape[1:]), dtype=local.dtype, device=local.device)
    for r in range(world_size):
        a, b = shard_range(n_slices, world_size, r)
        if r == dst:
            out[a:b].copy_(local)
        elif counts[r] > 0:
            buf = torch.empty((counts[r], *local.shape[1:]), dtype=local.dtype,
                              device=local.device)
            dist.recv(buf, src=r, group=group)
            out[a:b].copy_(buf)
    return out
