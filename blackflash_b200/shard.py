"""B x H slice sharding over ranks (collective-free data parallelism).

Every (b, h) slice of attention is independent, so G GPUs each take a
contiguous range of the flattened B*H slices and run the same kernel on it.
No data crosses GPUs. The reference has no multi-GPU mode; this is the
partitioning BASELINE.json prescribes for configs 1-4.
"""
from __future__ import annotations


def slice_range(total_slices: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, stop) of the flattened B*H slices owned by `rank`.

    The first total % world ranks take one extra slice, so sizes differ by at most 1.
    """
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} for world size {world}")
    if total_slices < 0:
        raise ValueError("total_slices must be >= 0")
    base, extra = divmod(total_slices, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return start, stop


def shard_bh(t, world: int, rank: int):
    """View of this rank's slices of a [B, H, N, d] tensor as [S, 1, N, d] (S = its slice count)."""
    B, H = t.shape[0], t.shape[1]
    start, stop = slice_range(B * H, world, rank)
    return t.reshape(B * H, 1, *t.shape[2:])[start:stop]
