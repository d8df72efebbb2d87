"""Shot sharding over the GPUs of one node: independent shots, no collective on the data path."""
from __future__ import annotations


def shard(total: int, world: int, rank: int) -> tuple[int, int]:
    """(start, count) of rank `rank` when `total` shots are split over `world` ranks as evenly as possible."""
    if world < 1 or not 0 <= rank < world or total < 0:
        raise ValueError("bad shard request")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)
