"""One process per GPU: which streams a rank decodes, and how the ranks' round timings combine.

Independent streams shard with no collective on the data path (the reference runs one process
per GPU, scripts/launch_ddp.sh:9-33).  The only collectives are on the host side of the bench:
the device time of a timed region is the slowest rank's, and the emitted tokens add up.
"""

from __future__ import annotations


def stream_partition(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous block of streams [first, first + count) for ``rank`` of ``world`` (the first
    ``total % world`` ranks take one extra stream)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if total < 0:
        raise ValueError("total streams must be >= 0")
    base, extra = divmod(total, world)
    count = base + (1 if rank < extra else 0)
    first = rank * base + min(rank, extra)
    return first, count


def combine_timing(ms: float, tokens: float, device=None) -> tuple[float, float]:
    """(max over ranks of ``ms``, sum over ranks of ``tokens``); identity without a process group."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(ms), float(tokens)
    dev = device if device is not None else ("cuda" if dist.get_backend() == "nccl" else "cpu")
    t = torch.tensor([float(ms)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    a = torch.tensor([float(tokens)], dtype=torch.float64, device=dev)
    dist.all_reduce(a, op=dist.ReduceOp.SUM)
    return float(t.item()), float(a.item())


__all__ = ["combine_timing", "stream_partition"]
