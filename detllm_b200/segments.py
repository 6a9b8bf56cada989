"""Segment-parallel compression across GPUs (one model replica per GPU).

A long byte stream is split into independent segments; each segment is a
complete compress stream with its own window state and its own DTLZ file,
so every segment's bytes are exactly those a single GPU would produce for
it.  Segments are dealt round-robin to the ranks of a torch.distributed job
(one process per GPU); the data path has no collective -- only the final
gather of the finished files and the timing reduction talk to other ranks.
"""
from __future__ import annotations

from typing import Callable, Sequence


def split_stream(data: bytes, n: int) -> list[bytes]:
    """`data` cut into `n` contiguous segments whose lengths differ by at most one."""
    if n <= 0:
        raise ValueError("n must be positive")
    q, r = divmod(len(data), n)
    out, off = [], 0
    for i in range(n):
        ln = q + (1 if i < r else 0)
        out.append(data[off:off + ln])
        off += ln
    return out


def my_segments(n_segments: int, rank: int, world_size: int) -> list[int]:
    """Indices of the segments rank `rank` encodes (round-robin)."""
    if not 0 <= rank < world_size:
        raise ValueError("rank out of range")
    return list(range(rank, n_segments, world_size))


def run_local(segments: Sequence[bytes], rank: int, world_size: int,
              fn: Callable[[bytes], bytes]) -> dict[int, bytes]:
    """Apply `fn` (e.g. compress with this rank's model) to this rank's segments."""
    return {i: fn(segments[i]) for i in my_segments(len(segments), rank, world_size)}


def gather(local: dict[int, bytes], n_segments: int, world_size: int, dst: int = 0):
    """Collect every rank's results on rank `dst` in segment order (None elsewhere)."""
    if world_size == 1:
        return [local[i] for i in range(n_segments)]
    import torch.distributed as dist

    rank = dist.get_rank()
    parts = [None] * world_size if rank == dst else None
    dist.gather_object(local, parts, dst=dst)
    if rank != dst:
        return None
    merged: dict[int, bytes] = {}
    for p in parts:
        merged.update(p)
    if sorted(merged) != list(range(n_segments)):
        raise RuntimeError("segments missing after gather")
    return [merged[i] for i in range(n_segments)]


def max_over_ranks(x: float, world_size: int, device=None) -> float:
    """The maximum of `x` over all ranks (times are reported as the slowest rank)."""
    if world_size == 1:
        return float(x)
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def compress_segments(model, data: bytes, n_segments: int, rank: int = 0, world_size: int = 1,
                      n_ctx: int = 0):
    """Compress `data` as `n_segments` independent DTLZ files, this rank's share
    on this rank's model; rank 0 returns all files in order."""
    from . import compress

    segs = split_stream(data, n_segments)
    local = run_local(segs, rank, world_size, lambda s: compress(model, s, n_ctx))
    return gather(local, n_segments, world_size)


def decompress_segments(model, files: Sequence[bytes]) -> bytes:
    """Concatenation of the decompressed segments."""
    from . import decompress

    return b"".join(decompress(model, f) for f in files)
