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


class SegmentError(RuntimeError):
    """Raised on every rank when one or more segments failed on any rank.

    `failures` lists (segment index, rank, error text) in segment order.  A
    failing segment is reported, not fatal to the job's collective steps: the
    rank that hit it still joins the gather, so no rank waits for it until a
    process-group timeout (det-cli reports each failure as an error on
    stderr, crates/det-cli/src/main.rs:10-18)."""

    def __init__(self, failures):
        self.failures = sorted(failures)
        text = "; ".join(f"segment {i} on rank {r}: {e}" for i, r, e in self.failures)
        super().__init__(f"{len(self.failures)} segment(s) failed: {text}")


class _Failed:
    """A segment's result slot when its work raised (pickled by the gather)."""

    def __init__(self, rank: int, error: str):
        self.rank, self.error = rank, error


def run_local(segments: Sequence[bytes], rank: int, world_size: int,
              fn: Callable[[bytes], bytes]) -> dict[int, object]:
    """Apply `fn` (e.g. compress with this rank's model) to this rank's
    segments.  A segment whose `fn` raises is recorded as failed, and the
    other segments still run; `gather` reports the failures."""
    out: dict[int, object] = {}
    for i in my_segments(len(segments), rank, world_size):
        try:
            out[i] = fn(segments[i])
        except Exception as e:  # reported by gather on every rank
            out[i] = _Failed(rank, f"{type(e).__name__}: {e}")
    return out


def _check(merged: dict, n_segments: int):
    failures = [(i, v.rank, v.error) for i, v in merged.items() if isinstance(v, _Failed)]
    if failures:
        raise SegmentError(failures)
    if sorted(merged) != list(range(n_segments)):
        raise RuntimeError("segments missing after gather")


def gather(local: dict, n_segments: int, world_size: int, dst: int = 0):
    """Collect every rank's results on rank `dst` in segment order (None
    elsewhere).  If any segment failed on any rank, every rank raises
    SegmentError after the same two collective steps (the gather, then a
    broadcast of the failure list), so the ranks stay in step."""
    if world_size == 1:
        _check(local, n_segments)
        return [local[i] for i in range(n_segments)]
    import torch.distributed as dist

    rank = dist.get_rank()
    parts = [None] * world_size if rank == dst else None
    dist.gather_object(local, parts, dst=dst)
    status = [None]
    merged: dict[int, object] = {}
    if rank == dst:
        for p in parts:
            merged.update(p)
        try:
            _check(merged, n_segments)
        except SegmentError as e:
            status[0] = e.failures
        except RuntimeError as e:
            status[0] = [(-1, dst, str(e))]
    dist.broadcast_object_list(status, src=dst)
    if status[0]:
        raise SegmentError(status[0])
    if rank != dst:
        return None
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
