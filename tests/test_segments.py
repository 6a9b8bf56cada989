"""Host logic of the multi-GPU segment mode, on CPU with torch.distributed
(gloo, world size 2): segment split and assignment, the ordered gather of
finished files, and the max-over-ranks timing reduction.  The per-segment
work is a stand-in function here; on GPUs it is `compress` on each rank's
model replica, whose output does not depend on the rank."""
import hashlib
import os
import socket
import time

import pytest
import torch.multiprocessing as mp

from detllm_b200 import segments as G


def test_split_stream_covers_input_in_order():
    data = bytes(range(256)) * 7 + b"tail"
    for n in (1, 2, 3, 8, 13):
        parts = G.split_stream(data, n)
        assert len(parts) == n
        assert b"".join(parts) == data
        assert max(map(len, parts)) - min(map(len, parts)) <= 1
    assert G.split_stream(b"", 4) == [b""] * 4
    with pytest.raises(ValueError):
        G.split_stream(b"x", 0)


def test_round_robin_assignment_is_a_partition():
    for ws in (1, 2, 4, 8):
        for n in (1, 5, 8, 17):
            got = sorted(i for r in range(ws) for i in G.my_segments(n, r, ws))
            assert got == list(range(n))
    with pytest.raises(ValueError):
        G.my_segments(4, 2, 2)


def _stand_in(seg: bytes) -> bytes:
    return hashlib.sha256(seg).digest() + seg[:3]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, ws, port, data, n, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        segs = G.split_stream(data, n)
        local = G.run_local(segs, rank, ws, _stand_in)
        assert sorted(local) == G.my_segments(n, rank, ws)
        files = G.gather(local, n, ws)
        slowest = G.max_over_ranks(1.0 + rank, ws)
        q.put((rank, files, slowest))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_rank_gather_matches_one_rank():
    data = os.urandom(10_001)
    n = 5
    want = [_stand_in(s) for s in G.split_stream(data, n)]
    assert G.gather(G.run_local(G.split_stream(data, n), 0, 1, _stand_in), n, 1) == want
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, data, n, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, files, slowest = q.get(timeout=100)
        res[rank] = (files, slowest)
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    assert res[0][0] == want  # rank 0 holds every file, in segment order
    assert res[1][0] is None
    assert res[0][1] == res[1][1] == 2.0  # the slowest rank's time


def _failing_stand_in(seg: bytes) -> bytes:
    if seg[:1] == b"\xff":
        raise ValueError("corrupt segment")
    return _stand_in(seg)


def _failing_worker(rank, ws, port, data, n, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        segs = G.split_stream(data, n)
        local = G.run_local(segs, rank, ws, _failing_stand_in)
        try:
            G.gather(local, n, ws)
            q.put((rank, None))
        except G.SegmentError as e:
            q.put((rank, e.failures))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_failing_segment_is_reported_on_every_rank():
    """A segment whose compress raises on rank 1 is reported by gather on
    both ranks (segment index, rank and error text), after the same
    collective steps, instead of leaving rank 0 blocked in the gather."""
    n = 4
    segs = [b"a" * 10, b"\xff" * 10, b"c" * 10, b"d" * 10]  # segment 1 -> rank 1 of 2
    data = b"".join(segs)
    with pytest.raises(G.SegmentError) as e:
        G.gather(G.run_local(segs, 0, 1, _failing_stand_in), n, 1)
    assert e.value.failures == [(1, 0, "ValueError: corrupt segment")]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, data, n, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=100) for _ in range(2))
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    assert res[0] == res[1] == [(1, 1, "ValueError: corrupt segment")]


def _leaving_worker(rank, ws, port, q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves between steps, without joining the gather
    t = time.time()
    try:
        G.gather({0: b"x"}, 2, ws)
        q.put(("returned", time.time() - t))
    except Exception as e:  # the missing peer surfaces as an error on rank 0
        q.put((type(e).__name__, time.time() - t))
    os._exit(0)


@pytest.mark.timeout(120)
def test_rank_that_leaves_ends_the_gather_with_an_error():
    """A rank that exits without joining the gather: rank 0's gather ends
    with an error within the process group's short timeout, not a hang."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    what, waited = q.get(timeout=100)
    for p in procs:
        p.join(timeout=30)
    assert what != "returned"
    assert waited < 60
