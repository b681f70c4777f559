"""World-size-2 tests of the multi-process plumbing on CPU (gloo): the stream shards of the
ranks, the max-over-ranks timing, and a rank that dies without hanging its peer. The GPU path
shards streams across ranks with no data-path collective; these are the host-side pieces."""
from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch.multiprocessing as mp


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    import sys
    import torch
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
    try:
        if mode == "shards":
            mine = torch.tensor(bench.shard_streams(rank, world))
            got = [torch.zeros_like(mine) for _ in range(world)]
            dist.all_gather(got, mine)
            bench.barrier(dist)
            slowest = bench.max_over_ranks(dist, 10.0 + rank)
            each = bench.gather_over_ranks(dist, 10.0 + rank)
            q.put((rank, sorted(torch.cat(got).tolist()), slowest, each))
        elif mode == "dead_peer":
            if rank == 1:
                os._exit(0)  # leaves between steps, nothing in flight
            try:
                bench.max_over_ranks(dist, 1.0)
                q.put((rank, "no error"))
            except Exception as e:  # the collective ends with an error instead of hanging
                q.put((rank, type(e).__name__))
    finally:
        if mode != "dead_peer":
            dist.destroy_process_group()


def _run(mode, world=2, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = []
    for p in procs:
        p.join(timeout)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail(f"rank {p.pid} hung")
    while not q.empty():
        out.append(q.get())
    return out


def test_ranks_own_disjoint_contiguous_shards_and_time_is_the_slowest_rank():
    res = _run("shards")
    assert len(res) == 2
    for rank, all_ids, slowest, each in res:
        assert all_ids == list(range(2 * 512))
        assert slowest == 11.0
        assert each == [10.0, 11.0]


def test_a_rank_that_leaves_does_not_hang_its_peer():
    res = _run("dead_peer")
    assert [r for r in res if r[0] == 0][0][1] != "no error"


def test_timed_frames_sit_in_the_middle_of_the_window():
    """K < 250 timed frames are centred in config 5's 250-frame window (the window's average KV
    read), with the warm-up frames just before them; K >= 250 cycle the window from frame 0."""
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    assert bench.timing_window(20, 5) == (110, 115)
    w0, t0 = bench.timing_window(20, 5)
    assert t0 + 20 / 2 == bench.FRAMES / 2
    assert bench.timing_window(248, 5) == (0, 1)
    assert bench.timing_window(250, 5) == (0, 5)
    assert bench.timing_window(1000, 3) == (0, 3)
    assert bench.spread([3.0, 1.0, 2.0]) == {"min": 1.0, "median": 2.0, "max": 3.0}


def test_more_ranks_than_streams_is_refused():
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    with pytest.raises(ValueError):
        bench.shard_streams(8, 9)
