"""The multi-GPU plumbing of bench.py on CPU: world-size-2 gloo ranks partition the requests (disjoint, complete,
balanced) and agree on the max-over-ranks timing.  No data-path collective exists to test: requests are
independent."""
import datetime
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, ws, port, queue):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=60))
    try:
        import bench

        total = bench.TOTAL_REQUESTS
        prefixes = bench.prefix_lengths(total)
        reqs = bench.partition(total, ws, rank, prefixes)
        mx = bench.max_over_ranks(ws, float(10 + rank))
        parts = [None] * ws
        dist.all_gather_object(parts, reqs)
        queue.put((rank, mx, parts, prefixes))
    finally:
        dist.destroy_process_group()


def test_two_rank_partition_and_timing_reduce():
    ws = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, ws, port, queue)) for r in range(ws)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in range(ws)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, mx, parts, prefixes in results:
        assert mx == 10.0 + ws - 1  # every rank sees the slowest rank's time
        flat = [r for part in parts for r in part]
        assert sorted(flat) == list(range(len(prefixes)))  # disjoint and complete
        assert len({len(part) for part in parts}) == 1  # same count per rank
        work = [sum(prefixes[r] for r in part) for part in parts]
        assert max(work) / min(work) < 1.05  # attention work balanced by prefix length
    # a request's prefix does not depend on the job size (inputs are seeded per request id)
    import bench
    assert bench.prefix_lengths(32) == bench.prefix_lengths(256)[:32]
