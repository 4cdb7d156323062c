"""bench.py's multi-GPU decode line (replicas only: one independent decoder per rank, no
data-path collective): the timed region is the slowest rank's, and the whole-job throughput
counts every rank's tokens. Two gloo ranks on the CPU."""
import multiprocessing as mp
import os
import socket

import pytest


def _rank(rank, world, port, q):
    import torch.distributed as dist

    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ms, e2e = bench.slowest_rank(100.0 + 50.0 * rank, 0.5 - 0.2 * rank, dist)
    dist.destroy_process_group()
    q.put((rank, ms, e2e))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_ranks_report_the_slowest_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got == [(0, 150.0, 0.5), (1, 150.0, 0.5)]


def test_one_rank_needs_no_collective_and_throughput_counts_every_replica():
    import bench

    assert bench.slowest_rank(12.5, 0.25, None) == (12.5, 0.25)
    value, e2e = bench.replica_throughput(4, 100, 250.0, 0.5)
    assert value == pytest.approx(1600.0) and e2e == pytest.approx(800.0)
