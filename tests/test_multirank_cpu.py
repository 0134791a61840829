"""The bench's multi-rank host logic on two gloo ranks (CPU): every rank takes the same collective
steps, the timed value is the max over ranks, per-rank inputs differ, and the whole-job rate
counts every rank's units over the slowest rank's time."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        barrier, max_over_ranks = bench.make_collectives(dist, world, "cpu")
        barrier()
        ms = 10.0 + 5.0 * rank  # rank 1 is the slow one
        worst = max_over_ranks(ms)
        barrier()
        out[rank] = (worst, bench.rank_seed(1, rank), bench.aggregate_rate(world, 128, worst))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_agree_on_the_slowest_time():
    world, port = 2, _free_port()
    with mp.get_context("spawn").Manager() as mgr:  # no fork: earlier tests leave threads running
        out = mgr.dict()
        mp.spawn(_rank, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    assert res[0][0] == res[1][0] == 15.0  # max over ranks, seen by both
    assert res[0][1] != res[1][1]  # each replica decodes its own sequences
    assert res[0][2] == res[1][2] == pytest.approx(2 * 128 / 15e-3)


def test_single_rank_needs_no_process_group():
    barrier, max_over_ranks = bench.make_collectives(None, 1, "cpu")
    barrier()
    assert max_over_ranks(3.5) == 3.5
    assert bench.aggregate_rate(1, 64, 32.0) == pytest.approx(2000.0)
