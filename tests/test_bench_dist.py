"""CPU: bench.py's multi-rank path (one process per GPU under torchrun) -- the barrier, the max over ranks of the
step time and the whole-job throughput -- run as two gloo ranks on 127.0.0.1."""
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, times, out):
    sys.path.insert(0, ROOT)
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        bench.dist_barrier(dist, device="cpu")
        ms = bench.max_over_ranks(times[rank], dist, device="cpu")
        acc = bench.config4_draws(rank, world, 16, 64)
        total = bench.sum_over_ranks(float(acc.sum()), dist, device="cpu")
        out[rank] = (ms, bench.job_rows_per_s(world, ms), acc.shape, total)
        bench.dist_barrier(dist, device="cpu")
    finally:
        dist.destroy_process_group()


def test_two_ranks_agree_on_the_slowest_step():
    world, times = 2, [4.0, 5.5]
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_rank, args=(world, _free_port(), times, out), nprocs=world, join=True)
        res = dict(out)
    everyone = float(bench_module().acceptance_draws(16 * 64).sum())
    for r in (0, 1):   # config 4: each rank its 32 sequences' draws, the job's sum the same as one GPU's
        assert res[r][:2] == (5.5, pytest.approx(2 * 8 / 5.5e-3))
        assert res[r][2] == (16, 32) and res[r][3] == everyone


def bench_module():
    sys.path.insert(0, ROOT)
    import bench
    return bench


def test_one_rank_needs_no_process_group():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.max_over_ranks(3.25, None, device="cpu") == 3.25
    assert bench.job_rows_per_s(1, 4.0) == pytest.approx(2000.0)
