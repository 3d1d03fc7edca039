"""Multi-process (world size 2, gloo, CPU) checks of the data-parallel bench plumbing:
every rank times its own replica of the verify stream, the job's time is the max over
ranks, the value is the whole-job rate, and the reference arm runs on rank 0 only."""

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


def _worker(rank, ws, port, out):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(ws), LOCAL_RANK=str(rank))
    import bench
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        assert bench.dist_env() == (ws, rank, rank)
        # rank r was slower by r ms on the first timing and faster on the second
        ms = bench.max_over_ranks([100.0 + rank, 50.0 - rank], "cpu")
        value = bench.weak_scaling_value(ws, 10, ms[0])
        # rank 0 alone runs the host-core reference arm; the others return at once
        ran = []

        class Args:
            steps, warmup = 1, 0
        orig = bench.CpuReference
        bench.CpuReference = lambda: ran.append(rank) or (_ for _ in ()).throw(RuntimeError("ran"))
        try:
            bench.run_reference(Args())
        except RuntimeError:
            pass
        finally:
            bench.CpuReference = orig
        dist.barrier()
        out[rank] = (ms, value, list(ran))
    finally:
        dist.destroy_process_group()


def test_two_rank_timing_reduction():
    ws = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(ws, _free_port(), out), nprocs=ws, join=True)
    for r in range(ws):
        ms, value, ran = out[r]
        assert ms == [101.0, 50.0]                       # max over ranks, per entry
        assert value == pytest.approx(ws * 10 / 0.101)   # whole-job verify steps per second
        assert ran == ([0] if r == 0 else [])


def test_single_process_is_identity():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.max_over_ranks([3.0, 4.0], "cpu") == [3.0, 4.0]
    assert bench.weak_scaling_value(1, 5, 500.0) == pytest.approx(10.0)
