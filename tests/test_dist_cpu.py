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


def _shard_worker(rank, ws, port, out):
    """Each rank computes its shard's partial o_proj and FFN for one fp32 layer; the sums
    over ranks (gloo all-reduce) must equal the unsharded layer."""
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.nn.functional as F
    from specfold_b200.folded import FoldedVerifyB200
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        g = torch.Generator().manual_seed(0)
        D, H, Hkv, hd, I, R = 64, 4, 2, 16, 96, 5
        w = {n: torch.randn(*sh, generator=g) for n, sh in {
            "q": (H * hd, D), "k": (Hkv * hd, D), "v": (Hkv * hd, D), "o": (D, H * hd),
            "g": (I, D), "u": (I, D), "d": (D, I)}.items()}
        b = {n: torch.randn(w[n].shape[0], generator=g) for n in "qkv"}
        x = torch.randn(R, D, generator=g)
        attn = torch.randn(R, H * hd, generator=g)
        wqkv, bqkv, wo, wg, wu, wd = FoldedVerifyB200.tp_shard(
            w["q"], w["k"], w["v"], b["q"], b["k"], b["v"], w["o"], w["g"], w["u"], w["d"],
            H, Hkv, rank, ws)
        hq = H // ws
        # this rank's q/k/v columns are the matching slices of the full projection
        full = torch.cat([x @ w["q"].T + b["q"], x @ w["k"].T + b["k"], x @ w["v"].T + b["v"]], 1)
        mine = x @ wqkv.T + bqkv
        qd, kd = H * hd, Hkv * hd
        want = torch.cat([full[:, rank * hq * hd:(rank + 1) * hq * hd],
                          full[:, qd + rank * (kd // ws):qd + (rank + 1) * (kd // ws)],
                          full[:, qd + kd + rank * (kd // ws):qd + kd + (rank + 1) * (kd // ws)]], 1)
        ok_qkv = torch.allclose(mine, want, atol=1e-5)
        # row-parallel o_proj and FFN: partial sums add up to the full results
        part_o = attn[:, rank * hq * hd:(rank + 1) * hq * hd] @ wo.T
        part_f = (F.silu(x @ wg.T) * (x @ wu.T)) @ wd.T
        dist.all_reduce(part_o)
        dist.all_reduce(part_f)
        ok_o = torch.allclose(part_o, attn @ w["o"].T, atol=1e-4)
        ok_f = torch.allclose(part_f, (F.silu(x @ w["g"].T) * (x @ w["u"].T)) @ w["d"].T, atol=1e-3)
        out[rank] = (ok_qkv, ok_o, ok_f)
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_shards_sum_to_the_layer():
    ws = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_shard_worker, args=(ws, _free_port(), out), nprocs=ws, join=True)
    for r in range(ws):
        assert out[r] == (True, True, True), (r, out[r])
