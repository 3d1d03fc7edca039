"""Tensor-parallel folded verify forward (the 14B configuration's scheme) on 2 GPUs:
each rank holds a head / intermediate shard, the o_proj and down partial sums are reduced
across the ranks -- by the consuming kernels reading every rank's partials over NVLink
("p2p", the default) or by NCCL all-reduces ("nccl") -- and every rank must return the
oracle's logits and fold masks (same tolerances as the single-GPU forward), identical on
both ranks.  Runs as two child processes, one per GPU; skipped with fewer than two GPUs.
The failure path (a partner that never arrives) is tested on one GPU: the bounded waits
end the forward with an error status instead of a hang."""
import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CASES = ["tiny_fp32_tree", "tiny_bf16_chain", "tiny_nld_fp32_tree"]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, ws, port, name, transport, out):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    from oracle import folded_oracle as orc
    from specfold_b200 import SpecFoldB200FastDLLMV2Generation, SpecFoldB200NLDGeneration
    from specfold_b200.synthetic import StandinExecutor
    from tests.golden.make_golden import build_case
    from tests.helpers import to_cuda_model
    from tests.test_gpu_forward import _check_against_oracle
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=ws,
                            timeout=datetime.timedelta(seconds=120))
    gen = None
    try:
        family, model, cache, ids, delta = build_case(name)
        cap = orc.Capture()
        with torch.no_grad():
            ref = orc.folded_forward(model, ids, cache, delta, family=family, capture=cap)
        cls = SpecFoldB200FastDLLMV2Generation if family == "fastdllm" else SpecFoldB200NLDGeneration
        gen = cls(model_executor=StandinExecutor(to_cuda_model(model)), delta=delta)
        gen.record_masks = True
        gen.set_tensor_parallel(rank, ws, transport=transport)
        cache_d = None if cache is None else cache.to("cuda")
        last = None
        for _ in range(3):     # direct, captured, replayed
            gen._fold_draft_positions = gen._fold_draft_recomputed = 0
            last = gen._batched_block_forward(ids.cuda(), cache_d)
            torch.cuda.synchronize()
            _check_against_oracle(f"{name} tp{ws} rank {rank}", ref, cap, last, gen)
        out[rank] = (last.cpu(), "ok")
    except Exception:   # reported to the parent
        import traceback
        out[rank] = (None, traceback.format_exc()[-1500:])
    finally:
        if gen is not None:
            gen.close_tensor_parallel()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("transport", ["p2p", "nccl"])
@pytest.mark.parametrize("name", CASES)
def test_tensor_parallel_two_ranks(name, transport):
    ws = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(ws, _free_port(), name, transport, out), nprocs=ws,
                       join=True, start_method="spawn")
    for r in range(ws):
        assert out[r][1] == "ok", f"rank {r}: {out[r][1]}"
    assert torch.equal(out[0][0], out[1][0]), "ranks disagree"


def test_peer_wait_times_out_with_status():
    """Failure detection of the peer-memory exchange, on one GPU and without a fault: rank
    0 of a two-rank peer table whose partner never runs.  Every reduction's handshake waits
    for a flag that nothing sets; the bounded wait (2 s) gives up, sets the timeout bit of
    the device error word and returns, so the forward ends with SpecFoldError and the
    context stays usable for the next forward."""
    import ctypes
    from specfold_b200 import SpecFoldB200FastDLLMV2Generation, _lib
    from specfold_b200.synthetic import (ModelDims, StandinExecutor, build_model,
                                         random_prefix_cache, tree_block_input)
    dims = ModelDims(hidden=512, heads=4, kv_heads=2, head_dim=128, inter=1024, layers=1,
                     vocab=256)
    model = build_model(dims, family="fastdllm", dtype=torch.bfloat16, seed=0, device="cuda")
    cache = random_prefix_cache(dims, 64, dtype=torch.bfloat16, seed=1, device="cuda")
    ids = tree_block_input(dims.vocab, N=32, edits_per_level=3).cuda()
    lib = _lib.load()
    nbytes = lib.sf_tp_exchange_bytes(256, dims.hidden)
    mine = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    absent = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")   # the partner's buffer
    peers = ctypes.c_void_p()
    _lib.check(lib.sf_tp_peers_init(0, 2, (ctypes.c_void_p * 2)(mine.data_ptr(), absent.data_ptr()),
                                    256, dims.hidden, ctypes.byref(peers)), "tp peer table")
    gen = SpecFoldB200FastDLLMV2Generation(model_executor=StandinExecutor(model), delta=0.1)
    gen._tp, gen._tp_transport = (0, 2, None), "p2p"
    gen._tp_peers, gen._tp_xbuf = peers.value, (mine, [])
    try:
        with pytest.raises(_lib.SpecFoldError, match="timed out"):
            gen._batched_block_forward(ids, cache)
            torch.cuda.synchronize()
    finally:
        gen.close_tensor_parallel()
    # the context is intact: a plain single-GPU forward still runs
    plain = SpecFoldB200FastDLLMV2Generation(model_executor=StandinExecutor(model), delta=0.1)
    out = plain._batched_block_forward(ids, cache)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
