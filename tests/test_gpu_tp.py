"""Tensor-parallel folded verify forward (the 14B configuration's scheme) on 2 GPUs:
each rank holds a head / intermediate shard, the o_proj and down partial sums are reduced
across the ranks -- by the consuming kernels reading every rank's partials over NVLink
("p2p", the default) or by NCCL all-reduces ("nccl") -- and every rank must return the
oracle's logits and fold masks (same tolerances as the single-GPU forward), identical on
both ranks.  Runs as two child processes, one per GPU; skipped with fewer than two GPUs."""
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
