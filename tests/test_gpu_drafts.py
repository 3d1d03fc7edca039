"""GPU draft construction (sf_draft_blocks through the generators' get_draft_blocks)
against the CPU oracle, which the reference's own methods pin bit for bit on
tests/golden/drafts.pt: the same nodes kept, identical draft states."""
import os

import pytest
import torch

from oracle import drafts
from specfold_b200.folded import SpecFoldB200FastDLLMV2Generation, SpecFoldB200NLDGeneration
from tests.golden.make_draft_golden import GRAPH, case

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "drafts.pt")


def _gens(graph):
    f = SpecFoldB200FastDLLMV2Generation(model_executor=None)
    n = SpecFoldB200NLDGeneration(model_executor=None)
    f.calibration_graph = n.calibration_graph = graph
    return f, n


def _same(got, ref, nodes):
    assert [nodes.index(d["node"]) for d in got] == [nodes.index(d["node"]) for d in ref]
    for d, r in zip(got, ref):
        assert torch.equal(d["state"].cpu(), r["state"])


def test_drafts_match_reference_fixtures():
    data = torch.load(GOLDEN)
    graph, nodes = data["graph"], data["graph"]["selected_nodes"]
    f, n = _gens(graph)
    for c in data["cases"]:
        L = c["x"].shape[0]
        x, p, m = c["x"].cuda(), c["logits"].cuda(), c["mask"].cuda()
        got_f = f.get_draft_blocks(x, p, m, start_pos=64, end_pos=64 + L,
                                   small_block_start=c["small"][0], small_block_end=c["small"][1])
        got_n = n.get_draft_blocks(x, p, m)
        assert [nodes.index(d["node"]) for d in got_f] == [k for _, k in c["fastdllm"]]
        assert [nodes.index(d["node"]) for d in got_n] == [k for _, k in c["nld"]]
        for d, (state, _) in zip(got_f, c["fastdllm"]):
            assert torch.equal(d["state"].cpu(), state) and d["start_pos"] == 64
        for d, (state, _) in zip(got_n, c["nld"]):
            assert torch.equal(d["state"].cpu(), state)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_drafts_qwen_vocabulary(dtype):
    """A 32-position block over a Qwen-sized vocabulary (152064)."""
    nodes = GRAPH["selected_nodes"]
    f, n = _gens(GRAPH)
    for seed, n_masked in ((7, 32), (8, 9)):
        x, p, m = case(seed, 32, 152064, dtype, n_masked)
        _same(f.get_draft_blocks(x.cuda(), p.cuda(), m.cuda(), start_pos=0, end_pos=32,
                                 small_block_start=0, small_block_end=32),
              drafts.fastdllm_draft_blocks(GRAPH, x, p, m, 0, 32, 0, 32), nodes)
        _same(n.get_draft_blocks(x.cuda(), p.cuda(), m.cuda()),
              drafts.nld_draft_blocks(GRAPH, x, p, m), nodes)


def test_no_graph_or_no_mask():
    f, _ = _gens(None)
    x, p, m = case(1, 32, 1000, torch.float32, 4)
    assert f.get_draft_blocks(x.cuda(), p.cuda(), m.cuda(), small_block_start=0, small_block_end=32) == []
    f.calibration_graph = GRAPH
    assert f.get_draft_blocks(x.cuda(), p.cuda(), torch.zeros(32, dtype=torch.bool, device="cuda"),
                              small_block_start=0, small_block_end=32) == []
