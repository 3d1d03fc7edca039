"""The CPU oracle reproduces the reference's PyTorch folded forward bit for bit.

Fixtures come from running the reference itself (tests/golden/make_golden.py); here the
same seeded inputs are rebuilt and fed to ``oracle.folded_oracle.folded_forward``.
"""
import os

import pytest
import torch

from oracle import folded_oracle as orc
from tests.golden.make_golden import CASES, build_case

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return torch.load(os.path.join(GOLDEN, f"{name}.pt"), weights_only=True)


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_golden(name):
    gold = _load(name)
    family, model, cache, ids, delta = build_case(name)
    assert torch.equal(ids, gold["ids"])
    cap = orc.Capture()
    with torch.no_grad():
        logits = orc.folded_forward(model, ids, cache, delta, family=family, capture=cap)
    assert logits.dtype == gold["logits"].dtype
    assert torch.equal(logits, gold["logits"]), (logits - gold["logits"]).abs().max()
    assert cap.positions == gold["positions"]
    assert cap.recomputed == gold["recomputed"]
    assert cap.parent[1:] == gold["parent"][1:]


def test_parent_map_cases():
    # draft 1 changes {3}; draft 2 changes {3, 5} -> parent 1; draft 3 changes {7} -> main;
    # draft 4 changes {3, 5, 9} -> parent 2; draft 5 changes {1, 2} -> no size-1 subset -> main
    base = torch.arange(12)
    rows = [base.clone() for _ in range(6)]
    rows[1][3] = 100
    rows[2][3] = 100; rows[2][5] = 101
    rows[3][7] = 102
    rows[4][3] = 100; rows[4][5] = 101; rows[4][9] = 103
    rows[5][1] = 104; rows[5][2] = 105
    parent, counts = orc.parent_map(torch.stack(rows))
    assert parent == [None, 0, 1, 0, 2, 0]
    assert counts == [0, 1, 2, 1, 3, 2]


def test_src_chain():
    rec = torch.tensor([[1, 1, 1], [0, 1, 0], [0, 0, 1]], dtype=torch.bool)
    src = orc.nearest_recomputing_ancestor(rec, [None, 0, 1])
    assert src.tolist() == [[0, 0, 0], [0, 1, 0], [0, 1, 2]]


def test_sampling_oracle_matches_reference():
    """oracle/sampling.py reproduces the reference's greedy top-p sampler
    (fastdllm_model_executor.py:109-155) bit for bit on the CPU fixtures."""
    import os
    from oracle import sampling
    path = os.path.join(os.path.dirname(__file__), "golden", "sampling.pt")
    data = torch.load(path)
    for name, case in data.items():
        tok, conf = sampling.greedy_confidence(case["logits"], case["top_p"])
        assert torch.equal(tok, case["tokens"]), name
        assert torch.equal(conf, case["conf"]), name


def test_draft_oracle_matches_reference():
    """oracle/drafts.py reproduces both reference draft constructions
    (fastdllm_v2_generation.py:387-474, nld_generation.py:108-151) on the fixtures."""
    import os
    from oracle import drafts
    data = torch.load(os.path.join(os.path.dirname(__file__), "golden", "drafts.pt"))
    graph, nodes = data["graph"], data["graph"]["selected_nodes"]
    for c in data["cases"]:
        L = c["x"].shape[0]
        f = drafts.fastdllm_draft_blocks(graph, c["x"], c["logits"], c["mask"], 64, 64 + L,
                                         c["small"][0], c["small"][1])
        n = drafts.nld_draft_blocks(graph, c["x"], c["logits"], c["mask"])
        for got, ref in ((f, c["fastdllm"]), (n, c["nld"])):
            assert [nodes.index(d["node"]) for d in got] == [k for _, k in ref]
            for d, (state, _) in zip(got, ref):
                assert torch.equal(d["state"], state)
