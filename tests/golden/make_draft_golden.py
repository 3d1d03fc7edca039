"""Golden vectors for draft construction, made by the reference itself.

Calls ``FastDLLMV2SpeculativeGeneration.get_draft_blocks``
(specfold/generate/fastdllm_v2_generation.py:387-474) and
``NLDDiffusionGeneration.get_draft_blocks`` (specfold/generate/nld_generation.py:108-151)
from a checkout of chungen04/specfold on seeded inputs, on the CPU, and saves inputs
and outputs to ``tests/golden/drafts.pt``:

    python tests/golden/make_draft_golden.py --reference /path/to/specfold

The logits give every position a distinct top probability and distinct top tokens, so
that torch.topk's order is defined (its order among equal values is not).
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from tests.golden.make_golden import import_reference  # noqa: E402

GRAPH = {"selected_nodes": [
    {"L": 1, "ij_set": [(0, 1)]},
    {"L": 1, "ij_set": [(1, 0)]},
    {"L": 2, "ij_set": [(0, 0), (1, 1)]},
    {"L": 2, "ij_set": [(0, 2), (2, 0)]},
    {"L": 3, "ij_set": [(0, 0), (1, 0), (2, 1)]},
    {"L": 1, "ij_set": []},
    {"L": 2, "ij_set": [(3, 3), (5, 0)]},
    {"L": 1, "ij_set": [(7, 1)]},
]}


def case(seed, L, V, dtype, n_masked):
    """Block tokens, logits [L, V] and a mask with n_masked masked positions."""
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(L, V, generator=g) * 0.1
    for pos in range(L):
        toks = torch.randperm(V, generator=g)[:6]
        base = 2.0 + 0.37 * ((pos * 7) % L)                  # distinct per position
        logits[pos, toks] += base - torch.arange(6, dtype=torch.float32) * 0.75
    x = torch.randint(0, V, (L,), generator=g)
    mask = torch.zeros(L, dtype=torch.bool)
    mask[torch.randperm(L, generator=g)[:n_masked]] = True
    return x, logits.to(dtype), mask


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=os.path.join(HERE, "drafts.pt"))
    args = ap.parse_args()
    import_reference(args.reference)
    import importlib
    fd = importlib.import_module("specfold.generate.fastdllm_v2_generation")
    nd = importlib.import_module("specfold.generate.nld_generation")
    fgen = object.__new__(fd.FastDLLMV2SpeculativeGeneration)
    fgen.calibration_graph = GRAPH
    ngen = object.__new__(nd.NLDDiffusionGeneration)
    ngen.calibration_graph = GRAPH
    data = {"graph": GRAPH, "cases": []}
    for i, (L, V, dtype, n_masked, small) in enumerate([
            (32, 1000, torch.float32, 20, (8, 16)), (32, 1000, torch.bfloat16, 12, (0, 32)),
            (32, 4096, torch.float32, 5, (16, 32)), (32, 4096, torch.bfloat16, 32, (8, 24)),
            (32, 1000, torch.float32, 2, (0, 8)), (16, 2048, torch.float32, 0, (0, 16))]):
        x, logits, mask = case(100 + i, L, V, dtype, n_masked)
        f = fgen.get_draft_blocks(x, logits, mask, start_pos=64, end_pos=64 + L,
                                  small_block_start=small[0], small_block_end=small[1])
        n = ngen.get_draft_blocks(x, logits, mask)
        data["cases"].append({"x": x, "logits": logits, "mask": mask, "small": small,
                              "fastdllm": [(d["state"], GRAPH["selected_nodes"].index(d["node"])) for d in f],
                              "nld": [(d["state"], GRAPH["selected_nodes"].index(d["node"])) for d in n]})
    torch.save(data, args.out)
    print("wrote", args.out, [(len(c["fastdllm"]), len(c["nld"])) for c in data["cases"]])


if __name__ == "__main__":
    main()
