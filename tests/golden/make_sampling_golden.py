"""Golden vectors for the greedy top-p sampler, made by the reference itself.

Calls ``FastDLLMModelExecutor.sample_with_top_p`` (specfold/generate/
fastdllm_model_executor.py:109-155) from a checkout of chungen04/specfold on seeded
logits, on the CPU, through its own implementation (the executor is built without a
model, so the model-provided sampler branch is not taken), and saves inputs and
outputs to ``tests/golden/sampling.pt``:

    python tests/golden/make_sampling_golden.py --reference /path/to/specfold
"""

from __future__ import annotations

import argparse
import importlib
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def cases():
    """(name, logits): bf16 and fp32 rows, peaked to flat, with exact ties."""
    out = []
    g = torch.Generator().manual_seed(1234)
    for dtype in (torch.bfloat16, torch.float32):
        for V in (1000, 4096):
            rows = []
            for scale in (0.05, 0.5, 2.0, 6.0):
                rows.append(torch.randn(6, V, generator=g) * scale)
            peak = torch.randn(6, V, generator=g)
            idx = torch.randint(0, V, (6,), generator=g)
            peak[torch.arange(6), idx] += torch.tensor([2.0, 4.0, 6.0, 8.0, 12.0, 30.0])
            rows.append(peak)
            tie = torch.randn(6, V, generator=g)
            top = tie.max(-1).values
            for r in range(6):
                j = torch.randint(0, V, (3,), generator=g)
                tie[r, j] = top[r]
            rows.append(tie)
            x = torch.cat(rows, 0).to(dtype)
            out.append((f"{str(dtype).split('.')[-1]}_V{V}", x))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=os.path.join(HERE, "sampling.pt"))
    args = ap.parse_args()
    # the package __init__s pull in the vendored NLD model (which does not import under
    # transformers 5.x): register the packages as bare namespaces, as make_golden.py does
    import types
    for name in ("specfold", "specfold.generate"):
        m = types.ModuleType(name)
        m.__path__ = [os.path.join(args.reference, *name.split("."))]
        sys.modules[name] = m
    sys.path.insert(0, args.reference)
    mod = importlib.import_module("specfold.generate.fastdllm_model_executor")
    ex = object.__new__(mod.FastDLLMModelExecutor)
    ex.model = object()                         # no model-provided sampler
    data = {}
    for name, x in cases():
        for top_p in (0.95, 0.5):
            tok, probs = ex.sample_with_top_p(x, top_p=top_p, temperature=0.0)
            conf = torch.gather(probs, -1, tok.unsqueeze(-1)).squeeze(-1)
            data[f"{name}_p{top_p}"] = {"logits": x, "top_p": top_p, "tokens": tok, "conf": conf}
    torch.save(data, args.out)
    print("wrote", args.out, sorted(data))


if __name__ == "__main__":
    main()
