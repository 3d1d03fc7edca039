"""Generate the golden vectors that pin the CPU oracle to the reference.

Runs the reference's own PyTorch folded forwards --
``SpecFoldFastDLLMV2Generation._batched_block_forward``
(specfold/generate/fastdllm_v2_folded.py:89-223) and
``SpecFoldNLDGeneration._batched_block_forward`` (specfold/generate/nld_folded.py:104-241)
-- imported from a checkout of chungen04/specfold, on the seeded synthetic inputs of
``specfold_b200.synthetic`` and saves inputs + outputs under ``tests/golden/``.

The reference has no tests, fixtures or golden vectors of its own, so these are the
parity anchor.  Run it where the reference checkout exists (it is not needed at test
time):

    python tests/golden/make_golden.py --reference /path/to/specfold

Importing the reference: ``specfold/__init__`` and ``specfold/generate/__init__`` pull
in the vendored NLD model, which does not import under transformers 5.x, and the
executors, which want checkpoints.  The folded forwards touch none of that, so the
package modules are pre-registered as empty namespaces and the two NLD modules that
``nld_generation`` imports are stubbed.
"""

from __future__ import annotations

import argparse
import os
import sys
import types

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from specfold_b200 import synthetic as syn  # noqa: E402


def import_reference(ref: str):
    for name in ("specfold", "specfold.generate", "specfold.model_cache",
                 "specfold.model_cache.nemotron_labs_diffusion"):
        mod = types.ModuleType(name)
        mod.__path__ = [os.path.join(ref, *name.split("."))]
        sys.modules[name] = mod
    ex = types.ModuleType("specfold.generate.nld_model_executor")
    ex.NLDModelExecutor = object
    sys.modules[ex.__name__] = ex
    mdl = types.ModuleType("specfold.model_cache.nemotron_labs_diffusion.modeling_nemotron_labs_diffusion")
    mdl._get_num_transfer_tokens = mdl._get_transfer_index = None
    sys.modules[mdl.__name__] = mdl
    sys.path.insert(0, ref)
    import importlib
    fd = importlib.import_module("specfold.generate.fastdllm_v2_folded")
    nd = importlib.import_module("specfold.generate.nld_folded")
    return fd.SpecFoldFastDLLMV2Generation, nd.SpecFoldNLDGeneration


def make_generator(cls, model, delta):
    """Instance of the reference class without its checkpoint-loading __init__: the
    folded forward reads only model_executor.model, delta and the counters."""
    g = object.__new__(cls)
    g.model_executor = syn.StandinExecutor(model)
    g.delta = float(delta)
    g._fold_stats = []
    return g


# name -> (family, shape, dtype, P, delta, input kind)
CASES = {
    "tiny_fp32_inject": ("fastdllm", "tiny", torch.float32, 16, 0.1, "inject"),
    "tiny_fp32_tree": ("fastdllm", "tiny", torch.float32, 24, 0.1, "tree"),
    "tiny_bf16_tree": ("fastdllm", "tiny", torch.bfloat16, 24, 0.1, "tree"),
    "tiny_fp32_noprefix": ("fastdllm", "tiny", torch.float32, 0, 0.1, "tree"),
    "tiny_fp32_dense": ("fastdllm", "tiny", torch.float32, 16, -1.0, "tree"),
    "tiny_bf16_inject": ("fastdllm", "tiny", torch.bfloat16, 16, 0.1, "inject"),
    "tiny_nld_fp32_tree": ("nld", "tiny", torch.float32, 24, 0.1, "tree"),
    "tiny_fp32_chain": ("fastdllm", "tiny", torch.float32, 24, 0.01, "chain"),
    "tiny_bf16_chain": ("fastdllm", "tiny", torch.bfloat16, 24, 0.02, "chain"),
    "tiny_nld_bf16_inject": ("nld", "tiny", torch.bfloat16, 16, 0.1, "inject"),
    # configuration 0: one Qwen2.5-1.5B-shape layer, fp32, P = 256, delta 0.1
    "config0": ("fastdllm", "qwen1.5b-1layer", torch.float32, 256, 0.1, "inject"),
    # NLD with a non-unit llama-4 query scale: original_max_position_embeddings is set to 8
    # so that block positions [24, 56) get scale 1 + beta * log(1 + floor(pos / 8))
    # (nld_folded.py:37-53); the reference's own fused class falls back to its PyTorch
    # path for this case (nld_folded.py:275-278)
    "tiny_nld_fp32_qscale": ("nld", "tiny", torch.float32, 24, 0.1, "tree+qscale"),
    "tiny_nld_bf16_qscale": ("nld", "tiny", torch.bfloat16, 24, 0.1, "tree+qscale"),
}

# llama-4 query-scale parameters of the "+qscale" cases
QSCALE_BETA, QSCALE_OMAX = 0.1, 8


def build_case(name):
    family, shape, dtype, P, delta, kind = CASES[name]
    dims = syn.SHAPES[shape]
    model = syn.build_model(dims, family=family, dtype=dtype, seed=0)
    cache = syn.random_prefix_cache(dims, P, dtype=dtype, seed=1)
    B1, N = 8, 32
    if kind.endswith("+qscale"):
        kind = kind[:-len("+qscale")]
        model.config.rope_parameters = dict(model.config.rope_parameters,
                                            llama_4_scaling_beta=QSCALE_BETA,
                                            original_max_position_embeddings=QSCALE_OMAX)
    if kind in ("tree", "chain"):
        ids = syn.tree_block_input(dims.vocab, N=N, edits_per_level=3 if kind == "tree" else 1,
                                   seed=2)
    else:
        ids = torch.zeros(B1, N, dtype=torch.int64)
        syn.inject_hidden(model, syn.config0_hidden(dims, B1, N, dtype=dtype))
    return family, model, cache, ids, delta


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SPECFOLD_REFERENCE"),
                    help="checkout of the reference (or set SPECFOLD_REFERENCE)")
    ap.add_argument("--only", nargs="*")
    args = ap.parse_args()
    if not args.reference:
        ap.error("pass --reference or set SPECFOLD_REFERENCE")
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    fd_cls, nd_cls = import_reference(args.reference)
    for name in (args.only or CASES):
        family, model, cache, ids, delta = build_case(name)
        gen = make_generator(fd_cls if family == "fastdllm" else nd_cls, model, delta)
        with torch.no_grad():
            logits = gen._batched_block_forward(ids, cache)
        out = {
            "case": name, "ids": ids, "logits": logits,
            "positions": int(getattr(gen, "_fold_draft_positions", 0)),
            "recomputed": int(getattr(gen, "_fold_draft_recomputed", 0)),
            "parent": fd_cls._build_parent_map(ids)[0],
            "torch": str(torch.__version__),
        }
        path = os.path.join(HERE, f"{name}.pt")
        torch.save(out, path)
        print(f"{name}: logits {tuple(logits.shape)} {logits.dtype} recomputed "
              f"{out['recomputed']}/{out['positions']} -> {os.path.getsize(path)/1e6:.2f} MB")


if __name__ == "__main__":
    main()
