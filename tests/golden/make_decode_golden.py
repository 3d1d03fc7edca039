"""Golden decode runs made by the reference's own decoding loops.

Runs ``FastDLLMV2SpeculativeGeneration.generate_with_draft_speculation``
(specfold/generate/fastdllm_v2_generation.py:483-720) with the reference's PyTorch folded
generator ``SpecFoldFastDLLMV2Generation`` (fastdllm_v2_folded.py:36-223) as the verify
seam, and the vanilla loop ``generate`` (:188-385), on the CPU, imported from a checkout
of chungen04/specfold, and saves the accepted tokens and the loop's counters under
``tests/golden/decode_*.pt``.  The B200 decode loop (specfold_b200/decode.py) must give
the same tokens on the GPU (tests/test_gpu_decode.py).

What the loop needs besides the folded forward comes from ``oracle/decode_standin.py``:
the model executor (its Fast-dLLM v2 model code is remote code outside the reference;
restated as the oracle's dense block forward with the cache update), the tokenizer (ids
in, ids out) and the synthetic model's per-position logit bias on its LM head; the
sampler is the reference's own ``FastDLLMModelExecutor.sample_with_top_p``.

    SPECFOLD_REFERENCE=/path/to/specfold python tests/golden/make_decode_golden.py [--only NAME]
"""

from __future__ import annotations

import argparse
import os
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from specfold_b200 import synthetic as syn  # noqa: E402

# name -> decode configuration
CASES = {
    # a small fp32 model: a third of the generated positions carry no bias, so their
    # tokens are the model's own argmax (fp32 leaves no near-ties between CPU and GPU)
    "decode_tiny_fp32": dict(shape="tiny", dtype=torch.float32, prompt=80, new=128,
                             vocab=512, mask_id=511, stop=510, frac_strong=0.4,
                             frac_free=0.3, strong=12.0, weak_base=3.0, weak_step=0.25,
                             modes=("folded", "dense", "vanilla")),
    # the end-to-end configuration of the 28-layer Qwen2.5-1.5B shape: 512-token prompt,
    # 256 generated tokens, draft graph B=7 D=8 S=3, delta 0.1, threshold 0.9; every
    # generated position is biased (bf16 rounding then cannot move a token)
    "decode_config1_bf16": dict(shape="qwen1.5b", dtype=torch.bfloat16, prompt=512, new=256,
                                vocab=151936, mask_id=151665, stop=151645, frac_strong=0.6,
                                frac_free=0.0, strong=20.0, weak_base=6.0, weak_step=0.5,
                                modes=("folded", "vanilla")),
}
SEEDS = dict(model=0, prompt=5, bias=7)
DELTA = 0.1
BLOCK, SMALL, THRESHOLD, TOP_P = 32, 8, 0.9, 0.95


def build(name, device="cpu"):
    """(model, prompt ids [T], bias, graph, case dict) of a decode case; the model is
    built on the CPU (seeded CPU generator) and then moved to ``device``."""
    c = CASES[name]
    dims = syn.SHAPES[c["shape"]]
    if dims.vocab != c["vocab"]:
        import dataclasses
        dims = dataclasses.replace(dims, vocab=c["vocab"])
    model = syn.build_model(dims, family="fastdllm", dtype=c["dtype"], seed=SEEDS["model"])
    if device != "cpu":
        model = model.to(device)
    excl = (c["mask_id"], c["stop"])
    prompt = syn.decode_prompt(c["vocab"], c["prompt"], seed=SEEDS["prompt"], exclude=excl)
    total = c["prompt"] + c["new"] + 2 * BLOCK
    bias = syn.decode_bias(c["vocab"], c["prompt"], total, seed=SEEDS["bias"],
                           frac_strong=c["frac_strong"], frac_free=c["frac_free"],
                           strong=c["strong"], weak_base=c["weak_base"],
                           weak_step=c["weak_step"], exclude=excl)
    return model, prompt, bias, syn.synthetic_draft_graph(), c


def run_reference(name, ref_path):
    from tests.golden.make_golden import import_reference
    from oracle.decode_standin import BiasedHead, IdTokenizer, OracleExecutor
    import importlib
    fd_cls, _ = import_reference(ref_path)
    gen_mod = importlib.import_module("specfold.generate.fastdllm_v2_generation")
    ex_mod = importlib.import_module("specfold.generate.fastdllm_model_executor")
    model, prompt, bias, graph, c = build(name)
    model.lm_head = BiasedHead(model.lm_head, bias)
    tok = IdTokenizer({"prompt": prompt})
    ex = OracleExecutor(model, tokenizer=tok, block=BLOCK,
                        sampler=ex_mod.FastDLLMModelExecutor.sample_with_top_p)

    forwards = []

    class Folded(fd_cls):
        # the LM head's bias needs the block's first position; the trace records the
        # branch count of every verify call
        def _batched_block_forward(self, batched_input, past_key_values):
            model.lm_head.base = past_key_values.get_seq_length() if past_key_values is not None else 0
            forwards.append(int(batched_input.shape[0]))
            return super()._batched_block_forward(batched_input, past_key_values)

    out = {"case": name, "prompt": prompt, "torch": str(torch.__version__)}
    kw = dict(block_length=BLOCK, model_executor=ex, threshold=THRESHOLD, top_p=TOP_P,
              mask_id=c["mask_id"], stop_token=c["stop"], max_new_tokens=c["new"],
              small_block_size=SMALL, temperature=0.0)
    for mode in c["modes"]:
        forwards.clear()
        if mode == "vanilla":
            g = Folded(calibration_graph=None, delta=DELTA, **kw)
            t0 = time.time()
            text, calls = gen_mod.FastDLLMV2SpeculativeGeneration.generate(g, prompt="prompt")
            dt = time.time() - t0
            rec = {"model_calls": int(calls), "drafts_computed": 0}
        else:
            g = Folded(calibration_graph=graph, delta=DELTA if mode == "folded" else -1.0, **kw)
            t0 = time.time()
            text, n_tok, calls, drafts = g.generate_with_draft_speculation(prompt="prompt")
            dt = time.time() - t0
            rec = {"model_calls": int(calls), "drafts_computed": int(drafts),
                   "fold_ratio": float(g.fold_ratio) if mode == "folded" else None}
        ids = [int(t) for t in text[0].split()] if text[0] else []
        rec.update(tokens=torch.tensor(ids, dtype=torch.int64), forwards=list(forwards),
                   cpu_s=dt, cpu_threads=torch.get_num_threads())
        out[mode] = rec
        print(f"{name} {mode}: {len(ids)} tokens, {rec['model_calls']} model calls, "
              f"{rec['drafts_computed']} drafts, {dt:.1f} s on the CPU", flush=True)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SPECFOLD_REFERENCE"),
                    help="checkout of the reference (or set SPECFOLD_REFERENCE)")
    ap.add_argument("--only", nargs="*")
    args = ap.parse_args()
    if not args.reference:
        ap.error("pass --reference or set SPECFOLD_REFERENCE")
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name in (args.only or CASES):
        out = run_reference(name, args.reference)
        path = os.path.join(HERE, f"{name}.pt")
        torch.save(out, path)
        print(f"{name} -> {os.path.getsize(path) / 1e3:.1f} kB", flush=True)


if __name__ == "__main__":
    main()
