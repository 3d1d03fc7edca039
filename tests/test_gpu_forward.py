"""End-to-end parity of the B200 folded verify forward against the CPU oracle.

For every golden case (which pins the oracle to the reference) the CUDA path runs the
same seeded inputs; fold masks and fold counters must be bit-identical, logits within
2e-2 (bf16) / 1e-4 (fp32) normwise relative error.
"""
import pytest
import torch

from oracle import folded_oracle as orc
from specfold_b200 import SpecFoldB200FastDLLMV2Generation, SpecFoldB200NLDGeneration
from specfold_b200.synthetic import (SHAPES, ModelDims, StandinExecutor, build_model,
                                     config0_hidden, inject_hidden, random_prefix_cache,
                                     tree_block_input)
from tests.golden.make_golden import CASES, build_case
from tests.helpers import assert_close, to_cuda_model

pytestmark = pytest.mark.gpu


def _run_both(name, fold_bucket=None):
    family, model, cache, ids, delta = build_case(name)
    cap = orc.Capture()
    with torch.no_grad():
        ref = orc.folded_forward(model, ids, cache, delta, family=family, capture=cap)
    cls = SpecFoldB200FastDLLMV2Generation if family == "fastdllm" else SpecFoldB200NLDGeneration
    gen = cls(model_executor=StandinExecutor(to_cuda_model(model)), delta=delta,
              fold_bucket=fold_bucket)
    gen.record_masks = True
    out = gen._batched_block_forward(ids.cuda(), None if cache is None else cache.to("cuda"))
    torch.cuda.synchronize()
    return ref, cap, out, gen


# A bf16 layer input computed on the GPU differs from the CPU oracle's by rounding
# (GEMM summation order), so past layer 0 a draft row whose distance to the threshold is
# inside that noise may legitimately land on the other side.  Such rows are allowed only
# where the oracle's own margin |moved / (delta * ||x_par||) - 1| is below this bound;
# layer 0 (identical inputs) and every fp32 layer must match bit for bit.  Identical
# inputs always give identical masks (tests/test_gpu_kernels.py::test_gate_and_compaction).
BF16_MARGIN = 0.05


def _descendants(b, parent):
    out = {b}
    changed = True
    while changed:
        changed = False
        for i, p in enumerate(parent):
            if p is not None and p in out and i not in out:
                out.add(i)
                changed = True
    return out


def _check_against_oracle(name, ref, cap, out, gen):
    dtype = ref.dtype
    assert out.dtype == dtype and out.shape == ref.shape
    masks = gen.last_rec_masks.bool().cpu()
    flips = []
    for li, lay in enumerate(cap.layers):
        diff = masks[li] != lay["rec"]
        if li == 0 or dtype == torch.float32:
            assert not diff.any(), f"layer {li} fold mask differs at {diff.nonzero().tolist()}"
        else:
            assert (lay["margin"][diff] < BF16_MARGIN).all(), \
                f"layer {li}: rows far from the threshold flipped: {diff.nonzero().tolist()}"
            flips += [(li, b, n) for b, n in diff.nonzero().tolist()]
    assert len(flips) <= 0.02 * cap.positions, f"{len(flips)} near-threshold flips"
    assert gen._fold_draft_positions == cap.positions
    if not flips:
        assert gen._fold_draft_recomputed == cap.recomputed
    # a flipped row changes its branch and every branch below it; all others must agree
    affected = set()
    for _, b, _ in flips:
        affected |= _descendants(b, cap.parent)
    keep = [b for b in range(ref.shape[0]) if b not in affected]
    assert keep and 0 in keep
    assert_close(out[keep], ref[keep], dtype, f"{name} logits (branches {keep})")
    return flips


@pytest.mark.parametrize("name", sorted(CASES))
def test_forward_matches_oracle(name):
    ref, cap, out, gen = _run_both(name)
    _check_against_oracle(name, ref, cap, out, gen)


# shapes large enough that the projections split K across CTAs (the golden shapes do not)
EXTRA = {
    "mid_bf16_tree": ("fastdllm", ModelDims(hidden=1024, heads=8, kv_heads=2, head_dim=128,
                                            inter=2816, layers=2, vocab=1000), 96, "tree"),
    "c0shape_bf16_inject": ("fastdllm", SHAPES["qwen1.5b-1layer"], 256, "inject"),
    "mid_nld_bf16_chain": ("nld", ModelDims(hidden=1024, heads=8, kv_heads=4, head_dim=128,
                                            inter=2048, layers=2, vocab=512, eps=1e-5,
                                            theta=5e5), 64, "chain"),
    # Qwen2.5's vocabulary: the tiled lm_head runs its last round's tiles as a split-K phase
    "mid_bf16_qwen_vocab": ("fastdllm", ModelDims(hidden=512, heads=4, kv_heads=2, head_dim=128,
                                                  inter=1408, layers=1, vocab=152064), 64, "tree"),
}
# a hidden size past 6144: the layer tail's fused norm keeps four vectors of 8 per thread
# (the instantiation every shape up to 6144 does not use)
EXTRA["wide_bf16_d8192"] = ("fastdllm", ModelDims(hidden=8192, heads=64, kv_heads=8,
                                                 head_dim=128, inter=1024, layers=1,
                                                 vocab=512), 64, "tree")
# long prefixes of the Llama-8B microbenchmark sweep (GQA group 4, RoPE theta 5e5): the
# prefix attention caps its key splits at 16, so each split streams P / 16 keys
_LONG = ModelDims(hidden=1024, heads=8, kv_heads=2, head_dim=128, inter=1024, layers=1,
                  vocab=512, eps=1e-5, theta=5e5)
for _p in (4096, 16384, 32768):
    EXTRA[f"long_prefix_{_p // 1024}k"] = ("nld", _LONG, _p, "tree")


@pytest.mark.parametrize("name", sorted(EXTRA))
def test_forward_split_k_shapes(name):
    family, dims, P, kind = EXTRA[name]
    dtype = torch.bfloat16
    model = build_model(dims, family=family, dtype=dtype, seed=0)
    cache = random_prefix_cache(dims, P, dtype=dtype, seed=1)
    if kind == "inject":
        ids = torch.zeros(8, 32, dtype=torch.int64)
        inject_hidden(model, config0_hidden(dims, 8, 32, dtype=dtype))
    else:
        ids = tree_block_input(dims.vocab, N=32, edits_per_level=3 if kind == "tree" else 1)
    delta = 0.1 if kind != "chain" else 0.02
    cap = orc.Capture()
    with torch.no_grad():
        ref = orc.folded_forward(model, ids, cache, delta, family=family, capture=cap)
    cls = SpecFoldB200FastDLLMV2Generation if family == "fastdllm" else SpecFoldB200NLDGeneration
    gen = cls(model_executor=StandinExecutor(to_cuda_model(model)), delta=delta)
    gen.record_masks = True
    out = gen._batched_block_forward(ids.cuda(), cache.to("cuda"))
    torch.cuda.synchronize()
    _check_against_oracle(name, ref, cap, out, gen)


def test_tiled_weights_bit_identical():
    """The 128x64 weight-tile layout changes only where the bytes sit: the tensor-core
    GEMMs run the same MMAs in the same order, so logits are bit-identical."""
    family, dims, P, kind = EXTRA["mid_bf16_tree"]
    model = build_model(dims, family=family, dtype=torch.bfloat16, seed=0, device="cuda")
    cache = random_prefix_cache(dims, P, dtype=torch.bfloat16, seed=1, device="cuda")
    ids = tree_block_input(dims.vocab, N=32, edits_per_level=3).cuda()
    outs = []
    for tiled in (True, False):
        gen = SpecFoldB200FastDLLMV2Generation(model_executor=StandinExecutor(model), delta=0.1)
        gen.tile_weights = tiled
        outs.append(gen._batched_block_forward(ids, cache))
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


def test_forward_repeatable():
    _, _, a, _ = _run_both("tiny_bf16_chain")
    _, _, b, _ = _run_both("tiny_bf16_chain")
    assert torch.equal(a, b), "two runs of the same inputs differ"


def test_small_bucket_overflow_reruns():
    # a bucket smaller than the recomputed row count overflows; the generator re-runs with
    # room for every row and still matches the oracle
    ref, cap, out, gen = _run_both("tiny_fp32_tree", fold_bucket=40)
    assert_close(out, ref, torch.float32, "overflow rerun logits")
