"""End-to-end decoding on the B200 kernels.

* The block commit forward (``commit_block_forward``: the dense block forward that also
  appends the block's keys and values to the cache inside the launch) against the CPU
  oracle: unshifted logits and the appended K/V within 2e-2 (bf16) / 1e-4 (fp32), the
  earlier prefix rows untouched.
* The device-side prefix length (a PreallocatedKVCache hands the kernels its length in
  device memory, so one captured graph serves every prefix length): bit-identical
  logits to the same prefix passed with a host-side length, across lengths whose key
  split counts differ, before and after graph capture.
* The batched block-causal prefill (k prompt blocks in one forward) against the oracle
  executor committing the blocks one at a time: cache rows and last-block logits.
* The decode loops (specfold_b200/decode.py) against golden runs of the reference's own
  loops (``generate_with_draft_speculation``, fastdllm_v2_generation.py:483-720, with the
  reference's PyTorch folded generator, and ``generate``, :188-385), made on the CPU by
  tests/golden/make_decode_golden.py: identical accepted tokens, model calls, drafts
  computed and verify-call branch counts.
"""
import os

import pytest
import torch

from oracle import folded_oracle as orc
from specfold_b200 import SpecFoldB200FastDLLMV2Generation
from specfold_b200.decode import FastDLLMV2Decoder
from specfold_b200.kv_cache import PreallocatedKVCache
from specfold_b200.synthetic import (ModelDims, PrefixCache, StandinExecutor, build_model,
                                     random_prefix_cache, tree_block_input)
from tests.golden.make_golden import build_case
from tests.helpers import assert_close, to_cuda_model

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("name", ["tiny_fp32_tree", "tiny_bf16_tree"])
def test_commit_forward_matches_oracle(name):
    family, model, cache, ids, delta = build_case(name)
    block = ids[:1]
    P = cache.get_seq_length()
    cap = orc.Capture()
    with torch.no_grad():
        ref = orc.folded_forward(model, block, cache, -1.0, family=family, capture=cap,
                                 shift=False)
    gen = SpecFoldB200FastDLLMV2Generation(model_executor=StandinExecutor(to_cuda_model(model)),
                                           delta=delta)
    pre = PreallocatedKVCache.from_cache(cache.to("cuda"), capacity=P + 40)
    out = gen.commit_block_forward(block.cuda(), pre)
    torch.cuda.synchronize()
    dtype = ref.dtype
    assert out.shape == ref.shape
    assert_close(out.cpu(), ref, dtype, f"{name} commit logits")
    assert pre.get_seq_length() == P + block.shape[1]
    for li, lay in enumerate(cap.layers):
        k, v = pre[li]
        assert torch.equal(k[:, :, :P].cpu(), cache[li][0]) and torch.equal(v[:, :, :P].cpu(), cache[li][1])
        assert_close(k[0, :, P:].cpu(), lay["k"][0], dtype, f"layer {li} committed keys")
        assert_close(v[0, :, P:].cpu(), lay["v"][0], dtype, f"layer {li} committed values")


def test_device_prefix_length_bit_identical():
    """bf16, head_dim 128 (tensor-core prefix attention): the cache capacity sizes the
    grid for four key splits while the actual prefixes need two or three; the splits
    past the actual length contribute empty partials, so the logits are bit-identical to
    the host-length launch -- on the direct call, the captured one and graph replays at
    other lengths."""
    dims = ModelDims(hidden=512, heads=4, kv_heads=2, head_dim=128, inter=768, layers=2, vocab=256)
    model = build_model(dims, family="fastdllm", dtype=torch.bfloat16, seed=0, device="cuda")
    ids = tree_block_input(dims.vocab, N=32, edits_per_level=3).cuda()
    full = random_prefix_cache(dims, 700, dtype=torch.bfloat16, seed=1, device="cuda")
    gen = SpecFoldB200FastDLLMV2Generation(model_executor=StandinExecutor(model), delta=0.1)
    pre = PreallocatedKVCache(dims.layers, dims.kv_heads, dims.head_dim, capacity=1024,
                              dtype=torch.bfloat16, device="cuda")
    for li in range(dims.layers):
        pre.update(full[li][0][:, :, :300], full[li][1][:, :, :300], li)
    lengths = [300, 300, 300, 332, 460, 700]
    for P in lengths:
        if pre.get_seq_length() < P:
            n0 = pre.get_seq_length()
            for li in range(dims.layers):
                pre.update(full[li][0][:, :, n0:P], full[li][1][:, :, n0:P], li)
        plain = PrefixCache([k[:, :, :P].contiguous() for k in full.keys],
                            [v[:, :, :P].contiguous() for v in full.values])
        a = gen._batched_block_forward(ids, pre)
        b = gen._batched_block_forward(ids, plain)
        torch.cuda.synchronize()
        assert torch.equal(a, b), f"prefix {P}: device-length forward differs"


def _golden(name):
    return torch.load(os.path.join(GOLDEN, f"{name}.pt"), weights_only=True)


@pytest.mark.parametrize("name", ["decode_tiny_fp32", "decode_config1_bf16"])
def test_decode_matches_reference_loop(name):
    from tests.golden.make_decode_golden import BLOCK, DELTA, SMALL, THRESHOLD, TOP_P, build
    gold = _golden(name)
    model, prompt, bias, graph, c = build(name, device="cuda")
    assert torch.equal(prompt, gold["prompt"])
    gen = SpecFoldB200FastDLLMV2Generation(model_executor=StandinExecutor(model), delta=DELTA)
    for mode in c["modes"]:
        dec = FastDLLMV2Decoder(gen, block_length=BLOCK, small_block_size=SMALL,
                                threshold=THRESHOLD, top_p=TOP_P, max_new_tokens=c["new"],
                                mask_id=c["mask_id"], stop_token=c["stop"],
                                calibration_graph=None if mode == "vanilla" else graph,
                                logit_bias=bias, seam="dense" if mode == "dense" else "folded")
        if mode == "vanilla":
            tokens, st = dec.generate(prompt.tolist())
        else:
            tokens, st = dec.generate_with_draft_speculation(prompt.tolist())
        ref = gold[mode]
        fwd = [n for kind, n in st["steps"] if kind == "forward"]
        print(f"{name} {mode}: {st['tokens_generated']} tokens, {st['model_calls']} model calls "
              f"(reference {ref['model_calls']}), {st['drafts_computed']} drafts (reference "
              f"{ref['drafts_computed']}), {st['draft_hits']} hits, fold ratio "
              f"{st['fold_ratio']:.3f} (reference {ref.get('fold_ratio')}), {st['tok_s']:.1f} tok/s "
              f"(reference loop on the CPU: {len(ref['tokens']) / ref['cpu_s']:.2f} tok/s)")
        assert tokens == ref["tokens"].tolist(), f"{mode}: accepted tokens differ"
        assert st["model_calls"] == ref["model_calls"], f"{mode}: model calls differ"
        assert st["drafts_computed"] == ref["drafts_computed"], f"{mode}: drafts differ"
        if mode != "vanilla":
            assert fwd == ref["forwards"], f"{mode}: branch counts of the verify calls differ"


@pytest.mark.parametrize("name", ["tiny_fp32_tree", "tiny_bf16_tree", "tiny128_bf16"])
@pytest.mark.parametrize("prefix", [0, 24])
def test_batched_prefill_matches_block_commits(name, prefix):
    """The batched block-causal prefill (sf_verify_args.prefill: k prompt blocks in one
    forward, every block attending to the prefix, the earlier blocks and itself) against
    the executor restatement of the oracle, which commits one block at a time
    (oracle/decode_standin.py): the cache rows and the last block's unshifted logits."""
    from oracle.decode_standin import GrowingCache, OracleExecutor
    from specfold_b200 import synthetic as syn
    if name == "tiny128_bf16":
        dims = syn.SHAPES["tiny128"]
        model = build_model(dims, family="fastdllm", dtype=torch.bfloat16, seed=0)
        cache = random_prefix_cache(dims, 24, dtype=torch.bfloat16, seed=1)
    else:
        _, model, cache, _, _ = build_case(name)
    dtype = next(model.parameters()).dtype
    vocab = model.config.vocab_size
    T = 4 * 32
    tokens = torch.randint(0, vocab, (1, T), generator=torch.Generator().manual_seed(9))
    L = len(model.model.layers)
    # oracle: block-by-block commits on top of the same prefix
    ref_cache = GrowingCache(L)
    if prefix:
        for li in range(L):
            ref_cache.update(cache[li][0][:, :, :prefix].clone(), cache[li][1][:, :, :prefix].clone(), li)
    ex = OracleExecutor(model, block=32)
    ref = ex.forward(tokens, ref_cache if prefix else None, update_past_key_values=True)
    ref_last = ref.logits[:, -32:]
    gen = SpecFoldB200FastDLLMV2Generation(model_executor=StandinExecutor(to_cuda_model(model)),
                                           delta=0.1)
    hkv, hd = cache[0][0].shape[1], cache[0][0].shape[3]
    pre = PreallocatedKVCache(L, hkv, hd, capacity=prefix + T + 64, dtype=dtype, device="cuda")
    if prefix:
        for li in range(L):
            pre.update(cache[li][0][:, :, :prefix].cuda(), cache[li][1][:, :, :prefix].cuda(), li)
    out = gen.prefill_forward(tokens.cuda(), pre, block=32, logits=True)
    torch.cuda.synchronize()
    assert pre.get_seq_length() == prefix + T
    assert out.shape == ref_last.shape
    assert_close(out.cpu(), ref_last, dtype, f"{name} prefill logits (last block)")
    got_cache = ref.past_key_values
    for li in range(L):
        k, v = pre[li]
        rk, rv = got_cache[li]
        assert_close(k.cpu(), rk, dtype, f"layer {li} prefill keys")
        assert_close(v.cpu(), rv, dtype, f"layer {li} prefill values")
