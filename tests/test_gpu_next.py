"""The rows next to the verify forward: the dense (unfolded) block forward on the same
kernels, and the preallocated prefix KV cache with its GPU append.

Dense forward: parity against the CPU oracle's folded forward at a negative threshold,
which recomputes every row and so is the dense bidirectional-in-block forward
(fastdllm_v2_folded.py:6).  KV cache: the append must equal the ``torch.cat`` of
``DynamicCache.update`` bit for bit, keep the cache's addresses while the capacity
lasts, and give the folded forward bit-identical logits to the same prefix held in
separate tensors.
"""
import pytest
import torch

from oracle import folded_oracle as orc
from specfold_b200 import SpecFoldB200FastDLLMV2Generation, SpecFoldB200NLDGeneration
from specfold_b200.kv_cache import PreallocatedKVCache
from specfold_b200.synthetic import PrefixCache, StandinExecutor
from tests.golden.make_golden import build_case
from tests.helpers import assert_close, to_cuda_model

pytestmark = pytest.mark.gpu


def _gen(family, model, delta):
    cls = SpecFoldB200FastDLLMV2Generation if family == "fastdllm" else SpecFoldB200NLDGeneration
    return cls(model_executor=StandinExecutor(to_cuda_model(model)), delta=delta)


@pytest.mark.parametrize("name", ["tiny_fp32_tree", "tiny_bf16_tree", "tiny_nld_fp32_tree",
                                  "tiny_fp32_chain"])
@pytest.mark.parametrize("branches", ["all", "main"])
def test_dense_block_forward(name, branches):
    family, model, cache, ids, delta = build_case(name)
    if branches == "main":
        ids = ids[:1]
    with torch.no_grad():
        ref = orc.folded_forward(model, ids, cache, -1.0, family=family)
    gen = _gen(family, model, delta)
    out = gen.dense_block_forward(ids.cuda(), None if cache is None else cache.to("cuda"))
    torch.cuda.synchronize()
    assert out.shape == ref.shape and out.dtype == ref.dtype
    assert_close(out.cpu(), ref, ref.dtype, f"{name} dense logits")
    # the fold counters belong to the folded forward only
    assert getattr(gen, "_fold_draft_positions", 0) == 0
    # and the folded forward of the same generator still uses its own threshold
    folded = gen._batched_block_forward(ids.cuda(), None if cache is None else cache.to("cuda"))
    with torch.no_grad():
        ref_f = orc.folded_forward(model, ids, cache, delta, family=family)
    assert_close(folded.cpu(), ref_f, ref_f.dtype, f"{name} folded logits after dense")


def _cat_update(ks, vs, li, k, v):
    """DynamicCache.update: the layer's prefix becomes cat(prefix, new) along the rows."""
    ks[li] = k if ks[li] is None else torch.cat([ks[li], k], dim=-2)
    vs[li] = v if vs[li] is None else torch.cat([vs[li], v], dim=-2)
    return ks[li], vs[li]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_kv_cache_update_matches_cat(dtype):
    L, Hkv, hd = 3, 4, 128
    g = torch.Generator(device="cuda").manual_seed(5)
    cache = PreallocatedKVCache(L, Hkv, hd, capacity=80, dtype=dtype, device="cuda")
    ks, vs = [None] * L, [None] * L
    ptr0 = None
    for step, n in enumerate([48, 32, 32, 1, 64]):          # crosses the capacity twice
        for li in range(L):
            k = torch.randn(1, Hkv, n, hd, generator=g, device="cuda").to(dtype)
            v = torch.randn(1, Hkv, n, hd, generator=g, device="cuda").to(dtype)
            if step == 3:                                    # non-contiguous new rows
                k = torch.randn(1, n, Hkv, hd, generator=g, device="cuda").to(dtype).transpose(1, 2)
            gk, gv = cache.update(k, v, li)
            rk, rv = _cat_update(ks, vs, li, k, v)
            assert torch.equal(gk, rk) and torch.equal(gv, rv)
        if step == 0:
            ptr0 = cache[0][0].data_ptr()
        if step == 1:
            # 80 rows, still within the capacity: the cache did not move
            assert cache[0][0].data_ptr() == ptr0
    assert cache.get_seq_length() == ks[0].shape[-2] == 177 and cache.capacity >= 177
    for li, (k, v) in enumerate(cache):
        assert torch.equal(k, ks[li]) and torch.equal(v, vs[li])
    cache.crop(100)
    assert cache.get_seq_length() == 100 and torch.equal(cache[1][0], ks[1][:, :, :100])
    cache.crop(-4)
    assert cache.get_seq_length() == 96


def test_kv_cache_rejects_bad_states():
    cache = PreallocatedKVCache(1, 2, 64, capacity=16, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        cache.update(torch.zeros(1, 4, 8, 64, dtype=torch.bfloat16, device="cuda"),
                     torch.zeros(1, 4, 8, 64, dtype=torch.bfloat16, device="cuda"), 0)
    with pytest.raises(ValueError):
        cache.update(torch.zeros(1, 2, 8, 64, device="cuda"), torch.zeros(1, 2, 8, 64, device="cuda"), 0)


@pytest.mark.parametrize("name", ["tiny_bf16_tree", "tiny_fp32_tree"])
def test_forward_with_preallocated_cache(name):
    """Same prefix, two containers: bit-identical logits; then a committed block appended
    in place keeps the addresses, and the forward over the longer prefix matches the
    forward over a torch.cat-grown copy."""
    family, model, cache, ids, delta = build_case(name)
    dims_cache = cache.to("cuda")
    gen = _gen(family, model, delta)
    a = gen._batched_block_forward(ids.cuda(), dims_cache)
    pre = PreallocatedKVCache.from_cache(dims_cache, capacity=dims_cache.get_seq_length() + 64)
    b = gen._batched_block_forward(ids.cuda(), pre)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    # commit one block of 32 rows per layer
    L = len(dims_cache)
    Hkv, hd = dims_cache[0][0].shape[1], dims_cache[0][0].shape[3]
    extra = random_prefix_cache_like(L, Hkv, hd, 32, dims_cache[0][0].dtype)
    ptrs = [pre[li][0].data_ptr() for li in range(L)]
    grown_k, grown_v = [], []
    for li in range(L):
        pre.update(extra[li][0], extra[li][1], li)
        grown_k.append(torch.cat([dims_cache[li][0], extra[li][0]], dim=-2))
        grown_v.append(torch.cat([dims_cache[li][1], extra[li][1]], dim=-2))
    assert [pre[li][0].data_ptr() for li in range(L)] == ptrs
    c = gen._batched_block_forward(ids.cuda(), pre)
    d = gen._batched_block_forward(ids.cuda(), PrefixCache(grown_k, grown_v))
    torch.cuda.synchronize()
    assert torch.equal(c, d)


def random_prefix_cache_like(L, Hkv, hd, n, dtype):
    g = torch.Generator(device="cuda").manual_seed(9)
    return [(torch.randn(1, Hkv, n, hd, generator=g, device="cuda").to(dtype),
             torch.randn(1, Hkv, n, hd, generator=g, device="cuda").to(dtype)) for _ in range(L)]
