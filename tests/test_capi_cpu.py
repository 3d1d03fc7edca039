"""The C-ABI library loads without a GPU, exports every function include/specfold_b200.h
declares, and rejects bad arguments before touching the device."""
import ctypes
import os
import re

import pytest

import torch

from specfold_b200 import _lib
from specfold_b200.folded import FoldedVerifyB200
from oracle import folded_oracle as orc

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "specfold_b200.h")


def declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sf_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported_and_bound():
    lib = _lib.load()
    names = declared()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.exported_symbols(), f"{n} not bound in _lib"
    # and nothing is bound that the header does not declare
    assert set(_lib.exported_symbols()) <= set(names)


def test_abi_version_and_workspace_sizes():
    lib = _lib.load()
    assert lib.sf_abi_version() == 1
    small = lib.sf_verify_workspace_bytes(1, 8, 32, 256, 4, 2, 64, 384, 128, 64)
    big = lib.sf_verify_workspace_bytes(1, 8, 32, 3584, 28, 4, 128, 18944, 152064, 1024)
    assert 0 < small < big < (1 << 30)


def test_argument_validation_without_device():
    lib = _lib.load()
    assert lib.sf_folded_verify_forward(None) == 1
    assert b"null" in lib.sf_last_error()
    args = _lib.SfVerifyArgs()
    args.dtype, args.B1, args.N, args.D, args.H, args.Hkv, args.hd = 1, 8, 32, 100, 4, 2, 64
    assert lib.sf_folded_verify_forward(ctypes.byref(args)) == 1      # D % 64 != 0
    assert b"multiple of 64" in lib.sf_last_error()
    args.D, args.hd = 256, 96
    assert lib.sf_folded_verify_forward(ctypes.byref(args)) == 1      # head_dim
    # gate: B1 beyond one warp per branch
    st = lib.sf_residual_delta_gate(1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, None, None, 0.1, 40, 32,
                                    256, 256, 1e-6, None, None)
    assert st == 1
    assert lib.sf_kv_append(1, 16, 16, 100, 16, 16, 1024, 4, 128, 0, 32, None) == 1  # capacity
    # sampler: row stride below V, non-positive top_p
    assert lib.sf_sample_top_p_greedy(1, 16, 4, 1000, 999, 0.95, 16, 16, None) == 1
    assert lib.sf_sample_top_p_greedy(1, 16, 4, 1000, 1000, 0.0, 16, 16, None) == 1
    assert b"sample_top_p_greedy" in lib.sf_last_error()
    # drafts: top-k depth beyond 16, positions outside the block, short workspace
    assert lib.sf_draft_blocks(1, 16, 1000, 32, 1000, 17, 0, 16, 16, 16, 2, 16, 32, 0, 16, 16,
                               16, 1 << 20, None) == 1
    assert lib.sf_draft_blocks(1, 16, 1000, 32, 1000, 4, 0, 16, 16, 16, 2, 16, 32, 8, 16, 16,
                               16, 1 << 20, None) == 1
    need = lib.sf_draft_workspace_bytes(32, 4)
    assert need >= 32 * 4 + 32 * 4 * 8
    assert lib.sf_draft_blocks(1, 16, 1000, 32, 1000, 4, 0, 16, 16, 16, 2, 16, 32, 0, 16, 16,
                               16, need - 1, None) == 4                          # workspace


def test_parent_map_matches_oracle():
    g = torch.Generator().manual_seed(0)
    for trial in range(50):
        B1, N = 8, 12
        base = torch.randint(0, 5, (N,), generator=g)
        rows = base.repeat(B1, 1)
        for i in range(1, B1):
            k = int(torch.randint(0, 4, (1,), generator=g))
            pos = torch.randperm(N, generator=g)[:k]
            rows[i, pos] = torch.randint(5, 9, (k,), generator=g)
        assert FoldedVerifyB200._build_parent_map(rows) == orc.parent_map(rows)


def test_preallocated_kv_cache_is_device_only():
    """The cache appends with a CUDA kernel; there is no host fallback."""
    import torch
    from specfold_b200.kv_cache import PreallocatedKVCache
    with pytest.raises(ValueError):
        PreallocatedKVCache(2, 4, 128, 64, dtype=torch.bfloat16, device="cpu")
    with pytest.raises(ValueError):
        PreallocatedKVCache(0, 4, 128, 64, dtype=torch.bfloat16, device="cuda")


def test_no_fallback_to_the_reference_sampler_or_drafts():
    """The generator hooks never hand work to a CPU or reference path: temperature
    sampling, CPU tensors and other dtypes raise before anything runs."""
    from specfold_b200 import SpecFoldB200FastDLLMV2Generation, SpecFoldB200NLDGeneration
    gen = SpecFoldB200FastDLLMV2Generation(model_executor=None)
    logits = torch.zeros(1, 4, 16)
    with pytest.raises(NotImplementedError):
        gen._sample_with_top_p(logits, top_p=0.95, temperature=0.0)      # CPU logits
    with pytest.raises(NotImplementedError):
        gen._sample_with_top_p(logits, top_p=0.95, temperature=0.7)      # temperature
    gen.calibration_graph = {"selected_nodes": [{"ij_set": [[0, 0]]}]}
    with pytest.raises(NotImplementedError):
        gen.get_draft_blocks(torch.zeros(8, dtype=torch.int64), torch.zeros(8, 16),
                             torch.ones(8, dtype=torch.bool), 0, 8, 0, 8)
    nld = SpecFoldB200NLDGeneration(model_executor=None)
    nld.calibration_graph = gen.calibration_graph
    with pytest.raises(NotImplementedError):
        nld.get_draft_blocks(torch.zeros(8, dtype=torch.int64), torch.zeros(8, 16),
                             torch.ones(8, dtype=torch.bool))


def test_tensor_parallel_entries_without_device():
    """The peer-memory exchange's host-side entry points: buffer sizing, the peer table's
    argument checks (it only records addresses, so it needs no device), and the IPC
    calls' rejection of missing arguments."""
    lib = _lib.load()
    assert lib.sf_tp_exchange_bytes(256, 3584) == 512 + 2 * 256 * 3584 * 4
    assert lib.sf_tp_exchange_bytes(0, 3584) == 0
    out = ctypes.c_void_p()
    two = (ctypes.c_void_p * 2)(0x10000, 0x20000)
    assert lib.sf_tp_peers_init(0, 1, two, 256, 512, ctypes.byref(out)) == 1      # size < 2
    assert lib.sf_tp_peers_init(2, 2, two, 256, 512, ctypes.byref(out)) == 1      # rank
    assert lib.sf_tp_peers_init(0, 2, two, 256, 510, ctypes.byref(out)) == 1      # D % 4
    odd = (ctypes.c_void_p * 2)(0x10000, 0x20008)
    assert lib.sf_tp_peers_init(0, 2, odd, 256, 512, ctypes.byref(out)) == 1      # unaligned
    assert b"unaligned" in lib.sf_last_error()
    assert lib.sf_tp_peers_init(1, 2, two, 256, 512, ctypes.byref(out)) == 0
    assert out.value
    assert lib.sf_tp_peers_destroy(out) == 0
    h = (ctypes.c_char * 64)()
    off = ctypes.c_size_t()
    assert lib.sf_tp_ipc_export(None, ctypes.cast(h, ctypes.c_void_p), 64, ctypes.byref(off)) == 1
    assert lib.sf_tp_ipc_export(0x10000, ctypes.cast(h, ctypes.c_void_p), 8, ctypes.byref(off)) == 1
    base = ctypes.c_void_p()
    assert lib.sf_tp_ipc_open(None, 64, ctypes.byref(base)) == 1
    assert lib.sf_tp_ipc_close(None) == 1

