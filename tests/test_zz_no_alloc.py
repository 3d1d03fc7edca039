"""The FFN entry point for callers that cannot allocate device memory.

``sf_fused_ffn_scatter_static`` must give the same result as ``sf_fused_ffn_scatter``
(which takes caller-allocated scratch) within the parity tolerance, on two calls in a
row through the C ABI -- the second call shows that what the first call left in the
shared static scratch does not leak into the next result.  This file is collected last;
it also passes when run alone in a fresh process.
"""
import ctypes

import pytest
import torch

from specfold_b200 import _lib
from specfold_b200 import kernels as K
from tests.helpers import assert_close

pytestmark = pytest.mark.gpu


def _inputs(seed, dtype, BN=256, D=512, I=1408, count=122):
    g = torch.Generator().manual_seed(seed)
    hp = torch.randn(BN, D, generator=g).to(dtype)
    ln = (1 + 0.1 * torch.randn(D, generator=g)).to(dtype)
    wg = (torch.randn(I, D, generator=g) * 0.05).to(dtype)
    wu = (torch.randn(I, D, generator=g) * 0.05).to(dtype)
    wd = (torch.randn(D, I, generator=g) * 0.05).to(dtype)
    rows = torch.randperm(BN, generator=g)[:count].sort().values
    return [t.cuda() for t in (hp, ln, wg, wu, wd, rows)] + [count]


def _static_call(hp, ln, wg, wu, wd, rows, count, eps=1e-6, bucket=None):
    BN, D = hp.shape
    bucket = BN if bucket is None else bucket
    I = wg.shape[0]
    ffn = torch.zeros(BN + 1, D, dtype=hp.dtype, device="cuda")
    cnt = torch.tensor([count], dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    lib = _lib.load()
    st = lib.sf_fused_ffn_scatter_static(
        K.dtype_code(hp), hp.data_ptr(), ln.data_ptr(), wg.data_ptr(), wu.data_ptr(),
        wd.data_ptr(), rows.data_ptr(), cnt.data_ptr(), ffn.data_ptr(), bucket, ctypes.c_float(eps),
        D, I, err.data_ptr(), torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "sf_fused_ffn_scatter_static")
    torch.cuda.synchronize()
    K.raise_device_error(err)
    return ffn


def _scratch_call(hp, ln, wg, wu, wd, rows, count, eps=1e-6, bucket=None):
    BN, D = hp.shape
    bucket = BN if bucket is None else bucket
    ffn = torch.zeros(BN + 1, D, dtype=hp.dtype, device="cuda")
    cnt = torch.tensor([count], dtype=torch.int32, device="cuda")
    out = K.fused_ffn_scatter(hp, ln, wg, wu, wd, rows, cnt, ffn, bucket, eps)
    torch.cuda.synchronize()
    K.raise_device_error(out["err"])
    return ffn


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_static_scratch_matches_allocating_entry_point(dtype):
    for seed, count in ((1, 122), (2, 200)):       # two calls in a row, different inputs
        args = _inputs(seed, dtype, count=count)
        got = _static_call(*args)
        want = _scratch_call(*args)
        rows = args[5]
        assert_close(got[rows], want[rows], dtype, f"static-scratch ffn (call seed {seed})")
        untouched = torch.ones(got.shape[0], dtype=torch.bool, device="cuda")
        untouched[rows] = False
        assert got[untouched].abs().max().item() == 0.0


def test_static_scratch_7b_shape():
    """The Qwen2.5-7B FFN (D = 3584, I = 18944) at a 160-row bucket, which fits the fixed
    scratch with the GEMMs split over K (gate/up and down both run several splits whose
    fp32 partials and tile counters live in the static array), two calls in a row."""
    for seed, count in ((3, 122), (4, 160)):
        args = _inputs(seed, torch.bfloat16, BN=256, D=3584, I=18944, count=count)
        hp, ln, wg, wu, wd, rows, cnt = args
        got = _static_call(hp, ln, wg, wu, wd, rows, cnt, bucket=160)
        want = _scratch_call(hp, ln, wg, wu, wd, rows, cnt, bucket=160)
        assert_close(got[rows], want[rows], torch.bfloat16, f"7B static-scratch ffn (seed {seed})")


def test_static_scratch_rejects_oversized_shapes():
    lib = _lib.load()
    # 7B-like FFN with a 1024-row bucket needs far more than the fixed scratch
    st = lib.sf_fused_ffn_scatter_static(1, 16, 16, 16, 16, 16, 16, 16, 16, 1024,
                                         ctypes.c_float(1e-6), 8192, 28672, None, None)
    assert st == 1
    assert b"limit" in lib.sf_last_error()
