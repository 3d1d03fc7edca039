"""Shared test utilities: tolerance-checked comparison and model/case transfer."""
import copy

import torch

# tolerances written into every parity test: relative error, normwise over the whole
# tensor and row by row (each row of the last dimension against its own largest entry)
TOL = {torch.bfloat16: 2e-2, torch.float32: 1e-4}


def rel_err(got: torch.Tensor, ref: torch.Tensor) -> float:
    """max |got - ref| / max |ref| over the whole tensor."""
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    den = ref.abs().max().item()
    return (got - ref).abs().max().item() / (den if den > 0 else 1.0)


def row_err(got: torch.Tensor, ref: torch.Tensor) -> float:
    """max over rows of max |got_r - ref_r| / max |ref_r| (rows = the last dimension),
    so that one small row that is badly wrong is not hidden by the other rows' scale.
    Rows of the reference that are (nearly) all zero are measured against 1e-3 of the
    tensor's largest entry instead."""
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    if ref.numel() == 0:
        return 0.0
    g = got.reshape(-1, got.shape[-1]) if got.dim() else got.reshape(1, 1)
    r = ref.reshape(-1, ref.shape[-1]) if ref.dim() else ref.reshape(1, 1)
    top = r.abs().max().item()
    den = r.abs().amax(-1).clamp_min(max(top * 1e-3, 1e-30))
    return ((g - r).abs().amax(-1) / den).max().item()


def assert_close(got, ref, dtype, what="", tol=None, rowwise=True):
    tol = TOL[dtype] if tol is None else tol
    e = rel_err(got, ref)
    assert e <= tol, f"{what}: relative error {e:.3e} > {tol:.1e}"
    if rowwise:
        er = row_err(got, ref)
        assert er <= tol, f"{what}: row-wise relative error {er:.3e} > {tol:.1e}"
    return e


def to_cuda_model(model):
    return copy.deepcopy(model).cuda()
