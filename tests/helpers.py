"""Shared test utilities: tolerance-checked comparison and model/case transfer."""
import copy

import torch

# tolerances written into every parity test: normwise max relative error
TOL = {torch.bfloat16: 2e-2, torch.float32: 1e-4}


def rel_err(got: torch.Tensor, ref: torch.Tensor) -> float:
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    den = ref.abs().max().item()
    return (got - ref).abs().max().item() / (den if den > 0 else 1.0)


def assert_close(got, ref, dtype, what="", tol=None):
    tol = TOL[dtype] if tol is None else tol
    e = rel_err(got, ref)
    assert e <= tol, f"{what}: relative error {e:.3e} > {tol:.1e}"
    return e


def to_cuda_model(model):
    return copy.deepcopy(model).cuda()
