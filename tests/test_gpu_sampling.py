"""GPU greedy top-p sampler against the CPU oracle (which the reference's own sampler
pins bit for bit on tests/golden/sampling.pt).

Tokens must match exactly.  Confidences may differ only through the nucleus cut: the
oracle's CPU cumsum rounds at every step, the kernel's sum is exact, so the cut can
move by a few tail tokens: in bf16 by at most one ulp, in fp32 by a relative 1e-4.
"""
import os

import pytest
import torch

from oracle import sampling
from specfold_b200 import kernels as K
from specfold_b200.folded import SpecFoldB200FastDLLMV2Generation

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "sampling.pt")


def _check(logits, top_p, name):
    tok, conf = K.sample_top_p_greedy(logits.cuda(), top_p)
    torch.cuda.synchronize()
    rt, rc = sampling.greedy_confidence(logits.cpu(), top_p)
    assert torch.equal(tok.cpu(), rt), f"{name}: tokens differ at {(tok.cpu() != rt).nonzero().flatten().tolist()[:8]}"
    c, r = conf.cpu().float(), rc.float()
    if logits.dtype == torch.bfloat16:
        ulp = torch.where(r > 0, 2.0 ** (torch.floor(torch.log2(r)) - 7), torch.full_like(r, 1e-30))
        bad = (c - r).abs() > ulp * 1.01
    else:
        bad = (c - r).abs() > 1e-4 * r.abs().clamp_min(1e-30)
    assert not bad.any(), f"{name}: confidence rows {bad.nonzero().flatten().tolist()[:8]}: {c[bad][:4]} vs {r[bad][:4]}"
    return (c == r).float().mean().item()


def test_sampler_matches_reference_fixtures():
    data = torch.load(GOLDEN)
    for name, case in data.items():
        _check(case["logits"], case["top_p"], name)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("scale", [0.1, 1.0, 4.0])
def test_sampler_qwen_vocabulary(dtype, scale):
    """Rows of a Qwen-sized vocabulary (152064), from near-uniform (the nucleus holds
    most of the vocabulary) to peaked."""
    g = torch.Generator().manual_seed(int(scale * 10))
    x = (torch.randn(24, 152064, generator=g) * scale)
    x[torch.arange(0, 24, 3), torch.randint(0, 152064, (8,), generator=g)] += 12.0
    _check(x.to(dtype), 0.95, f"{dtype} scale {scale}")


def test_sampler_strided_rows_and_generator_hook():
    """A slice of [B, N, V] logits (non-contiguous rows) through the generator's
    _sample_with_top_p: tokens, and the probabilities gathered at the tokens as the
    decode loop reads them (fastdllm_v2_generation.py:346-351)."""
    g = torch.Generator().manual_seed(3)
    full = (torch.randn(2, 40, 5000, generator=g) * 2.0).to(torch.bfloat16).cuda()
    logits = full[:, 4:36]
    gen = SpecFoldB200FastDLLMV2Generation(model_executor=None)
    x1, p1 = gen._sample_with_top_p(logits, top_p=0.95, temperature=0.0)
    conf = torch.gather(p1, -1, x1.unsqueeze(-1)).squeeze(-1)
    rt, rc = sampling.greedy_confidence(logits.cpu(), 0.95)
    assert p1.shape == logits.shape
    assert torch.equal(x1.cpu(), rt)
    assert torch.allclose(conf.cpu().float(), rc.float(), rtol=2 ** -7, atol=0)
