"""CPU restatement of the reference's greedy top-p sampling (the parity oracle).

TEST INFRASTRUCTURE ONLY: used by ``tests/`` and the CPU-baseline legs of the
benchmarks; never by the product path in ``specfold_b200``.

Restates ``FastDLLMModelExecutor.sample_with_top_p``'s own implementation
(specfold/generate/fastdllm_model_executor.py:130-155), the one the decode loops call
through ``_sample_with_top_p`` (fastdllm_v2_generation.py:134-149, :346) when the
model has no built-in sampler, with the same torch op sequence so that on the CPU it
reproduces the reference bit for bit (pinned by ``tests/test_oracle_golden.py``
against ``tests/golden/sampling.pt``, made by ``tests/golden/make_sampling_golden.py``
from the reference itself).

On the CPU, torch accumulates the ``cumsum`` of bf16 probabilities in fp32 and rounds
each prefix to bf16; that is the semantics the GPU sampler implements.  (torch's CUDA
``cumsum`` of a bf16 tensor accumulates in bf16 and stalls below 0.95 on flat rows, so
the same reference code run on a GPU keeps every token of such rows.)
"""

from __future__ import annotations

from typing import Tuple

import torch


def sample_with_top_p(logits: torch.Tensor, top_p: float = 0.95,
                      temperature: float = 0.0) -> Tuple[torch.Tensor, torch.Tensor]:
    """(tokens, probs): argmax tokens and the top-p filtered probabilities over the
    last dimension (temperature 0; the reference scales by 1/temperature otherwise)."""
    if temperature > 0:
        logits = logits / temperature
    sorted_logits, sorted_indices = torch.sort(logits, descending=True, dim=-1)
    cumulative_probs = torch.cumsum(torch.softmax(sorted_logits, dim=-1), dim=-1)
    sorted_indices_to_remove = cumulative_probs > top_p
    sorted_indices_to_remove[..., 1:] = sorted_indices_to_remove[..., :-1].clone()
    sorted_indices_to_remove[..., 0] = False
    indices_to_remove = sorted_indices_to_remove.scatter(-1, sorted_indices, sorted_indices_to_remove)
    logits = logits.masked_fill(indices_to_remove, float("-inf"))
    probs = torch.softmax(logits, dim=-1)
    if temperature > 0:
        raise NotImplementedError("the oracle restates the greedy (temperature 0) path")
    return torch.argmax(probs, dim=-1), probs


def greedy_confidence(logits: torch.Tensor, top_p: float = 0.95) -> Tuple[torch.Tensor, torch.Tensor]:
    """(tokens, confidence of each token) as the decode loops use them
    (fastdllm_v2_generation.py:346-351): probs gathered at the sampled token."""
    tokens, probs = sample_with_top_p(logits, top_p=top_p, temperature=0.0)
    return tokens, torch.gather(probs, -1, tokens.unsqueeze(-1)).squeeze(-1)
