"""CPU stand-ins for what the reference's decoding loop needs besides the folded forward.

TEST INFRASTRUCTURE ONLY: used by ``tests/golden/make_decode_golden.py`` (which runs the
reference's own ``FastDLLMV2SpeculativeGeneration.generate_with_draft_speculation``,
specfold/generate/fastdllm_v2_generation.py:483-720, and ``generate``, :188-385, on the
CPU) and by the tests; never by the product path in ``specfold_b200``.

* ``OracleExecutor`` -- the model executor (specfold/generate/fastdllm_model_executor.py:
  59-107).  The Fast-dLLM v2 model code behind it is HF remote code that is not in the
  reference checkout, so its forward is restated as what the folded path already
  defines: the dense block forward (the oracle's folded forward at a negative threshold,
  every row recomputed; fastdllm_v2_folded.py:6), one block of ``block`` tokens at a
  time, each attending bidirectionally to itself and to everything before it
  (block-causal, the block-diffusion pattern the decode loop itself commits in).  With
  ``update_past_key_values`` every block's keys (after RoPE) and values are appended to
  the cache the way ``DynamicCache.update`` does (a ``torch.cat`` per layer).  Returns
  the unshifted logits, as the model does.
* ``BiasedHead`` -- the synthetic model's LM head: the wrapped head's output plus the
  seeded per-position logit bias (``specfold_b200.synthetic.DecodeBias``) at the rows'
  absolute positions; the executor and the golden generator set ``base`` to the prefix
  length before each forward.
* ``IdTokenizer`` -- maps a prompt key to its token ids and back.
"""

from __future__ import annotations

import types
from typing import Dict, List, Optional

import torch

from . import folded_oracle as orc


class GrowingCache:
    """Prefix cache with the reads the folded forward makes (``get_seq_length``, ``len``,
    ``[li] -> (k, v)``, iteration) and ``DynamicCache.update``'s append by concatenation."""

    def __init__(self, num_layers: int):
        self.keys: List[Optional[torch.Tensor]] = [None] * num_layers
        self.values: List[Optional[torch.Tensor]] = [None] * num_layers

    def get_seq_length(self, layer_idx: int = 0) -> int:
        k = self.keys[layer_idx]
        return 0 if k is None else int(k.shape[-2])

    def __len__(self) -> int:
        return 0 if self.keys[0] is None else len(self.keys)

    def __getitem__(self, li):
        return self.keys[li], self.values[li]

    def __iter__(self):
        return iter(zip(self.keys, self.values))

    def update(self, k: torch.Tensor, v: torch.Tensor, li: int):
        self.keys[li] = k if self.keys[li] is None else torch.cat([self.keys[li], k], dim=-2)
        self.values[li] = v if self.values[li] is None else torch.cat([self.values[li], v], dim=-2)
        return self.keys[li], self.values[li]


class BiasedHead(torch.nn.Module):
    """``head(x)`` plus the decode bias: output row n of a block whose first position is
    ``base`` predicts position base + n + 1 (Fast-dLLM, before the logit shift)."""

    def __init__(self, head: torch.nn.Module, bias):
        super().__init__()
        self.head = head
        self.bias = bias
        self.base = 0

    @property
    def weight(self):
        return self.head.weight

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = self.head(x)
        n = y.shape[-2]
        pred = torch.arange(self.base + 1, self.base + 1 + n)
        return self.bias.apply(y, pred)


class OracleExecutor:
    """``FastDLLMModelExecutor`` stand-in on the oracle (see the module docstring)."""

    def __init__(self, model, tokenizer=None, block: int = 32, family: str = "fastdllm",
                 sampler=None):
        self.model = model
        self.tokenizer = tokenizer
        self.block = block
        self.family = family
        self._sampler = sampler
        self.calls = 0

    def _head(self):
        return self.model.lm_head

    def forward(self, input_seq: torch.Tensor, past_key_values=None, use_cache: bool = True,
                update_past_key_values: bool = False, **kwargs):
        B, T = input_seq.shape
        assert B == 1, "batch-1 decoding"
        cache = past_key_values
        if cache is None:
            cache = GrowingCache(len(self.model.model.layers))
        outs = []
        for s in range(0, T, self.block):
            blk = input_seq[:, s:s + self.block]
            P = cache.get_seq_length()
            head = self._head()
            if isinstance(head, BiasedHead):
                head.base = P
            cap = orc.Capture() if update_past_key_values else None
            with torch.no_grad():
                logits = orc.folded_forward(self.model, blk, cache if P > 0 else None, -1.0,
                                            family=self.family, capture=cap, shift=False)
            outs.append(logits)
            if update_past_key_values:
                for li, lay in enumerate(cap.layers):
                    cache.update(lay["k"][0:1].clone(), lay["v"][0:1].clone(), li)
            elif s + self.block < T:
                raise ValueError("a forward without a cache update covers one block")
        self.calls += 1
        return types.SimpleNamespace(logits=torch.cat(outs, dim=1),
                                     past_key_values=cache if update_past_key_values else past_key_values)

    def sample_with_top_p(self, logits, top_p=0.95, temperature=0.0):
        return self._sampler(self, logits, top_p=top_p, temperature=temperature)

    def get_tokenizer(self):
        return self.tokenizer


class IdTokenizer:
    """Prompt key -> token ids (``input_ids`` [1, T]); ids -> space-separated text."""

    def __init__(self, prompts: Dict[str, torch.Tensor]):
        self.prompts = prompts

    def __call__(self, text, return_tensors="pt"):
        return types.SimpleNamespace(input_ids=self.prompts[text].view(1, -1).clone())

    def batch_decode(self, ids, skip_special_tokens=True):
        return [" ".join(str(int(t)) for t in row) for row in ids]
