"""CPU restatement of the reference's draft construction (the parity oracle).

TEST INFRASTRUCTURE ONLY: used by ``tests/``; never by the product path in
``specfold_b200``.

Restates, with the same torch op sequence,

* ``FastDLLMV2SpeculativeGeneration.get_draft_blocks``
  (specfold/generate/fastdllm_v2_generation.py:387-474): confidences from the softmax
  of the small block's logits in their own dtype, and
* ``NLDDiffusionGeneration.get_draft_blocks`` (specfold/generate/nld_generation.py:
  108-151): fp32 softmax over the whole block,

pinned bit for bit by ``tests/test_oracle_golden.py`` against ``tests/golden/drafts.pt``
(made by ``tests/golden/make_draft_golden.py`` with the reference's own methods).
"""

from __future__ import annotations

from typing import Dict, List, Optional

import torch


def fastdllm_draft_blocks(graph, x: torch.Tensor, p: torch.Tensor, mask_index: torch.Tensor,
                          start_pos=None, end_pos=None, small_block_start: Optional[int] = None,
                          small_block_end: Optional[int] = None) -> List[Dict]:
    if graph is None:
        return []
    if small_block_start is not None and small_block_end is not None:
        small_mask = mask_index[small_block_start:small_block_end] if mask_index is not None else None
        small_logits = p[small_block_start:small_block_end, :]
    else:
        small_mask, small_logits = mask_index, p
    if small_mask is None or small_mask.sum() == 0:
        return []
    out = []
    for node in graph.get("selected_nodes", []):
        ij_set = node.get("ij_set", [])
        if not ij_set:
            continue
        draft = x.clone()
        confidence = torch.softmax(small_logits, dim=-1).max(dim=-1).values
        confidence = torch.where(~small_mask, float("-inf"), confidence)
        max_pos_rank = max(r for r, _ in ij_set)
        if max_pos_rank >= small_mask.sum().item():
            continue
        _, top_positions = torch.topk(confidence, k=max_pos_rank + 1)
        for pos_rank, vocab_rank in ij_set:
            pos = top_positions[pos_rank]
            _, top_vocabs = torch.topk(small_logits[pos], k=vocab_rank + 1)
            off = small_block_start if small_block_start is not None else 0
            draft[off + pos] = top_vocabs[vocab_rank]
        out.append({"state": draft, "start_pos": start_pos, "end_pos": end_pos, "node": node})
    return out


def nld_draft_blocks(graph, x_block: torch.Tensor, logits_block: torch.Tensor,
                     mask_index: torch.Tensor) -> List[Dict]:
    nodes = [] if graph is None else [n for n in graph.get("selected_nodes", []) if n.get("ij_set")]
    if not nodes or mask_index.sum() == 0:
        return []
    confidence = torch.softmax(logits_block.float(), dim=-1).max(dim=-1).values
    confidence = torch.where(~mask_index, float("-inf"), confidence)
    n_mask = int(mask_index.sum().item())
    out = []
    for node in nodes:
        ij_set = node["ij_set"]
        max_pos_rank = max(r for r, _ in ij_set)
        if max_pos_rank >= n_mask:
            continue
        _, top_positions = torch.topk(confidence, k=max_pos_rank + 1)
        draft = x_block.clone()
        for pos_rank, vocab_rank in ij_set:
            pos = top_positions[pos_rank]
            _, top_vocabs = torch.topk(logits_block[pos], k=vocab_rank + 1)
            draft[pos] = top_vocabs[vocab_rank]
        out.append({"state": draft, "node": node})
    return out
