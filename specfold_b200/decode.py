"""End-to-end decoding on the B200 kernels: the reference's decode loops with the folded
verify forward, the block commit, the sampler and the draft construction all on the GPU.

``FastDLLMV2SpeculativeGeneration.generate_with_draft_speculation``
(specfold/generate/fastdllm_v2_generation.py:483-720) and ``generate`` (:188-385) are the
loops a SpecFold run drives; inside a Python process that has the reference, mixing
``SpecFoldB200FastDLLMV2Generation`` in front of them is the drop-in (folded.py).  This
module restates the two loops step for step for processes without the reference (the
GPU boxes, the benchmark) -- same prefill, block and small-block structure, draft-logit
cache and hit test, unmask rule (threshold in the logits' dtype plus the most confident
masked position), stop-token checks and token accounting -- with one difference in
*where* the bookkeeping lives: the block's token ids are kept on the host, where every
decision of the loop is taken anyway, so that a step costs one device synchronisation
(the sampled tokens, their confidences and the next drafts come back together) instead
of the reference's several small ones.  The results -- tokens, model calls, drafts
computed, cache hits -- are those of the reference loop.

``B200Executor`` stands in for ``FastDLLMModelExecutor.forward`` (fastdllm_model_executor.
py:59-107), whose Fast-dLLM v2 model code is HF remote code outside the reference: the
prefill and the block commit run the dense block forward on the same kernels with a
block-causal pattern (each block attends bidirectionally to itself and to every earlier
block) and append the blocks' keys and values to a preallocated cache inside the forward:
``commit_block_forward`` for one block, ``prefill_forward`` for up to 16 prompt blocks per
forward.
"""

from __future__ import annotations

import time
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import kernels as K
from .kv_cache import PreallocatedKVCache


class ExecutorOutput:
    __slots__ = ("logits", "past_key_values")

    def __init__(self, logits, past_key_values):
        self.logits = logits
        self.past_key_values = past_key_values


class B200Executor:
    """``forward(input_seq, past_key_values, use_cache, update_past_key_values)`` of the
    model executor on the B200 kernels (see the module docstring); logits unshifted.

    ``generator`` is a ``SpecFoldB200*Generation`` (it owns the packed weights and the
    per-configuration state); ``capacity`` sizes a new cache (rows per layer)."""

    def __init__(self, generator, block: int = 32, capacity: int = 4096, logit_bias=None,
                 all_logits: bool = False):
        self.gen = generator
        self.block = block
        self.capacity = capacity
        self.logit_bias = logit_bias
        # False: a multi-block prefill returns the logits of its last block only (the rows
        # the loops read); True: of every block, as the model's forward does
        self.all_logits = all_logits
        # True: multi-block prompts use the batched block-causal prefill forward
        self.batched_prefill = True
        self.model = generator.model_executor.model

    def new_cache(self, device) -> PreallocatedKVCache:
        cfg = self.model.config
        base = self.gen._base()
        hd = base.layers[0].self_attn.head_dim
        dtype = base.layers[0].self_attn.q_proj.weight.dtype
        return PreallocatedKVCache(len(base.layers), cfg.num_key_value_heads, hd,
                                   self.capacity, dtype=dtype, device=device)

    def _bias(self, logits, P):
        if self.logit_bias is not None:
            n = logits.shape[-2]
            pred = torch.arange(P + 1, P + 1 + n, device=logits.device)
            self.logit_bias.apply(logits, pred)
        return logits

    @torch.no_grad()
    def forward(self, input_seq: torch.Tensor, past_key_values=None, use_cache: bool = True,
                update_past_key_values: bool = False, **kwargs) -> ExecutorOutput:
        if input_seq.dim() != 2 or input_seq.shape[0] != 1:
            raise ValueError(f"batch-1 decoding: input [1, T], got {tuple(input_seq.shape)}")
        cache = past_key_values if past_key_values is not None else self.new_cache(input_seq.device)
        if not isinstance(cache, PreallocatedKVCache):
            raise TypeError("the B200 executor keeps the prefix in a PreallocatedKVCache")
        T = input_seq.shape[1]
        if not update_past_key_values:
            if T != self.block:
                raise ValueError("a forward without a cache update covers one block")
            P = cache.get_seq_length()
            cache.reserve(T)
            logits, _ = self.gen._run(input_seq, cache, T, count_stats=False, delta=-1.0,
                                      shift=False)
            return ExecutorOutput(self._bias(logits, P), past_key_values)
        if T % self.block:
            raise ValueError(f"prefill / commit of {T} tokens: a multiple of {self.block} expected")
        # every block is committed; the logits of the last one are the ones the loops read
        # (the next token, fastdllm_v2_generation.py:522-524 / :571).  A multi-block
        # prompt goes through the batched block-causal prefill (one forward per 16 blocks,
        # the same attention pattern as committing the blocks one by one) unless every
        # block's logits are wanted
        P0 = cache.get_seq_length()
        if T > self.block and not self.all_logits and self.batched_prefill:
            lg = self.gen.prefill_forward(input_seq, cache, self.block, logits=True)
            return ExecutorOutput(self._bias(lg, P0 + T - self.block), cache)
        outs = []
        for s in range(0, T, self.block):
            P = cache.get_seq_length()
            last = s + self.block >= T
            lg = self.gen.commit_block_forward(input_seq[:, s:s + self.block], cache,
                                               logits=last or self.all_logits)
            if lg is not None:
                outs.append(self._bias(lg, P))
        return ExecutorOutput(outs[0] if len(outs) == 1 else torch.cat(outs, dim=1), cache)


class DecodeStats(dict):
    """tokens_generated, model_calls, drafts_computed, draft_hits, elapsed_s, tok_s,
    fold_ratio, steps (forward or hit per loop iteration)."""


class FastDLLMV2Decoder:
    """The reference's Fast-dLLM v2 decode loops (fastdllm_v2_generation.py:188-385 and
    :483-720) over the B200 generator.

    ``seam`` selects the verify forward: "folded" (the SpecFold path, the generator's
    ``_batched_block_forward``) or "dense" (every branch computed in full, the base
    class's unfolded multi-branch forward).  ``logit_bias`` (synthetic.DecodeBias) is
    added to every logits tensor the model produces, at the rows' predicted positions."""

    def __init__(self, generator, block_length: int = 32, small_block_size: int = 8,
                 threshold: float = 0.9, top_p: float = 0.95, max_new_tokens: int = 256,
                 mask_id: int = 151665, stop_token: int = 151645, calibration_graph=None,
                 logit_bias=None, capacity: Optional[int] = None, seam: str = "folded"):
        if seam not in ("folded", "dense"):
            raise ValueError(f"seam {seam!r}")
        self.gen = generator
        self.block_length = int(block_length)
        self.small_block_size = int(small_block_size)
        self.threshold = float(threshold)
        self.top_p = float(top_p)
        self.max_new_tokens = int(max_new_tokens)
        self.mask_id = int(mask_id)
        self.stop_token = int(stop_token)
        self.logit_bias = logit_bias
        self.seam = seam
        self.capacity = capacity
        generator.calibration_graph = calibration_graph
        generator.defer_stats = True
        self._executor = None
        self._stage = None          # pinned staging of the batched block ids

    # ------------------------------------------------------------------ helpers
    def executor(self, prompt_len: int) -> B200Executor:
        cap = self.capacity or (prompt_len + self.max_new_tokens + 2 * self.block_length)
        if self._executor is None or self._executor.capacity < cap:
            self._executor = B200Executor(self.gen, self.block_length, cap, self.logit_bias)
        return self._executor

    def _threshold_in(self, dtype) -> torch.Tensor:
        # the reference compares the logits-dtype confidences with a Python float, which
        # torch casts to that dtype (0.9 -> 0.8984375 in bf16)
        return torch.tensor(self.threshold, dtype=dtype)

    def _verify(self, batched: torch.Tensor, cache) -> torch.Tensor:
        """The seam over [B1, N] -> shifted logits [B1, N, V] with the bias applied."""
        P = cache.get_seq_length()
        if hasattr(cache, "reserve"):
            cache.reserve(batched.shape[1])
        if self.seam == "folded":
            logits = self.gen._batched_block_forward(batched, cache)
        else:
            logits = self.gen.dense_block_forward(batched, cache)
        if self.logit_bias is not None:
            N = batched.shape[1]
            # shifted row n holds the prediction of position P + n (row 0: a copy of the
            # row predicting P + 1); offsets kept on the device, no host round trip
            off = self.__dict__.get("_pred_off")
            if off is None or off.numel() != N or off.device != logits.device:
                off = torch.arange(N, device=logits.device)
                off[0] = 1
                self._pred_off = off
            self.logit_bias.apply(logits, off + P)
        return logits

    def _to_device(self, rows: List[List[int]], dev) -> torch.Tensor:
        """[B1, N] int64 on the device from host rows, through a pinned buffer (the previous
        copy out of it has completed: every step ends in a synchronisation)."""
        n = len(rows) * len(rows[0])
        if self._stage is None or self._stage.numel() < n:
            self._stage = torch.empty(max(n, 16 * self.block_length), dtype=torch.int64).pin_memory()
        st = self._stage[:n]
        st.copy_(torch.tensor(rows, dtype=torch.int64).view(-1))
        return st.to(dev, non_blocking=True).view(len(rows), -1)

    def _sample(self, logits_rows: torch.Tensor):
        """tokens, confidences (logits dtype) of rows [R, V] on the GPU."""
        return K.sample_top_p_greedy(logits_rows, self.top_p)

    def _drafts(self, block: torch.Tensor, logits: torch.Tensor, mask: torch.Tensor, s0: int,
                s1: int):
        """(drafts [n_nodes, N], valid [n_nodes]) of the calibration graph from the main
        block's logits [N, V] over the small block [s0, s1) (mask [N]: masked positions),
        left on the device; None when the graph has no usable node."""
        nodes, drafts, valid = self.gen._draft_states_async(block, logits[s0:s1], mask[s0:s1], s0)
        return (drafts, valid) if nodes else None

    def _has_graph(self, dev) -> bool:
        return bool(getattr(self.gen, "calibration_graph", None)) and \
            self.gen._graph_pairs(dev) is not None

    def _sync(self, dev) -> None:
        torch.cuda.current_stream(dev).synchronize()

    @staticmethod
    def _stop_reached(x: List[int], prompt_length: int, stop: int, mask: int) -> bool:
        """The reference's in-block stop test (fastdllm_v2_generation.py:550-555): a stop
        token after the block start with no mask before it."""
        gen = x[prompt_length:]
        if stop not in gen:
            return False
        k = gen.index(stop)
        return mask not in gen[:k]

    def _unmask(self, x: List[int], s0: int, s1: int, small_mask: List[bool], tokens, conf):
        """The commit rule of fastdllm_v2_generation.py:667-700 on the host: positions
        whose confidence exceeds the threshold, plus the most confident masked one (the
        first of equal maxima, as torch.argmax).  The confidences are the logits dtype's
        values, exactly representable as Python floats, and the threshold is that dtype's
        rounding of it, so the comparisons are the reference's."""
        thr = float(self._threshold_in(conf.dtype))
        c = conf.tolist()
        tk = tokens.tolist()
        best, best_j = float("-inf"), 0
        pick = []
        for j, m in enumerate(small_mask):
            v = c[j] if m else float("-inf")
            if v > best:
                best, best_j = v, j
            if m and v > thr:
                pick.append(j)
        if small_mask[best_j] and best_j not in pick:
            pick.append(best_j)
        base = len(x) - self.block_length + s0
        for j in pick:
            x[base + j] = int(tk[j])

    def _finish(self, x, orig_len, t0, model_calls, drafts, hits, steps, fold0, dev):
        self.gen.settle_stats()
        self._sync(dev)
        elapsed = time.perf_counter() - t0
        final = x[orig_len:]
        if self.stop_token in final:
            final = final[:final.index(self.stop_token) + 1]
        tokens = [t for t in final if t != self.mask_id]
        pos = getattr(self.gen, "_fold_draft_positions", 0) - fold0[0]
        rec = getattr(self.gen, "_fold_draft_recomputed", 0) - fold0[1]
        return tokens, DecodeStats(tokens_generated=len(tokens), model_calls=model_calls,
                                   drafts_computed=drafts, draft_hits=hits, elapsed_s=elapsed,
                                   tok_s=len(tokens) / elapsed if elapsed > 0 else 0.0,
                                   fold_ratio=(1.0 - rec / pos) if pos else float("nan"),
                                   steps=steps)

    def _prefill(self, x: List[int], dev):
        """Prefill of the prompt's whole blocks (fastdllm_v2_generation.py:510-524)."""
        bl = self.block_length
        ex = self.executor(len(x))
        cache = ex.new_cache(dev)
        calls = 0
        if len(x) > bl:
            n = (len(x) // bl) * bl
            out = ex.forward(torch.tensor([x[:n]], device=dev), cache, use_cache=True,
                             update_past_key_values=True)
            calls += 1
            if len(x) % bl == 0:
                x.append(int(out.logits[0, -1].argmax()))
        return cache, calls

    def _commit(self, x: List[int], cache, dev):
        """All masks filled: the commit forward, then the next block's first token
        (fastdllm_v2_generation.py:559-575)."""
        bl = self.block_length
        out = self.executor(len(x)).forward(torch.tensor([x[-bl:]], device=dev), cache,
                                            use_cache=True, update_past_key_values=True)
        x.append(int(out.logits[0, -1].argmax()))

    # ------------------------------------------------------------------ the loops
    @torch.no_grad()
    def generate_with_draft_speculation(self, prompt_ids: Sequence[int], device="cuda"
                                        ) -> Tuple[List[int], DecodeStats]:
        """fastdllm_v2_generation.py:483-720 (see the module docstring)."""
        dev = torch.device(device)
        self._sync(dev)
        t0 = time.perf_counter()
        fold0 = (getattr(self.gen, "_fold_draft_positions", 0),
                 getattr(self.gen, "_fold_draft_recomputed", 0))
        bl, sbs = self.block_length, self.small_block_size
        mask, stop = self.mask_id, self.stop_token
        x = [int(t) for t in prompt_ids]
        orig_len = len(x)
        cache, model_calls = self._prefill(x, dev)
        drafts_computed = hits = 0
        steps: List[Tuple[str, int]] = []
        graph = self._has_graph(dev)
        draft_states: List[List[int]] = []          # the reference's draft_blocks
        called: List[Tuple[List[int], torch.Tensor]] = []   # its called_drafts
        for _ in range(self.max_new_tokens // bl):
            if stop in x[orig_len:]:
                break
            prompt_length = len(x)
            x += [mask] * (bl - prompt_length % bl)
            while True:
                if self._stop_reached(x, prompt_length, stop, mask):
                    break
                block = x[-bl:]
                if mask not in block:
                    self._commit(x, cache, dev)
                    model_calls += 1
                    draft_states, called = [], []
                    break
                for sb in range(bl // sbs):
                    s0, s1 = sb * sbs, sb * sbs + sbs
                    while True:
                        block = x[-bl:]
                        mask_row = [t == mask for t in block]
                        small = mask_row[s0:s1]
                        if not any(small):
                            break
                        if self._stop_reached(x, prompt_length, stop, mask):
                            break
                        hit = next((i for i, (st, _) in enumerate(called) if st == block), -1)
                        if hit >= 0:
                            _, lg = called.pop(hit)
                            tok, conf = self._sample(lg[0, s0:s1])
                            tok, conf = tok.cpu(), conf.cpu()
                            hits += 1
                            steps.append(("hit", 0))
                        else:
                            rows = [block] + draft_states
                            batched = self._to_device(rows, dev)
                            logits = self._verify(batched, cache)
                            model_calls += 1
                            steps.append(("forward", len(rows)))
                            for i, st in enumerate(draft_states):
                                called.append((st, logits[i + 1:i + 2]))
                            tok_d, conf_d = self._sample(logits[0, s0:s1])
                            pending = [tok_d, conf_d]
                            new_states: List[List[int]] = []
                            if graph:
                                # the next drafts from this step's main logits
                                # (fastdllm_v2_generation.py:653-664)
                                blk_dev = batched[0]
                                dv = self._drafts(blk_dev, logits[0], blk_dev == mask, s0, s1)
                                if dv is not None:
                                    pending += list(dv)
                            host = [t.to("cpu", non_blocking=True) for t in pending]
                            self._sync(dev)
                            tok, conf = host[0], host[1]
                            if len(host) > 2:
                                dr, vd = host[2].tolist(), host[3].tolist()
                                new_states = [dr[k] for k in range(len(dr)) if vd[k]]
                            if graph:
                                draft_states = new_states
                                drafts_computed += len(new_states)
                        self._unmask(x, s0, s1, small, tok, conf)
        return self._finish(x, orig_len, t0, model_calls, drafts_computed, hits, steps, fold0, dev)

    @torch.no_grad()
    def generate(self, prompt_ids: Sequence[int], device="cuda") -> Tuple[List[int], DecodeStats]:
        """The vanilla loop without speculation (fastdllm_v2_generation.py:188-385): one
        dense forward of the main block per step through the executor."""
        dev = torch.device(device)
        self._sync(dev)
        t0 = time.perf_counter()
        bl, sbs = self.block_length, self.small_block_size
        mask, stop = self.mask_id, self.stop_token
        x = [int(t) for t in prompt_ids]
        orig_len = len(x)
        cache, model_calls = self._prefill(x, dev)
        ex = self.executor(len(x))
        steps: List[Tuple[str, int]] = []
        for _ in range(self.max_new_tokens // bl):
            if stop in x[orig_len:]:
                break
            prompt_length = len(x)
            x += [mask] * (bl - prompt_length % bl)
            while True:
                if self._stop_reached(x, prompt_length, stop, mask):
                    break
                block = x[-bl:]
                if mask not in block:
                    self._commit(x, cache, dev)
                    model_calls += 1
                    break
                for sb in range(bl // sbs):
                    s0, s1 = sb * sbs, sb * sbs + sbs
                    while True:
                        block = x[-bl:]
                        small = [t == mask for t in block[s0:s1]]
                        if not any(small):
                            break
                        if self._stop_reached(x, prompt_length, stop, mask):
                            break
                        out = ex.forward(torch.tensor([block], device=dev), cache, use_cache=True,
                                         update_past_key_values=False)
                        logits = self.gen._shift_logits(out.logits)
                        model_calls += 1
                        steps.append(("forward", 1))
                        tok, conf = self._sample(logits[0, s0:s1])
                        self._unmask(x, s0, s1, small, tok.cpu(), conf.cpu())
        return self._finish(x, orig_len, t0, model_calls, 0, 0, steps, (0, 0), dev)
