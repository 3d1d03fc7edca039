"""The decode loop's host logic on the CPU.

``specfold_b200.decode.FastDLLMV2Decoder`` restates the reference's decode loops
(fastdllm_v2_generation.py:188-385 and :483-720).  Here its device pieces -- the verify
forward, the sampler, the draft construction, the executor and the synchronisation --
are replaced by the CPU oracle (the restatements pinned to the reference), so the loop
itself (prefill, blocks and small blocks, the draft-logit cache and its hits, the
unmask rule, the commits, the stop tests and the token accounting) must reproduce the
golden runs of the reference's own loops bit for bit: tokens, model calls, drafts
computed and the branch count of every verify call.
"""
import os

import pytest
import torch

from oracle import folded_oracle as orc
from oracle.decode_standin import BiasedHead, GrowingCache, OracleExecutor
from oracle.drafts import fastdllm_draft_blocks
from oracle.sampling import greedy_confidence
from specfold_b200.decode import FastDLLMV2Decoder

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


class _Gen:
    """What the loop reads from its generator besides the hooks replaced below."""
    calibration_graph = None
    defer_stats = False

    def settle_stats(self):
        pass

    @staticmethod
    def _shift_logits(logits):
        return torch.cat([logits[:, :1, :], logits[:, :-1, :]], dim=1)


class _OracleExecutor(OracleExecutor):
    def new_cache(self, device):
        return GrowingCache(len(self.model.model.layers))


class OracleDecoder(FastDLLMV2Decoder):
    def __init__(self, model, delta, **kw):
        super().__init__(_Gen(), **kw)
        self.model = model
        self.delta = delta
        self._ex = _OracleExecutor(model, block=self.block_length)

    def executor(self, prompt_len):
        return self._ex

    def _verify(self, batched, cache):
        P = cache.get_seq_length()
        self.model.lm_head.base = P
        delta = self.delta if self.seam == "folded" else -1.0
        with torch.no_grad():
            return orc.folded_forward(self.model, batched, cache if P else None, delta)

    def _to_device(self, rows, dev):
        return torch.tensor(rows, dtype=torch.int64)

    def _sample(self, rows):
        return greedy_confidence(rows, self.top_p)

    def _drafts(self, block, logits, mask, s0, s1):
        out = fastdllm_draft_blocks(self.gen.calibration_graph, block, logits, mask,
                                    small_block_start=s0, small_block_end=s1)
        if not out:
            return None
        return torch.stack([d["state"] for d in out]), torch.ones(len(out), dtype=torch.int32)

    def _has_graph(self, dev):
        return self.gen.calibration_graph is not None

    def _sync(self, dev):
        pass


@pytest.mark.parametrize("mode", ["folded", "dense", "vanilla"])
def test_decode_loop_matches_reference_loop(mode):
    from tests.golden.make_decode_golden import BLOCK, DELTA, SMALL, THRESHOLD, TOP_P, build
    name = "decode_tiny_fp32"
    gold = torch.load(os.path.join(GOLDEN, f"{name}.pt"), weights_only=True)
    model, prompt, bias, graph, c = build(name)
    assert torch.equal(prompt, gold["prompt"])
    model.lm_head = BiasedHead(model.lm_head, bias)
    dec = OracleDecoder(model, DELTA, block_length=BLOCK, small_block_size=SMALL,
                        threshold=THRESHOLD, top_p=TOP_P, max_new_tokens=c["new"],
                        mask_id=c["mask_id"], stop_token=c["stop"],
                        calibration_graph=None if mode == "vanilla" else graph,
                        seam="dense" if mode == "dense" else "folded")
    if mode == "vanilla":
        tokens, st = dec.generate(prompt.tolist(), device="cpu")
    else:
        tokens, st = dec.generate_with_draft_speculation(prompt.tolist(), device="cpu")
    ref = gold[mode]
    assert tokens == ref["tokens"].tolist()
    assert st["model_calls"] == ref["model_calls"]
    assert st["drafts_computed"] == ref["drafts_computed"]
    if mode != "vanilla":
        assert [n for kind, n in st["steps"] if kind == "forward"] == ref["forwards"]
        assert st["draft_hits"] > 0
