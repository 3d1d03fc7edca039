"""Seeded synthetic stand-ins for the models, prefix caches and block inputs that the
reference's folded verify forward runs on.

The reference loads Fast-dLLM v2 (Qwen2 architecture) and Nemotron-Labs-Diffusion
(Ministral3 / Llama-style) checkpoints (``specfold/registry.py:27-68``).  Neither the
checkpoints nor any dataset exist on these machines, so every test and benchmark uses
random-init weights of the named architecture shapes:

* Fast-dLLM family: ``transformers.Qwen2ForCausalLM`` (QKV bias, RMSNorm eps 1e-6,
  logit shift), the attributes ``_batched_block_forward`` reads
  (``fastdllm_v2_folded.py:96-103,118-121,152-156,208,214-216,222-223``).
* NLD family: ``transformers.LlamaForCausalLM`` wrapped so that ``.encoder`` is the
  decoder stack and ``.diffusion_head`` the LM head (``nld_folded.py:111-113,241``),
  no QKV bias, eps 1e-5, no logit shift.

Weights are drawn N(0, 0.02) from a seeded ``torch.Generator`` (norm gains 1), the
prefix K/V cache N(0, 1), as the benchmark configurations prescribe.
"""

from __future__ import annotations

import dataclasses
import math
from typing import Dict, List, Optional, Sequence, Tuple

import torch


@dataclasses.dataclass(frozen=True)
class ModelDims:
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    inter: int
    layers: int
    vocab: int
    eps: float = 1e-6
    theta: float = 1e6

    @property
    def q_dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    def weight_bytes(self, elt: int = 2) -> int:
        """Bytes of every weight the verify step streams (layers + lm_head)."""
        per_layer = (self.hidden * (self.q_dim + 2 * self.kv_dim) + self.q_dim * self.hidden
                     + 3 * self.hidden * self.inter)
        return elt * (self.layers * per_layer + self.hidden * self.vocab)


# Shapes named by the benchmark configurations.
SHAPES: Dict[str, ModelDims] = {
    # small shapes for golden vectors and fast parity tests
    "tiny": ModelDims(hidden=256, heads=4, kv_heads=2, head_dim=64, inter=384, layers=2, vocab=128),
    "tiny128": ModelDims(hidden=512, heads=4, kv_heads=2, head_dim=128, inter=768, layers=2, vocab=256),
    # config 0: one Qwen2.5-1.5B-shape layer (vocab stand-in; config 0 has no head)
    "qwen1.5b-1layer": ModelDims(hidden=1536, heads=12, kv_heads=2, head_dim=128, inter=8960,
                                 layers=1, vocab=1024),
    # config 1: full Qwen2.5-1.5B shape
    "qwen1.5b": ModelDims(hidden=1536, heads=12, kv_heads=2, head_dim=128, inter=8960,
                          layers=28, vocab=151936),
    # config 2: Qwen2.5-7B shape
    "qwen7b": ModelDims(hidden=3584, heads=28, kv_heads=4, head_dim=128, inter=18944,
                        layers=28, vocab=152064),
    # config 3: Llama-style 8B shape (kernel microbenchmark)
    "llama8b": ModelDims(hidden=4096, heads=32, kv_heads=8, head_dim=128, inter=14336,
                         layers=32, vocab=128256, eps=1e-5, theta=5e5),
    # config 4: Llama-style 14B shape
    "llama14b": ModelDims(hidden=5120, heads=40, kv_heads=8, head_dim=128, inter=13824,
                          layers=40, vocab=131072, eps=1e-5, theta=5e5),
}


def _init_(module: torch.nn.Module, gen: torch.Generator, std: float = 0.02) -> None:
    """N(0, std) for every matrix and bias, 1 for norm gains; drawn on the CPU generator
    (device-independent) in parameter order, then copied to the module's device."""
    for name, p in module.named_parameters():
        if name.endswith("norm.weight") or "layernorm" in name:
            with torch.no_grad():
                p.fill_(1.0)
            continue
        cpu = torch.empty(p.shape, dtype=torch.float32).normal_(0.0, std, generator=gen)
        with torch.no_grad():
            p.copy_(cpu.to(p.dtype))


def _init_fast_(module: torch.nn.Module, seed: int, std: float = 0.02) -> None:
    """Device-side variant of :func:`_init_` for multi-GB shapes (same distribution,
    draws on the module's device generator)."""
    dev = next(module.parameters()).device
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    for name, p in module.named_parameters():
        with torch.no_grad():
            if name.endswith("norm.weight") or "layernorm" in name:
                p.fill_(1.0)
            else:
                p.normal_(0.0, std, generator=gen)


class StandinExecutor:
    """Holds ``.model`` the way ``FastDLLMModelExecutor`` / ``NLDModelExecutor`` do
    (``fastdllm_model_executor.py:36-41``, ``nld_model_executor.py:34-41``)."""

    def __init__(self, model: torch.nn.Module):
        self.model = model


class NLDStandin(torch.nn.Module):
    """Llama decoder exposed under the NLD attribute names ``encoder`` /
    ``diffusion_head`` (``modeling_nemotron_labs_diffusion.py``)."""

    def __init__(self, llama):
        super().__init__()
        self.config = llama.config
        self.encoder = llama.model
        self.diffusion_head = llama.lm_head


def build_model(dims: ModelDims, family: str = "fastdllm", dtype=torch.float32, seed: int = 0,
                device: str = "cpu") -> torch.nn.Module:
    """Random-init stand-in of the given shape. ``family`` is "fastdllm" (Qwen2) or
    "nld" (Llama wrapped as NLD)."""
    import transformers

    common = dict(hidden_size=dims.hidden, intermediate_size=dims.inter,
                  num_attention_heads=dims.heads, num_key_value_heads=dims.kv_heads,
                  head_dim=dims.head_dim, num_hidden_layers=dims.layers, vocab_size=dims.vocab,
                  rms_norm_eps=dims.eps, max_position_embeddings=65536, tie_word_embeddings=False)
    if family == "fastdllm":
        cfg = transformers.Qwen2Config(rope_theta=dims.theta, **common)
        ctor = transformers.Qwen2ForCausalLM
    elif family == "nld":
        cfg = transformers.LlamaConfig(rope_theta=dims.theta, attention_bias=False,
                                       mlp_bias=False, **common)
        ctor = transformers.LlamaForCausalLM
    else:
        raise ValueError(f"unknown family {family!r}")
    cfg._attn_implementation = "eager"
    big = dims.weight_bytes() > (2 << 30)
    with torch.device(device):
        model = ctor(cfg).to(dtype).eval()
    if big and device != "cpu":
        _init_fast_(model, seed)
    else:
        gen = torch.Generator().manual_seed(seed)
        _init_(model, gen)
    if family == "nld":
        model = NLDStandin(model).eval()
    return model


class PrefixCache:
    """Read-only prefix KV cache with the four calls the folded forward makes on
    ``past_key_values`` (``fastdllm_v2_folded.py:104,122-123``): ``get_seq_length``,
    ``len``, ``[li] -> (k, v)`` with k, v shaped [1, Hkv, P, hd], and iteration."""

    def __init__(self, keys: List[torch.Tensor], values: List[torch.Tensor]):
        assert len(keys) == len(values)
        self.keys = keys
        self.values = values

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return int(self.keys[layer_idx].shape[-2]) if self.keys else 0

    def __len__(self) -> int:
        return len(self.keys)

    def __getitem__(self, li: int) -> Tuple[torch.Tensor, torch.Tensor]:
        return self.keys[li], self.values[li]

    def __iter__(self):
        return iter(zip(self.keys, self.values))

    def to(self, device) -> "PrefixCache":
        return PrefixCache([k.to(device) for k in self.keys], [v.to(device) for v in self.values])


def random_prefix_cache(dims: ModelDims, P: int, dtype=torch.float32, seed: int = 1,
                        device: str = "cpu") -> Optional[PrefixCache]:
    """Prefix K/V ~ N(0, 1), one [1, Hkv, P, hd] pair per layer (None when P == 0)."""
    if P == 0:
        return None
    gen = torch.Generator(device=device if device != "cpu" else "cpu").manual_seed(seed)
    ks, vs = [], []
    for _ in range(dims.layers):
        shape = (1, dims.kv_heads, P, dims.head_dim)
        ks.append(torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dtype))
        vs.append(torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dtype))
    return PrefixCache(ks, vs)


# ----------------------------------------------------------------------------- drafts

DEFAULT_TREE: Tuple[int, ...] = (0, 0, 1, 1, 2, 0, 5)   # parent of drafts 1..7 (0 = main)


def tree_block_input(vocab: int, N: int = 32, parents: Sequence[int] = DEFAULT_TREE,
                     edits_per_level: int = 1, seed: int = 2,
                     mask_id: Optional[int] = None) -> torch.Tensor:
    """[B1, N] token block: row 0 is the main block; draft i copies its parent's row
    and re-fills ``edits_per_level`` positions the parent did not change, so the
    differing-position sets nest the way the calibration-graph drafts do
    (``fastdllm_v2_generation.py:434-465``).  With ``edits_per_level == 1`` the parent
    map (``fastdllm_v2_folded.py:55-75``) finds a chain of the same depth; it compares
    position sets only, so it may pick another branch whose set is also a subset."""
    gen = torch.Generator().manual_seed(seed)
    B1 = len(parents) + 1
    rows = torch.empty(B1, N, dtype=torch.int64)
    hi = vocab if mask_id is None else mask_id
    rows[0] = torch.randint(0, hi, (N,), generator=gen)
    changed: List[set] = [set()]
    for i, p in enumerate(parents, start=1):
        assert p < i, "parents must precede children"
        rows[i] = rows[p]
        free = [n for n in range(N) if n not in changed[p]]
        perm = torch.randperm(len(free), generator=gen)[:edits_per_level].tolist()
        pos = [free[j] for j in perm]
        for n in pos:
            old = int(rows[p, n])
            new = int(torch.randint(0, hi - 1, (1,), generator=gen))
            rows[i, n] = new if new < old else new + 1   # guaranteed to differ
        changed.append(changed[p] | set(pos))
    return rows


def noise_hidden(base: torch.Tensor, B1: int, frac_recompute: float = 0.4,
                 sigma_fold: float = 0.01, sigma_rec: float = 0.5, seed: int = 3) -> torch.Tensor:
    """Configuration-0 injection: draft rows = main hidden + noise.  A seeded
    ``frac_recompute`` share of draft rows gets sigma_rec noise (recomputed at
    delta = 0.1), the rest sigma_fold (folded).  ``base`` is the main block [N, D]."""
    gen = torch.Generator().manual_seed(seed)
    N, D = base.shape
    out = base.unsqueeze(0).repeat(B1, 1, 1).float()
    nd = (B1 - 1) * N
    n_rec = int(round(frac_recompute * nd))
    order = torch.randperm(nd, generator=gen)
    sig = torch.full((nd,), sigma_fold)
    sig[order[:n_rec]] = sigma_rec
    eps = torch.randn(nd, D, generator=gen) * sig[:, None]
    out[1:] += eps.view(B1 - 1, N, D)
    return out.to(base.dtype)


class InjectedEmbedding(torch.nn.Module):
    """Stands in for ``embed_tokens``: returns a fixed seeded hidden block instead of a
    table lookup, so configuration 0's "main hidden + noise" rows enter layer 0 of the
    folded forward (``fastdllm_v2_folded.py:110``)."""

    def __init__(self, hidden: torch.Tensor):
        super().__init__()
        self.register_buffer("hidden", hidden, persistent=False)

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        assert ids.shape == self.hidden.shape[:2], (ids.shape, self.hidden.shape)
        return self.hidden.to(ids.device)


def inject_hidden(model: torch.nn.Module, hidden: torch.Tensor) -> None:
    base = model.encoder if hasattr(model, "encoder") else model.model
    base.embed_tokens = InjectedEmbedding(hidden)


def config0_hidden(dims: ModelDims, B1: int = 8, N: int = 32, dtype=torch.float32,
                   seed: int = 3, frac_recompute: float = 0.4) -> torch.Tensor:
    """Main hidden x0 ~ N(0, 1) [N, D] plus per-draft-row noise (60% sigma 0.01,
    40% sigma 0.5)."""
    gen = torch.Generator().manual_seed(seed + 1000)
    x0 = torch.randn(N, dims.hidden, generator=gen)
    return noise_hidden(x0, B1, frac_recompute=frac_recompute, seed=seed).to(dtype)


# ----------------------------------------------------------------------------- decoding
# The end-to-end decode configurations generate from random-init models, whose logits
# carry no signal.  A seeded per-position logit bias stands in for a trained model's
# confidence: for every generated position q it names a target token and a strength, and
# the model's output row that predicts q (Fast-dLLM: the row before q, which the logit
# shift moves onto q; fastdllm_v2_generation.py:121-126) gets the strength added at the
# target's column.  "strong" positions reach a top-p confidence of 1 and are committed by
# the threshold test in the first step they are masked; "weak" ones stay below it and are
# committed one per step by the max-confidence rule (fastdllm_v2_generation.py:673-676),
# their strengths spaced so that the order of commits is set by the bias rather than by
# rounding noise; "free" positions (no bias) take the model's own argmax.


@dataclasses.dataclass
class DecodeBias:
    """target[q] (int64, -1 = free) and strength[q] (float32) per absolute position q."""
    target: torch.Tensor
    strength: torch.Tensor

    def _on(self, device):
        cache = self.__dict__.setdefault("_dev", {})
        key = str(device)
        if key not in cache:
            cache[key] = (self.target.to(device), self.strength.to(device))
        return cache[key]

    def apply(self, logits: torch.Tensor, pred_positions: torch.Tensor) -> torch.Tensor:
        """In place on logits [..., R, V]: row r gets strength[q_r] added at column
        target[q_r], q_r = pred_positions[r] (positions outside the table, or free, get
        nothing), rounded once to the logits' dtype -- the bf16 / fp32 add torch performs
        on the model's output.  No host synchronisation: every row is gathered and
        written back, unbiased rows unchanged."""
        target, strength = self._on(logits.device)
        q = pred_positions.to(device=logits.device, dtype=torch.int64)
        ok = (q >= 0) & (q < target.numel())
        qc = q.clamp(0, target.numel() - 1)
        tok = torch.where(ok, target[qc], torch.full_like(qc, -1))
        r = torch.arange(q.numel(), device=logits.device)
        col = tok.clamp(min=0)
        cur = logits[..., r, col]
        new = (cur.float() + strength[qc]).to(logits.dtype)
        logits[..., r, col] = torch.where(tok >= 0, new, cur)
        return logits


def decode_bias(vocab: int, start: int, total: int, seed: int = 7, frac_strong: float = 0.6,
                frac_free: float = 0.0, strong: float = 20.0, weak_base: float = 6.0,
                weak_step: float = 0.5, exclude: Sequence[int] = ()) -> DecodeBias:
    """Bias table over positions [0, total): positions [start, total) are the generated
    ones (the prompt's own positions are free).  Each is strong with probability
    ``frac_strong``, free with ``frac_free``, else weak with strength weak_base +
    weak_step * ((q * 10) mod 11) -- distinct within any 8 consecutive positions."""
    gen = torch.Generator().manual_seed(seed)
    target = torch.full((total,), -1, dtype=torch.int64)
    strength = torch.zeros(total, dtype=torch.float32)
    n = total - start
    if n <= 0:
        return DecodeBias(target, strength)
    bad = torch.tensor(sorted(set(int(x) for x in exclude)), dtype=torch.int64)
    tok = torch.randint(0, vocab - len(bad), (n,), generator=gen)
    for b in bad.tolist():                         # skip the excluded ids (ascending)
        tok = tok + (tok >= b).to(torch.int64)
    u = torch.rand(n, generator=gen)
    q = torch.arange(start, total)
    weak = weak_base + weak_step * ((q * 10) % 11).float()
    kind_strong = u < frac_strong
    kind_free = (u >= frac_strong) & (u < frac_strong + frac_free)
    s = torch.where(kind_strong, torch.full_like(weak, strong), weak)
    target[start:] = torch.where(kind_free, torch.full_like(tok, -1), tok)
    strength[start:] = torch.where(kind_free, torch.zeros_like(s), s)
    return DecodeBias(target, strength)


def decode_prompt(vocab: int, length: int, seed: int = 5,
                  exclude: Sequence[int] = ()) -> torch.Tensor:
    """[length] uniform-random prompt token ids (seeded), avoiding ``exclude``."""
    gen = torch.Generator().manual_seed(seed)
    bad = sorted(set(int(x) for x in exclude))
    tok = torch.randint(0, vocab - len(bad), (length,), generator=gen)
    for b in bad:
        tok = tok + (tok >= b).to(torch.int64)
    return tok


def synthetic_draft_graph() -> dict:
    """A draft graph in the calibration output format (specfold/calibration/
    calibration.py:246-264): 7 nodes (budget B = 7) over three levels, at most three per
    level (S = 3), depth within D = 8.  ij_set pairs are (pos_rank, vocab_rank): fill the
    pos_rank-th most confident masked position with its vocab_rank-th most likely token."""
    sets = [[(0, 0)], [(1, 0)], [(0, 1)],
            [(0, 0), (1, 0)], [(0, 0), (2, 0)], [(0, 1), (1, 0)],
            [(0, 0), (1, 0), (2, 0)]]
    parents = [None, None, None, 1, 1, 1, 2]
    nodes = []
    for k, ij in enumerate(sets):
        nodes.append({"L": len(ij), "ij_set": sorted(ij), "frequency": 100 - 10 * k,
                      "score": float(100 - 10 * k),
                      "parent_L": parents[k]})
    return {"selected_nodes": nodes, "tree_roots": []}
