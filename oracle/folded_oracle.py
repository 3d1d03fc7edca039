"""CPU restatement of SpecFold's PyTorch folded verify forward (the parity oracle).

TEST INFRASTRUCTURE ONLY: used by ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline legs of ``bench.py``; never by the product path in ``specfold_b200``.

It restates, op for op, the reference classes

* ``SpecFoldFastDLLMV2Generation._batched_block_forward``
  (specfold/generate/fastdllm_v2_folded.py:89-223), and
* ``SpecFoldNLDGeneration._batched_block_forward``
  (specfold/generate/nld_folded.py:104-241),

so that on the CPU it reproduces the reference bit for bit.  That claim is pinned by
``tests/test_oracle_golden.py`` against fixtures produced by running the reference
itself (``tests/golden/make_golden.py``).  The torch op sequence is kept identical to
the reference's on purpose: a different but mathematically equal sequence would round
differently and the oracle would no longer be bit-exact.

On top of the logits it can record, per layer, every intermediate the fused kernels
produce (fold masks, sources, Q/K/V tables, softmax state, FFN outputs), which the GPU
parity tests compare kernel by kernel.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE helper (fastdllm_v2_folded.py:22-25)."""
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def _expand_kv(t: torch.Tensor, rep: int) -> torch.Tensor:
    """[1, Hkv, S, hd] -> [1, Hkv*rep, S, hd], each kv head repeated ``rep`` times
    consecutively (fastdllm_v2_folded.py:29-34)."""
    b, hkv, s, d = t.shape
    if rep == 1:
        return t
    return t[:, :, None, :, :].expand(b, hkv, rep, s, d).reshape(b, hkv * rep, s, d)


def parent_map(batched_input: torch.Tensor) -> Tuple[List[Optional[int]], List[int]]:
    """par(i) = first branch j != i whose differing-position set (vs the main block) has
    one element fewer and is a subset of draft i's; main (0) when none qualifies.
    (fastdllm_v2_folded.py:55-75, nld_folded.py:72-90.)"""
    B1 = batched_input.shape[0]
    differs = batched_input != batched_input[0:1]
    counts = differs.sum(1).tolist()
    # escapes[i][j]: branch j differs somewhere branch i does not
    escapes = (differs.unsqueeze(0) & ~differs.unsqueeze(1)).any(-1).tolist()
    parent: List[Optional[int]] = [None] + [0] * (B1 - 1)
    for i in range(1, B1):
        for j in range(B1):
            if j != i and counts[j] == counts[i] - 1 and not escapes[i][j]:
                parent[i] = j
                break
    return parent, counts


def gate_rows(x: torch.Tensor, xp: torch.Tensor, delta: float) -> torch.Tensor:
    """Positions whose layer input moved more than delta relative to the parent's:
    ``||x - x_par|| > delta * ||x_par||`` in the model dtype
    (fastdllm_v2_folded.py:139-141).  x, xp: [N, D]."""
    moved = (x - xp).norm(dim=-1)
    scale = xp.norm(dim=-1)
    return (moved > delta * scale).nonzero(as_tuple=True)[0]


def nearest_recomputing_ancestor(rec: torch.Tensor, parent: List[Optional[int]]) -> torch.Tensor:
    """src[b, n]: the first branch on b's parent chain (b included) that recomputed
    position n -- the row whose Q/K/V, softmax state and FFN output branch b inherits
    at n.  Follows from the table inheritance at fastdllm_v2_folded.py:146-162,212."""
    B1, N = rec.shape
    src = torch.empty(B1, N, dtype=torch.int64)
    for b in range(B1):
        for n in range(N):
            c = b
            while not bool(rec[c, n]):
                c = parent[c]
            src[b, n] = c
    return src


class Capture:
    """Per-layer record of the folded forward's intermediates, indexed [layer][branch]."""

    def __init__(self):
        self.parent: List[Optional[int]] = []
        self.counts: List[int] = []
        self.order: List[int] = []
        self.layers: List[Dict[str, torch.Tensor]] = []
        self.positions = 0      # draft positions seen by the gate
        self.recomputed = 0     # draft positions recomputed


def folded_forward(model, batched_input: torch.Tensor, past_key_values, delta: float,
                   family: str = "fastdllm", capture: Optional[Capture] = None,
                   rec_override: Optional[torch.Tensor] = None,
                   shift: Optional[bool] = None) -> torch.Tensor:
    """Logits of the folded B1 x N verify forward (Fast-dLLM: shifted, NLD: unshifted;
    ``shift=False`` returns the model's unshifted Fast-dLLM logits, as its executor
    forward does).

    ``model`` is the object the reference reads as ``self.model_executor.model``;
    ``past_key_values`` offers ``get_seq_length``, ``len`` and ``[li] -> (k, v)``.

    ``rec_override`` ([L, B1, N] bool, optional) replaces the gate's decisions of the
    draft branches with the given masks (the main branch always recomputes).  Parity
    tests use it to re-run the oracle with the fold decisions a GPU run took where a
    near-tie landed on the other side of the threshold, so that every branch can be
    compared.  The recorded margins still describe the oracle's own inputs.
    """
    if family == "fastdllm":
        base = model.model
    elif family == "nld":
        base = model.encoder
    else:
        raise ValueError(family)
    cfg = model.config
    B1, N = batched_input.shape
    dev = batched_input.device
    H = cfg.num_attention_heads
    Hkv = cfg.num_key_value_heads
    G = H // Hkv
    P = int(past_key_values.get_seq_length()) if past_key_values is not None else 0
    delta = float(delta)

    parent, counts = parent_map(batched_input)
    order = sorted(range(B1), key=lambda i: counts[i])
    if capture is not None:
        capture.parent, capture.counts, capture.order = parent, counts, order

    hidden = base.embed_tokens(batched_input)
    D = hidden.shape[-1]
    pos = torch.arange(P, P + N, device=dev).unsqueeze(0)
    cos, sin = base.rotary_emb(hidden, pos)
    cos, sin = cos[0], sin[0]
    q_scale = _nld_q_scale(cfg, P, N, dev) if family == "nld" else None
    rows = [hidden[i:i + 1] for i in range(B1)]

    for lyr in base.layers:
        att = lyr.self_attn
        hd = att.head_dim
        sc = att.scaling
        li = att.layer_idx
        have_prefix = past_key_values is not None and len(past_key_values) > li
        if have_prefix:
            pk, pv = past_key_values[li]
            pk_h = _expand_kv(pk, G)[0]
            pv_h = _expand_kv(pv, G)[0]

        st: Dict[str, list] = {k: [None] * B1 for k in
                               ("q", "k", "v", "m", "Z", "O", "ffn", "hp", "out", "rbar")}
        for i in order:
            x = rows[i]
            pj = parent[i]
            if pj is None:
                rbar = torch.arange(N, device=dev)
            else:
                rbar = gate_rows(x[0], rows[pj][0], delta)
                if rec_override is not None:
                    rbar = rec_override[li][i].to(dev).nonzero(as_tuple=True)[0]
                if capture is not None:
                    capture.positions += N
                    capture.recomputed += int(rbar.numel())
                    # relative distance to the threshold (diagnostic only)
                    moved = (x[0] - rows[pj][0]).float().norm(dim=-1)
                    ref = rows[pj][0].float().norm(dim=-1)
                    st.setdefault("ratio", [None] * B1)[i] = moved / (delta * ref) - 1.0
            R = int(rbar.numel())

            # Q/K/V tables: inherit the parent's, overwrite the recomputed positions
            if pj is None:
                qt = x.new_zeros(H, N, hd); kt = x.new_zeros(Hkv, N, hd); vt = x.new_zeros(Hkv, N, hd)
            else:
                qt = st["q"][pj].clone(); kt = st["k"][pj].clone(); vt = st["v"][pj].clone()
            if R:
                xn = lyr.input_layernorm(x)[0, rbar]
                qn = att.q_proj(xn).view(R, H, hd).transpose(0, 1)
                kn = att.k_proj(xn).view(R, Hkv, hd).transpose(0, 1)
                vn = att.v_proj(xn).view(R, Hkv, hd).transpose(0, 1)
                c = cos[rbar].unsqueeze(0); s = sin[rbar].unsqueeze(0)
                qn = qn * c + _rotate_half(qn) * s
                kr = kn * c + _rotate_half(kn) * s
                if q_scale is not None:
                    qn = qn * q_scale[rbar].view(1, R, 1).to(qn.dtype)
                k_prev = kt[:, rbar].clone() if pj is not None else None
                v_prev = vt[:, rbar].clone() if pj is not None else None
                qt[:, rbar] = qn; kt[:, rbar] = kr; vt[:, rbar] = vn
            st["q"][i], st["k"][i], st["v"][i] = qt, kt, vt

            k_h = _expand_kv(kt.unsqueeze(0), G)[0] if Hkv != H else kt
            v_h = _expand_kv(vt.unsqueeze(0), G)[0] if Hkv != H else vt
            Kall = torch.cat([pk_h, k_h], dim=1) if have_prefix else k_h
            Vall = torch.cat([pv_h, v_h], dim=1) if have_prefix else v_h

            m = torch.full((H, N), float("-inf"), dtype=torch.float32, device=dev)
            Z = torch.zeros(H, N, dtype=torch.float32, device=dev)
            O = torch.zeros(H, N, hd, dtype=torch.float32, device=dev)
            if pj is not None:
                m.copy_(st["m"][pj]); Z.copy_(st["Z"][pj]); O.copy_(st["O"][pj])

            if R:   # recomputed rows: full softmax over prefix + block, state kept
                s_r = torch.einsum("hrd,hkd->hrk", qt[:, rbar].float(), Kall.float()) * sc
                m_r = s_r.max(dim=-1).values
                e_r = torch.exp(s_r - m_r.unsqueeze(-1))
                Z_r = e_r.sum(-1)
                O_r = torch.einsum("hrk,hkd->hrd", e_r, Vall.float()) / Z_r.unsqueeze(-1)
                m[:, rbar] = m_r; Z[:, rbar] = Z_r; O[:, rbar] = O_r

            if pj is not None and R:   # folded rows: exact update for the changed keys
                keep = torch.ones(N, dtype=torch.bool, device=dev); keep[rbar] = False
                L = keep.nonzero(as_tuple=True)[0]
                if L.numel():
                    qL = qt[:, L].float()
                    ko = _expand_kv(k_prev.unsqueeze(0), G)[0] if Hkv != H else k_prev
                    vo = _expand_kv(v_prev.unsqueeze(0), G)[0] if Hkv != H else v_prev
                    kn_h = k_h[:, rbar]; vn_h = v_h[:, rbar]
                    s_old = torch.einsum("hld,hed->hle", qL, ko.float()) * sc
                    s_new = torch.einsum("hld,hed->hle", qL, kn_h.float()) * sc
                    m_par = st["m"][pj][:, L]
                    m_up = torch.maximum(m_par, s_new.max(-1).values)
                    rescale = torch.exp(m_par - m_up)
                    a_old = torch.exp(s_old - m_up.unsqueeze(-1))
                    a_new = torch.exp(s_new - m_up.unsqueeze(-1))
                    Zp = st["Z"][pj][:, L] * rescale
                    num = st["O"][pj][:, L] * (Zp).unsqueeze(-1)
                    num = num - torch.einsum("hle,hed->hld", a_old, vo.float()) \
                              + torch.einsum("hle,hed->hld", a_new, vn_h.float())
                    Zu = Zp - a_old.sum(-1) + a_new.sum(-1)
                    m[:, L] = m_up; Z[:, L] = Zu
                    O[:, L] = num / Zu.unsqueeze(-1)
            st["m"][i], st["Z"][i], st["O"][i] = m, Z, O

            # residual stream is never folded
            O_rows = O.permute(1, 0, 2).reshape(N, H * hd).to(x.dtype)
            hp = x + (O_rows @ att.o_proj.weight.t()).unsqueeze(0)
            st["hp"][i] = hp

            # FFN: recomputed rows run it, folded rows inherit the parent's output
            ffn = st["ffn"][pj].clone() if pj is not None else x.new_zeros(1, N, D)
            if R:
                mlp = lyr.mlp
                z = lyr.post_attention_layernorm(hp[0, rbar])
                ffn[0, rbar] = mlp.down_proj(F.silu(mlp.gate_proj(z)) * mlp.up_proj(z))
            st["ffn"][i] = ffn
            st["out"][i] = hp + ffn
            st["rbar"][i] = rbar

        if capture is not None:
            rec = torch.zeros(B1, N, dtype=torch.bool)
            margin = torch.full((B1, N), float("inf"))
            for b in range(B1):
                rec[b, st["rbar"][b].cpu()] = True
                if "ratio" in st and st["ratio"][b] is not None:
                    margin[b] = st["ratio"][b].abs().cpu()
            capture.layers.append({
                "hidden_in": torch.cat(rows, 0).detach().clone(),
                "rec": rec,
                "margin": margin,
                "src": nearest_recomputing_ancestor(rec, parent),
                "q": torch.stack(st["q"]), "k": torch.stack(st["k"]), "v": torch.stack(st["v"]),
                "m": torch.stack(st["m"]), "Z": torch.stack(st["Z"]), "O": torch.stack(st["O"]),
                "hp": torch.cat(st["hp"], 0), "ffn": torch.cat(st["ffn"], 0),
                "hidden_out": torch.cat(st["out"], 0),
            })
        rows = st["out"]

    final = base.norm(torch.cat(rows, dim=0))
    if family == "fastdllm":
        logits = model.lm_head(final)
        if shift is False:
            return logits
        return torch.cat([logits[:, :1, :], logits[:, :-1, :]], dim=1)   # generation.py:121-126
    return model.diffusion_head(final)


def _nld_q_scale(cfg, P: int, N: int, device) -> Optional[torch.Tensor]:
    """llama-4 query scale for block positions [P, P+N); None when identically 1
    (nld_folded.py:37-53)."""
    rp = getattr(cfg, "rope_parameters", None) or {}
    beta = rp.get("llama_4_scaling_beta")
    omax = rp.get("original_max_position_embeddings")
    if beta is None or omax is None:
        return None
    pos = torch.arange(P, P + N, device=device, dtype=torch.float32)
    scale = 1.0 + beta * torch.log(1.0 + torch.floor(pos / omax))
    if bool((scale == 1.0).all()):
        return None
    return scale


def fold_stats(capture: Capture) -> Dict[str, float]:
    """The reference's fold_ratio = 1 - recomputed / draft positions
    (fastdllm_v2_folded.py:49-53)."""
    tot = capture.positions
    return {"positions": tot, "recomputed": capture.recomputed,
            "fold_ratio": (1.0 - capture.recomputed / tot) if tot else float("nan")}
