"""Tensor-level wrappers of the C-ABI entry points, one per launch of the reference's
fused path (specfold/generate/triton_kernels.py, launched from
fastdllm_v2_folded.py:306-361).  They take torch CUDA tensors, launch on the current
stream and return without synchronising.  Used by the per-kernel parity tests; the
generator calls the whole-forward entry point instead.
"""

from __future__ import annotations

from typing import Dict, Optional

import torch

from . import _lib

_WS: Dict[int, torch.Tensor] = {}


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return _lib.SF_DTYPE_BF16
    if t.dtype == torch.float32:
        return _lib.SF_DTYPE_F32
    raise TypeError(f"unsupported dtype {t.dtype}; the kernels take float32 or bfloat16")


def _check_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("specfold_b200 kernels take CUDA tensors")
        if t is not None and not t.is_contiguous():
            raise ValueError("specfold_b200 kernels take contiguous tensors")


_DRAFT_WS = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Zero-initialised scratch shared by the GEMM entry points (split-K partials and
    tile counters; the kernels leave the counters at zero)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _WS.get(idx)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WS[idx] = ws
    return ws


def error_word(device) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=device)


def raise_device_error(err: torch.Tensor) -> None:
    bits = int(err.item())
    if bits:
        raise _lib.SpecFoldError("device error: " + _lib.describe_device_error(bits))


def residual_delta_gate(Hf: torch.Tensor, par_idx: torch.Tensor, delta: float, B1: int, N: int,
                        bucket: int, eps: float, ln_w: Optional[torch.Tensor] = None,
                        err: Optional[torch.Tensor] = None) -> Dict[str, torch.Tensor]:
    _check_cuda(Hf, par_idx, ln_w)
    dev = Hf.device
    BN, D = B1 * N, Hf.shape[-1]
    out = {
        "rstd": torch.empty(BN, dtype=torch.float32, device=dev),
        "f": torch.empty(BN, dtype=torch.int64, device=dev),
        "rec": torch.empty(BN, dtype=torch.int8, device=dev),
        "rows": torch.zeros(bucket, dtype=torch.int64, device=dev),
        "count": torch.zeros(1, dtype=torch.int32, device=dev),
        "seg": torch.zeros(BN, dtype=torch.int64, device=dev),
        "segcnt": torch.zeros(B1, dtype=torch.int32, device=dev),
        "src": torch.empty(BN, dtype=torch.int64, device=dev),
        "xn": torch.zeros(bucket, D, dtype=Hf.dtype, device=dev) if ln_w is not None else None,
    }
    err = err if err is not None else error_word(dev)
    lib = _lib.load()
    _lib.check(lib.sf_residual_delta_gate(
        dtype_code(Hf), Hf.data_ptr(), par_idx.data_ptr(), out["rstd"].data_ptr(),
        out["f"].data_ptr(), out["rec"].data_ptr(), out["rows"].data_ptr(),
        out["count"].data_ptr(), out["seg"].data_ptr(), out["segcnt"].data_ptr(),
        out["src"].data_ptr(), _ptr(out["xn"]), _ptr(ln_w), float(delta), B1, N, D, bucket,
        float(eps), err.data_ptr(), _stream()), "residual_delta_gate")
    out["err"] = err
    return out


def parent_map(ids: torch.Tensor) -> torch.Tensor:
    """par_idx [B1] int64 of a [B1, N] int64 token block, on the device
    (SpecFold*Generation._build_parent_map, fastdllm_v2_folded.py:55-75)."""
    _check_cuda(ids)
    ids = ids.contiguous()
    B1, N = ids.shape
    out = torch.empty(B1, dtype=torch.int64, device=ids.device)
    _lib.check(_lib.load().sf_parent_map(ids.data_ptr(), B1, N, out.data_ptr(), _stream()),
               "parent map")
    return out


def src_resolve(f: torch.Tensor, B1: int, N: int, err: Optional[torch.Tensor] = None):
    _check_cuda(f)
    src = torch.empty_like(f)
    err = err if err is not None else error_word(f.device)
    _lib.check(_lib.load().sf_src_resolve(f.data_ptr(), src.data_ptr(), B1, N, err.data_ptr(),
                                          _stream()), "src_resolve")
    return src


def _ws_args(device, BN, D, H, Hkv, hd, I, V):
    need = _lib.load().sf_workspace_bytes(BN, D, H, Hkv, hd, I, V)
    ws = workspace(device, need)
    return ws.data_ptr(), ws.numel()


def fused_ln_qkv_rope_scatter(xn, w_qkv, b_qkv, rows, count, cos, sin, q_buf, kv_buf, N, bucket,
                              H, Hkv, hd, q_scale=None, err=None):
    _check_cuda(xn, w_qkv, b_qkv, rows, count, cos, sin, q_buf, kv_buf, q_scale)
    D = xn.shape[-1]
    err = err if err is not None else error_word(xn.device)
    wp, wn = _ws_args(xn.device, bucket, D, H, Hkv, hd, 64, 64)
    _lib.check(_lib.load().sf_fused_ln_qkv_rope_scatter(
        dtype_code(xn), xn.data_ptr(), w_qkv.data_ptr(), _ptr(b_qkv), rows.data_ptr(),
        count.data_ptr(), cos.data_ptr(), sin.data_ptr(), _ptr(q_scale), q_buf.data_ptr(),
        kv_buf.data_ptr(), D, N, bucket, H, Hkv, hd, wp, wn, err.data_ptr(), _stream()),
        "fused_ln_qkv_rope_scatter")
    return err


def flash_attn_gqa(q_buf, pk, pv, kv_head_stride, kv_buf, src, rows, count, O, M, Z, P, N, scale,
                   bucket, B1, H, Hkv, hd, err=None):
    _check_cuda(q_buf, kv_buf, src, rows, count, O, M, Z)
    err = err if err is not None else error_word(q_buf.device)
    lib = _lib.load()
    need = lib.sf_attn_workspace_bytes(dtype_code(q_buf), bucket, H, Hkv, hd, P)
    ws = workspace(q_buf.device, need + (16 << 10)) if need else None
    # the scratch follows the GEMM tile counters, which must stay untouched
    wp = None if ws is None else ws.data_ptr() + (16 << 10)
    _lib.check(lib.sf_flash_attn_gqa(
        dtype_code(q_buf), q_buf.data_ptr(), _ptr(pk), _ptr(pv), int(kv_head_stride),
        kv_buf.data_ptr(), src.data_ptr(), rows.data_ptr(), count.data_ptr(), O.data_ptr(),
        M.data_ptr(), Z.data_ptr(), P, N, float(scale), bucket, B1, H, Hkv, hd, wp, need,
        err.data_ptr(), _stream()), "flash_attn_gqa")
    return err


def chain_correction_gqa(q_buf, kv_buf, src, par_idx, rec, seg, segcnt, O, M, Z, B1, N, scale, H,
                         Hkv, hd, err=None):
    _check_cuda(q_buf, kv_buf, src, par_idx, rec, seg, segcnt, O, M, Z)
    err = err if err is not None else error_word(q_buf.device)
    _lib.check(_lib.load().sf_chain_correction_gqa(
        dtype_code(q_buf), q_buf.data_ptr(), kv_buf.data_ptr(), src.data_ptr(), par_idx.data_ptr(),
        rec.data_ptr(), seg.data_ptr(), segcnt.data_ptr(), O.data_ptr(), M.data_ptr(),
        Z.data_ptr(), B1, N, float(scale), H, Hkv, hd, err.data_ptr(), _stream()),
        "chain_correction_gqa")
    return err


def o_proj_residual(Hf, O_tab, w_o, err=None):
    _check_cuda(Hf, O_tab, w_o)
    BN, D = Hf.shape
    q_dim = O_tab.shape[1]
    hp = torch.empty_like(Hf)
    err = err if err is not None else error_word(Hf.device)
    wp, wn = _ws_args(Hf.device, BN, D, q_dim // 64, 1, 64, 64, 64)
    _lib.check(_lib.load().sf_o_proj_residual(
        dtype_code(Hf), Hf.data_ptr(), O_tab.data_ptr(), w_o.data_ptr(), hp.data_ptr(), BN, D,
        q_dim, wp, wn, err.data_ptr(), _stream()), "o_proj_residual")
    return hp, err


def fused_ffn_scatter(hp_all, ln_w, w_gate, w_up, w_down, rows, count, ffn_buf, bucket, eps,
                      err=None):
    _check_cuda(hp_all, ln_w, w_gate, w_up, w_down, rows, count, ffn_buf)
    D = hp_all.shape[-1]
    I = w_gate.shape[0]
    dev = hp_all.device
    act = torch.zeros(bucket, I, dtype=hp_all.dtype, device=dev)
    xn = torch.zeros(bucket, D, dtype=hp_all.dtype, device=dev)
    rstd = torch.zeros(bucket, dtype=torch.float32, device=dev)
    err = err if err is not None else error_word(dev)
    wp, wn = _ws_args(dev, bucket, D, 1, 1, 64, I, 64)
    _lib.check(_lib.load().sf_fused_ffn_scatter(
        dtype_code(hp_all), hp_all.data_ptr(), ln_w.data_ptr(), w_gate.data_ptr(),
        w_up.data_ptr(), w_down.data_ptr(), rows.data_ptr(), count.data_ptr(), ffn_buf.data_ptr(),
        bucket, act.data_ptr(), xn.data_ptr(), rstd.data_ptr(), float(eps), D, I, wp, wn,
        err.data_ptr(), _stream()), "fused_ffn_scatter")
    return {"act": act, "xn": xn, "rstd": rstd, "err": err}


def combine(hp_all, ffn_buf, src, B1, N, err=None):
    _check_cuda(hp_all, ffn_buf, src)
    D = hp_all.shape[-1]
    hidden = torch.empty(B1 * N, D, dtype=hp_all.dtype, device=hp_all.device)
    err = err if err is not None else error_word(hp_all.device)
    _lib.check(_lib.load().sf_combine(dtype_code(hp_all), hp_all.data_ptr(), ffn_buf.data_ptr(),
                                      src.data_ptr(), hidden.data_ptr(), B1, N, D,
                                      err.data_ptr(), _stream()), "combine")
    return hidden, err


def final_norm_lm_head(hidden, norm_w, lm_w, B1, N, eps, shift, err=None):
    _check_cuda(hidden, norm_w, lm_w)
    D = hidden.shape[-1]
    V = lm_w.shape[0]
    dev = hidden.device
    logits = torch.empty(B1, N, V, dtype=hidden.dtype, device=dev)
    xn = torch.empty(B1 * N, D, dtype=hidden.dtype, device=dev)
    err = err if err is not None else error_word(dev)
    wp, wn = _ws_args(dev, B1 * N, D, 1, 1, 64, 64, V)
    _lib.check(_lib.load().sf_final_norm_lm_head(
        dtype_code(hidden), hidden.data_ptr(), norm_w.data_ptr(), lm_w.data_ptr(),
        logits.data_ptr(), xn.data_ptr(), B1, N, D, V, float(eps), int(shift), wp, wn,
        err.data_ptr(), _stream()), "final_norm_lm_head")
    return logits, err


def sample_top_p_greedy(logits: torch.Tensor, top_p: float = 0.95):
    """Greedy top-p sampling over the last dimension on the GPU: (tokens int64, the
    tokens' top-p filtered probabilities in the logits' dtype), both shaped
    logits.shape[:-1] (sf_sample_top_p_greedy; the reference's
    FastDLLMModelExecutor.sample_with_top_p at temperature 0)."""
    if not logits.is_cuda:
        raise ValueError("specfold_b200 kernels take CUDA tensors")
    V = logits.shape[-1]
    x = logits.reshape(-1, V)
    if x.stride(-1) != 1:
        x = x.contiguous()
    rows = x.shape[0]
    tokens = torch.empty(rows, dtype=torch.int64, device=x.device)
    conf = torch.empty(rows, dtype=x.dtype, device=x.device)
    _lib.check(_lib.load().sf_sample_top_p_greedy(
        dtype_code(x), x.data_ptr(), rows, V, x.stride(0), float(top_p), tokens.data_ptr(),
        conf.data_ptr(), _stream()), "sample_top_p_greedy")
    return tokens.view(logits.shape[:-1]), conf.view(logits.shape[:-1])


def draft_blocks(logits: torch.Tensor, mask: torch.Tensor, block: torch.Tensor, pos_offset: int,
                 pairs: torch.Tensor, node_off: torch.Tensor, K: int, conf_fp32: bool):
    """Draft blocks from the calibration graph on the GPU (sf_draft_blocks): logits
    [n_pos, V] of the positions [pos_offset, pos_offset + n_pos) of ``block`` (int64
    [L]), mask bool [n_pos], pairs int32 [n_pairs, 2] (pos_rank, vocab_rank), node_off
    int32 [n_nodes + 1].  Returns (drafts int64 [n_nodes, L], valid int32 [n_nodes])."""
    for t in (logits, mask, block, pairs, node_off):
        if not t.is_cuda:
            raise ValueError("specfold_b200 kernels take CUDA tensors")
    n_pos, V = logits.shape
    x = logits if logits.stride(-1) == 1 else logits.contiguous()
    m = mask.contiguous().view(torch.uint8) if mask.dtype == torch.bool else mask.to(torch.uint8)
    blk = block.contiguous()
    n_nodes = node_off.numel() - 1
    drafts = torch.empty(max(n_nodes, 1), blk.numel(), dtype=torch.int64, device=x.device)[:n_nodes]
    valid = torch.empty(max(n_nodes, 1), dtype=torch.int32, device=x.device)[:n_nodes]
    lib = _lib.load()
    nbytes = lib.sf_draft_workspace_bytes(n_pos, K)
    # scratch of its own: the GEMM workspace's counters must stay zero
    idx = x.device.index if x.device.index is not None else torch.cuda.current_device()
    ws = _DRAFT_WS.get(idx)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 16), dtype=torch.uint8, device=x.device)
        _DRAFT_WS[idx] = ws
    _lib.check(lib.sf_draft_blocks(
        dtype_code(x), x.data_ptr(), x.stride(0), n_pos, V, K, 1 if conf_fp32 else 0,
        m.data_ptr(), pairs.data_ptr(), node_off.data_ptr(), n_nodes, blk.data_ptr(), blk.numel(),
        int(pos_offset), drafts.data_ptr(), valid.data_ptr(), ws.data_ptr(), ws.numel(), _stream()),
        "draft_blocks")
    return drafts, valid


def kv_append(cache_k, cache_v, new_k, new_v, P):
    """cache_{k,v}: [Hkv, cap, hd] (any head stride, inner dims contiguous); new_{k,v}:
    [Hkv, n, hd].  Writes positions [P, P+n)."""
    Hkv, cap, hd = cache_k.shape
    n = new_k.shape[1]
    for t in (cache_k, cache_v):
        if t.stride(2) != 1 or t.stride(1) != hd:
            raise ValueError("cache rows must be contiguous [cap, hd] per head")
    if cache_v.stride(0) != cache_k.stride(0):
        raise ValueError("cache_k and cache_v must share one head stride")
    for t in (new_k, new_v):
        if t.stride(2) != 1 or (n > 1 and t.stride(1) != hd):
            raise ValueError("new rows must be contiguous [n, hd] per head")
    if new_v.stride(0) != new_k.stride(0):
        raise ValueError("new_k and new_v must share one head stride")
    if P + n > cap:
        raise ValueError(f"cache capacity {cap} < {P + n}")
    _lib.check(_lib.load().sf_kv_append(
        dtype_code(cache_k), cache_k.data_ptr(), cache_v.data_ptr(), cache_k.stride(0),
        new_k.data_ptr(), new_v.data_ptr(), new_k.stride(0), Hkv, hd, P, n, _stream()),
        "kv_append")
