"""Kernel-level parity through the C ABI: each entry point is fed the inputs the oracle
(the reference's PyTorch folded forward) sees at a layer and compared with the oracle's
recorded intermediates.  Indices and fold masks bit-exact; floating point within 2e-2
(bf16) / 1e-4 (fp32) normwise relative error.
"""
import pytest
import torch
import torch.nn.functional as F

from oracle import folded_oracle as orc
from specfold_b200 import kernels as K
from tests.golden.make_golden import build_case
from tests.helpers import TOL, assert_close

pytestmark = pytest.mark.gpu

CASES = ["tiny_fp32_chain", "tiny_bf16_chain", "tiny_bf16_tree", "tiny_nld_fp32_tree"]


def _capture(name):
    family, model, cache, ids, delta = build_case(name)
    cap = orc.Capture()
    with torch.no_grad():
        orc.folded_forward(model, ids, cache, delta, family=family, capture=cap)
    return family, model, cache, ids, delta, cap


def _flat_q(q):      # [B1, H, N, hd] -> [B1*N, H*hd]
    B1, H, N, hd = q.shape
    return q.permute(0, 2, 1, 3).reshape(B1 * N, H * hd)


def _flat_hn(m):     # [B1, H, N] -> [B1*N, H]
    B1, H, N = m.shape
    return m.permute(0, 2, 1).reshape(B1 * N, H)


def _bookkeeping(rec, parent):
    """rows / seg / segcnt / src / f the way the reference's tables imply them."""
    B1, N = rec.shape
    flat = rec.reshape(-1)
    rows = flat.nonzero(as_tuple=True)[0]
    seg = torch.zeros(B1 * N, dtype=torch.int64)
    segcnt = torch.zeros(B1, dtype=torch.int32)
    for b in range(B1):
        r = (rec[b].nonzero(as_tuple=True)[0] + b * N)
        seg[b * N: b * N + r.numel()] = r
        segcnt[b] = r.numel()
    src = orc.nearest_recomputing_ancestor(rec, parent).reshape(-1)
    f = torch.tensor([b if rec[b, n] else (parent[b] or 0) for b in range(B1) for n in range(N)])
    return rows, seg, segcnt, src, f


def _par_idx(parent):
    return torch.tensor([0] + [p for p in parent[1:]], dtype=torch.int64)


# --------------------------------------------------------------------------- gate
@pytest.mark.parametrize("name", CASES)
def test_gate_and_compaction(name):
    family, model, cache, ids, delta, cap = _capture(name)
    base = model.encoder if family == "nld" else model.model
    B1, N = ids.shape
    for li, lay in enumerate(cap.layers):
        x = lay["hidden_in"]
        D = x.shape[-1]
        dtype = x.dtype
        ln_w = base.layers[li].input_layernorm.weight
        eps = base.layers[li].input_layernorm.variance_epsilon
        out = K.residual_delta_gate(x.reshape(B1 * N, D).cuda(), _par_idx(cap.parent).cuda(),
                                    delta, B1, N, B1 * N, eps, ln_w=ln_w.cuda())
        torch.cuda.synchronize()
        K.raise_device_error(out["err"])
        rec = out["rec"].cpu().bool().view(B1, N)
        assert torch.equal(rec, lay["rec"]), f"layer {li}: fold mask"
        rows, seg, segcnt, src, f = _bookkeeping(lay["rec"], cap.parent)
        cnt = int(out["count"].item())
        assert cnt == rows.numel()
        assert torch.equal(out["rows"][:cnt].cpu(), rows)
        assert torch.equal(out["segcnt"].cpu(), segcnt)
        for b in range(B1):
            k = int(segcnt[b])
            assert torch.equal(out["seg"][b * N: b * N + k].cpu(), seg[b * N: b * N + k])
        assert torch.equal(out["src"].cpu(), src)
        assert torch.equal(out["f"].cpu(), f)
        assert torch.equal(lay["src"].reshape(-1), src)
        # rstd and the normalised QKV input
        xf = x.reshape(B1 * N, D).float()
        rstd_ref = torch.rsqrt(xf.pow(2).mean(-1) + eps)
        assert_close(out["rstd"].cpu(), rstd_ref, torch.float32, "rstd", tol=1e-6)
        xn_ref = base.layers[li].input_layernorm(x.reshape(B1 * N, D))[rows]
        assert_close(out["xn"][:cnt].cpu(), xn_ref, dtype, "xn")


def test_gate_randomised_margins():
    """Random draft rows at relative distances spread log-uniformly over [1e-3, 1] of
    their parent around delta = 0.1 (no deliberate exact ties); both dtypes."""
    g = torch.Generator().manual_seed(11)
    B1, N, D = 8, 32, 1024
    parent = [None, 0, 0, 1, 1, 2, 0, 5]
    for dtype in (torch.float32, torch.bfloat16):
        x = torch.empty(B1, N, D)
        x[0] = torch.randn(N, D, generator=g)
        for b in range(1, B1):
            sig = torch.exp(torch.empty(N, 1).uniform_(-6.9, 0.0, generator=g))
            x[b] = x[parent[b]] + torch.randn(N, D, generator=g) * sig
        x = x.to(dtype)
        rec_ref = torch.zeros(B1, N, dtype=torch.bool)
        rec_ref[0] = True
        for b in range(1, B1):
            rec_ref[b, orc.gate_rows(x[b], x[parent[b]], 0.1)] = True
        out = K.residual_delta_gate(x.reshape(B1 * N, D).cuda(), _par_idx(parent).cuda(), 0.1,
                                    B1, N, B1 * N, 1e-6)
        torch.cuda.synchronize()
        assert torch.equal(out["rec"].cpu().bool().view(B1, N), rec_ref), dtype
        src = orc.nearest_recomputing_ancestor(rec_ref, parent).reshape(-1)
        assert torch.equal(out["src"].cpu(), src)


def test_src_resolve_entry_point():
    rec = torch.tensor([[1, 1, 1, 1], [0, 1, 0, 0], [0, 0, 1, 0], [1, 0, 0, 0]], dtype=torch.bool)
    parent = [None, 0, 1, 2]
    _, _, _, src, f = _bookkeeping(rec, parent)
    got = K.src_resolve(f.cuda(), 4, 4)
    torch.cuda.synchronize()
    assert torch.equal(got.cpu(), src)


# --------------------------------------------------------------------------- QKV
@pytest.mark.parametrize("name", CASES)
def test_qkv_rope_scatter(name):
    family, model, cache, ids, delta, cap = _capture(name)
    base = model.encoder if family == "nld" else model.model
    cfg = model.config
    B1, N = ids.shape
    H, Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
    for li, lay in enumerate(cap.layers):
        att = base.layers[li].self_attn
        hd = att.head_dim
        x = lay["hidden_in"]
        D = x.shape[-1]
        dtype = x.dtype
        rows = lay["rec"].reshape(-1).nonzero(as_tuple=True)[0]
        xn = base.layers[li].input_layernorm(x.reshape(B1 * N, D))[rows].contiguous()
        w = torch.cat([att.q_proj.weight, att.k_proj.weight, att.v_proj.weight], 0)
        bias = (torch.cat([att.q_proj.bias, att.k_proj.bias, att.v_proj.bias], 0)
                if att.q_proj.bias is not None else None)
        P = 0 if cache is None else cache.get_seq_length()
        cos, sin = base.rotary_emb(x, torch.arange(P, P + N).unsqueeze(0))
        q_buf = torch.zeros(B1 * N + 1, H * hd, dtype=dtype, device="cuda")
        kv_buf = torch.zeros(B1 * N + 1, 2 * Hkv * hd, dtype=dtype, device="cuda")
        cnt = torch.tensor([rows.numel()], dtype=torch.int32, device="cuda")
        err = K.fused_ln_qkv_rope_scatter(
            xn.cuda(), w.contiguous().cuda(), None if bias is None else bias.cuda(), rows.cuda(),
            cnt, cos[0].to(dtype).contiguous().cuda(), sin[0].to(dtype).contiguous().cuda(),
            q_buf, kv_buf, N, B1 * N, H, Hkv, hd)
        torch.cuda.synchronize()
        K.raise_device_error(err)
        q_ref = _flat_q(lay["q"])[rows]
        kv_ref = torch.cat([_flat_q(lay["k"]), _flat_q(lay["v"])], 1)[rows]
        assert_close(q_buf[rows.cuda()].cpu(), q_ref, dtype, f"layer {li} q")
        assert_close(kv_buf[rows.cuda()].cpu(), kv_ref, dtype, f"layer {li} kv")


def _rope_ref(x, cos, sin, pos):
    """x [n, heads, hd] fp32; the rotate-half RoPE at block positions pos."""
    c, s_ = cos[pos].float().unsqueeze(1), sin[pos].float().unsqueeze(1)
    h = x.shape[-1] // 2
    rot = torch.cat([-x[..., h:], x[..., :h]], -1)
    return x * c + rot * s_


@pytest.mark.parametrize("count", [1, 122, 128, 129, 256])
def test_qkv_rope_scatter_7b_shape(count):
    """The QKV GEMM at the Qwen2.5-7B shape (D = 3584 -> 4608 outputs), split over K and
    with its k-steps spread over independent TMEM accumulators (four at <= 128 rows, two
    above), against a torch fp32 GEMM + bias + RoPE + scatter on the same bf16 inputs."""
    D, H, Hkv, hd, N, BN = 3584, 28, 4, 128, 32, 256
    g = torch.Generator().manual_seed(11 + count)
    n_out = (H + 2 * Hkv) * hd
    xn = torch.randn(BN, D, generator=g).to(torch.bfloat16)
    w = (torch.randn(n_out, D, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(n_out, generator=g) * 0.02).to(torch.bfloat16)
    ang = torch.rand(N, hd // 2, generator=g) * 6.0
    cos = torch.cat([ang.cos(), ang.cos()], -1).to(torch.bfloat16)
    sin = torch.cat([ang.sin(), ang.sin()], -1).to(torch.bfloat16)
    rows = torch.randperm(BN, generator=g)[:count].sort().values
    q_buf = torch.zeros(BN + 1, H * hd, dtype=torch.bfloat16, device="cuda")
    kv_buf = torch.zeros(BN + 1, 2 * Hkv * hd, dtype=torch.bfloat16, device="cuda")
    cnt = torch.tensor([count], dtype=torch.int32, device="cuda")
    err = K.fused_ln_qkv_rope_scatter(xn.cuda(), w.cuda(), b.cuda(), rows.cuda(), cnt, cos.cuda(),
                                      sin.cuda(), q_buf, kv_buf, N, BN, H, Hkv, hd)
    torch.cuda.synchronize()
    K.raise_device_error(err)
    y = xn[:count].float() @ w.float().t() + b.float()
    pos = rows % N
    q = _rope_ref(y[:, :H * hd].reshape(count, H, hd), cos, sin, pos).reshape(count, -1)
    k = _rope_ref(y[:, H * hd:(H + Hkv) * hd].reshape(count, Hkv, hd), cos, sin, pos).reshape(count, -1)
    v = y[:, (H + Hkv) * hd:]
    assert_close(q_buf[rows.cuda()].cpu(), q, torch.bfloat16, f"q at {count} rows")
    assert_close(kv_buf[rows.cuda()].cpu(), torch.cat([k, v], 1), torch.bfloat16, f"kv at {count} rows")
    # rows that were not recomputed stay untouched
    keep = torch.ones(BN + 1, dtype=torch.bool)
    keep[rows] = False
    keep[BN] = False                                  # the sink row of padded slots
    assert not q_buf.cpu()[keep].any() and not kv_buf.cpu()[keep].any()


# --------------------------------------------------------------------------- attention + merge
@pytest.mark.parametrize("name", CASES)
def test_attention_and_chain_correction(name):
    family, model, cache, ids, delta, cap = _capture(name)
    cfg = model.config
    B1, N = ids.shape
    BN = B1 * N
    H, Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
    base = model.encoder if family == "nld" else model.model
    for li, lay in enumerate(cap.layers):
        att = base.layers[li].self_attn
        hd, scale = att.head_dim, float(att.scaling)
        dtype = lay["hidden_in"].dtype
        rec = lay["rec"]
        rows, seg, segcnt, src, f = _bookkeeping(rec, cap.parent)
        q_buf = torch.zeros(BN + 1, H * hd, dtype=dtype)
        q_buf[:BN] = _flat_q(lay["q"])
        kv_buf = torch.zeros(BN + 1, 2 * Hkv * hd, dtype=dtype)
        kv_buf[:BN] = torch.cat([_flat_q(lay["k"]), _flat_q(lay["v"])], 1)
        O = torch.zeros(BN, H * hd, dtype=dtype, device="cuda")
        M = torch.zeros(BN, H, device="cuda")
        Z = torch.zeros(BN, H, device="cuda")
        if cache is not None:
            pk, pv = cache[li]
            pk, pv, P = pk[0].contiguous().cuda(), pv[0].contiguous().cuda(), pk.shape[2]
            stride = pk.stride(0)
        else:
            pk = pv = None
            P, stride = 0, 0
        qb, kvb = q_buf.cuda(), kv_buf.cuda()
        srcd, rowsd = src.cuda(), rows.cuda()
        cnt = torch.tensor([rows.numel()], dtype=torch.int32, device="cuda")
        err = K.flash_attn_gqa(qb, pk, pv, stride, kvb, srcd, rowsd, cnt, O, M, Z, P, N, scale,
                               BN, B1, H, Hkv, hd)
        torch.cuda.synchronize()
        K.raise_device_error(err)
        O_ref = _flat_q(lay["O"])
        M_ref, Z_ref = _flat_hn(lay["m"]), _flat_hn(lay["Z"])
        assert_close(O[rowsd].cpu(), O_ref[rows], dtype, f"layer {li} O (recomputed)")
        assert_close(M[rowsd].cpu(), M_ref[rows], torch.float32, "M", tol=TOL[dtype] / 10)
        assert_close(Z[rowsd].cpu(), Z_ref[rows], dtype, "Z")
        err = K.chain_correction_gqa(qb, kvb, srcd, _par_idx(cap.parent).cuda(),
                                     rec.reshape(-1).to(torch.int8).cuda(), seg.cuda(),
                                     segcnt.cuda(), O, M, Z, B1, N, scale, H, Hkv, hd)
        torch.cuda.synchronize()
        K.raise_device_error(err)
        folded = (~rec.reshape(-1)).nonzero(as_tuple=True)[0]
        if folded.numel():
            fd = folded.cuda()
            assert_close(O[fd].cpu(), O_ref[folded], dtype, f"layer {li} O (folded)")
            assert_close(M[fd].cpu(), M_ref[folded], torch.float32, "M folded", tol=TOL[dtype] / 10)
            assert_close(Z[fd].cpu(), Z_ref[folded], dtype, "Z folded")


# --------------------------------------------------------------------------- projections
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(256, 512, 512), (256, 3584, 3584), (100, 1536, 1536)])
def test_o_proj_residual(dtype, shape):
    BN, D, qd = shape
    g = torch.Generator().manual_seed(3)
    Hf = torch.randn(BN, D, generator=g).to(dtype)
    O = torch.randn(BN, qd, generator=g).to(dtype)
    Wo = (torch.randn(D, qd, generator=g) * 0.02).to(dtype)
    hp, err = K.o_proj_residual(Hf.cuda(), O.cuda(), Wo.cuda())
    torch.cuda.synchronize()
    K.raise_device_error(err)
    ref = Hf.float() + (O.float() @ Wo.float().t()).to(dtype).float()
    assert_close(hp.cpu(), ref, dtype, "o_proj")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("count", [1, 17, 122, 200, 256])
def test_ffn_scatter(dtype, count):
    BN, D, I, eps = 256, 512, 1408, 1e-6
    g = torch.Generator().manual_seed(count)
    hp = torch.randn(BN, D, generator=g).to(dtype)
    ln = (1 + 0.1 * torch.randn(D, generator=g)).to(dtype)
    Wg = (torch.randn(I, D, generator=g) * 0.05).to(dtype)
    Wu = (torch.randn(I, D, generator=g) * 0.05).to(dtype)
    Wd = (torch.randn(D, I, generator=g) * 0.05).to(dtype)
    rows = torch.randperm(BN, generator=g)[:count].sort().values
    ffn = torch.zeros(BN + 1, D, dtype=dtype, device="cuda")
    cnt = torch.tensor([count], dtype=torch.int32, device="cuda")
    out = K.fused_ffn_scatter(hp.cuda(), ln.cuda(), Wg.cuda(), Wu.cuda(), Wd.cuda(), rows.cuda(),
                              cnt, ffn, BN, eps)
    torch.cuda.synchronize()
    K.raise_device_error(out["err"])
    x = hp[rows].float()
    z = (ln.float() * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)).to(dtype).float()).to(dtype)
    act = (F.silu((z.float() @ Wg.float().t()).to(dtype)) * (z.float() @ Wu.float().t()).to(dtype))
    ref = (act.float() @ Wd.float().t()).to(dtype)
    assert_close(ffn[rows.cuda()].cpu(), ref, dtype, "ffn")
    # rows that were not listed are untouched
    mask = torch.ones(BN + 1, dtype=torch.bool)
    mask[rows] = False
    assert ffn.cpu()[mask].abs().max().item() == 0.0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shift", [0, 1])
def test_final_norm_lm_head(dtype, shift):
    B1, N, D, V, eps = 8, 32, 512, 1000, 1e-6
    g = torch.Generator().manual_seed(7 + shift)
    h = torch.randn(B1 * N, D, generator=g).to(dtype)
    nw = (1 + 0.1 * torch.randn(D, generator=g)).to(dtype)
    W = (torch.randn(V, D, generator=g) * 0.05).to(dtype)
    logits, err = K.final_norm_lm_head(h.cuda(), nw.cuda(), W.cuda(), B1, N, eps, shift)
    torch.cuda.synchronize()
    K.raise_device_error(err)
    x = h.float()
    z = (nw.float() * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)).to(dtype).float()).to(dtype)
    ref = (z.float() @ W.float().t()).to(dtype).view(B1, N, V)
    if shift:
        ref = torch.cat([ref[:, :1], ref[:, :-1]], 1)
    assert_close(logits.cpu(), ref, dtype, "logits")


def test_final_norm_lm_head_wave_tail():
    """A Qwen-sized vocabulary (152064 = 1188 weight tiles): 594 two-tile units leave a
    last round of 2 units on 148 SMs, so the library runs the last 4 tiles as a split-K
    phase of the same launch.  Logits of every tile, the tail's included, match."""
    dtype, B1, N, D, V, eps = torch.bfloat16, 8, 32, 1024, 152064, 1e-6
    g = torch.Generator(device="cuda").manual_seed(11)
    h = torch.randn(B1 * N, D, generator=g, device="cuda").to(dtype)
    nw = (1 + 0.1 * torch.randn(D, generator=g, device="cuda")).to(dtype)
    W = (torch.randn(V, D, generator=g, device="cuda") * 0.05).to(dtype)
    logits, err = K.final_norm_lm_head(h, nw, W, B1, N, eps, 0)
    torch.cuda.synchronize()
    K.raise_device_error(err)
    x = h.float()
    z = (nw.float() * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)).to(dtype).float()).to(dtype)
    ref = (z.float() @ W.float().t()).to(dtype).view(B1, N, V)
    assert_close(logits[..., -1024:].cpu(), ref[..., -1024:].cpu(), dtype, "logits (tail tiles)")
    assert_close(logits.cpu(), ref.cpu(), dtype, "logits")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_kv_append(dtype):
    Hkv, cap, hd, P, n = 4, 256, 128, 100, 32
    ck = torch.randn(Hkv, cap, hd).to(dtype).cuda()
    cv = torch.randn(Hkv, cap, hd).to(dtype).cuda()
    before_k, before_v = ck.clone(), cv.clone()
    nk = torch.randn(Hkv, n, hd).to(dtype).cuda()
    nv = torch.randn(Hkv, n, hd).to(dtype).cuda()
    K.kv_append(ck, cv, nk, nv, P)
    torch.cuda.synchronize()
    ref_k = before_k.clone(); ref_k[:, P:P + n] = nk
    ref_v = before_v.clone(); ref_v[:, P:P + n] = nv
    assert torch.equal(ck, ref_k) and torch.equal(cv, ref_v)


# --------------------------------------------------------------------------- parent map
@pytest.mark.parametrize("B1,N", [(8, 32), (4, 16), (32, 32), (1, 8)])
def test_parent_map_matches_host(B1, N):
    """Device parent map == the reference helper's host computation, on draft blocks
    built as nested edit sets (chains, trees) plus unrelated drafts."""
    from specfold_b200.folded import FoldedVerifyB200
    g = torch.Generator().manual_seed(B1 * 100 + N)
    for trial in range(20):
        main = torch.randint(0, 50, (N,), generator=g)
        rows = [main.clone()]
        for i in range(1, B1):
            if i > 1 and torch.rand(1, generator=g).item() < 0.7:
                base = rows[int(torch.randint(0, i, (1,), generator=g))].clone()
            else:
                base = main.clone()
            pos = int(torch.randint(0, N, (1,), generator=g))
            base[pos] = (base[pos] + 1 + int(torch.randint(0, 5, (1,), generator=g))) % 50
            rows.append(base)
        ids = torch.stack(rows).to(torch.int64)
        parent, _ = FoldedVerifyB200._build_parent_map(ids)
        want = torch.tensor([0] + [parent[i] for i in range(1, B1)], dtype=torch.int64)
        got = K.parent_map(ids.cuda()).cpu()
        assert torch.equal(got, want), (trial, got.tolist(), want.tolist())
