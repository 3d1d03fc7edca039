"""Kernel microbenchmarks of the folded verify forward (one C-ABI entry point at a time).

    python -m specfold_b200.microbench --kernel qkv|o_proj|ffn|lm_head|attention|merge|gate
        [--shape qwen7b|llama8b|...] [--rows R] [--prefix P] [--fold F] [--branches B1]
        [--iters K]

Each run builds seeded inputs of the named shape on cuda:0, launches the entry point
``--iters`` times after 3 warm-ups, and prints one JSON line per configuration with the
mean CUDA-event time per launch, the algorithmic bytes and FLOPs of one launch, and the
achieved GB/s / TFLOP/s.  Weight matrices at these shapes exceed L2, so every launch
streams them from HBM.  Suitable under ``ncu -k regex:<kernel>`` for counter capture.
"""

from __future__ import annotations

import argparse
import json
import math

import torch

from . import _lib
from . import kernels as K
from .synthetic import SHAPES


def _events(fn, iters, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def _report(name, ms, bytes_, flops, extra=None):
    out = {"kernel": name, "ms": round(ms, 5), "bytes": int(bytes_), "flops": int(flops),
           "gbs": round(bytes_ / (ms / 1e3) / 1e9, 1),
           "tflops": round(flops / (ms / 1e3) / 1e12, 2)}
    out.update(extra or {})
    print(json.dumps(out), flush=True)
    return out


def _rows(BN, count, g):
    return torch.randperm(BN, generator=g)[:count].sort().values.cuda()


def bench_qkv(dims, rows, iters, g):
    D, H, Hkv, hd = dims.hidden, dims.heads, dims.kv_heads, dims.head_dim
    BN = 256
    n_out = (H + 2 * Hkv) * hd
    xn = torch.randn(BN, D, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(n_out, D, generator=g) * 0.02).to(torch.bfloat16).cuda()
    b = (torch.randn(n_out, generator=g) * 0.02).to(torch.bfloat16).cuda()
    cos = torch.randn(32, hd, generator=g).to(torch.bfloat16).cuda()
    sin = torch.randn(32, hd, generator=g).to(torch.bfloat16).cuda()
    r = _rows(BN, rows, g)
    cnt = torch.tensor([rows], dtype=torch.int32, device="cuda")
    q_buf = torch.zeros(BN + 1, H * hd, dtype=torch.bfloat16, device="cuda")
    kv_buf = torch.zeros(BN + 1, 2 * Hkv * hd, dtype=torch.bfloat16, device="cuda")
    err = K.error_word("cuda")
    ms = _events(lambda: K.fused_ln_qkv_rope_scatter(xn, w, b, r, cnt, cos, sin, q_buf, kv_buf,
                                                       32, BN, H, Hkv, hd, err=err), iters)
    K.raise_device_error(err)
    return _report("qkv", ms, n_out * D * 2 + rows * D * 2 + rows * n_out * 2,
                   2 * rows * n_out * D, {"rows": rows})


def bench_o_proj(dims, rows, iters, g):
    D, qd = dims.hidden, dims.heads * dims.head_dim
    BN = rows
    Hf = torch.randn(BN, D, generator=g).to(torch.bfloat16).cuda()
    O = torch.randn(BN, qd, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(D, qd, generator=g) * 0.02).to(torch.bfloat16).cuda()
    err = K.error_word("cuda")
    ms = _events(lambda: K.o_proj_residual(Hf, O, w, err=err), iters)
    K.raise_device_error(err)
    return _report("o_proj", ms, D * qd * 2 + BN * (qd + 2 * D) * 2, 2 * BN * D * qd,
                   {"rows": BN})


def bench_ffn(dims, rows, iters, g):
    D, I = dims.hidden, dims.inter
    BN = 256
    hp = torch.randn(BN, D, generator=g).to(torch.bfloat16).cuda()
    ln = torch.ones(D, dtype=torch.bfloat16, device="cuda")
    wg = (torch.randn(I, D, generator=g) * 0.02).to(torch.bfloat16).cuda()
    wu = (torch.randn(I, D, generator=g) * 0.02).to(torch.bfloat16).cuda()
    wd = (torch.randn(D, I, generator=g) * 0.02).to(torch.bfloat16).cuda()
    r = _rows(BN, rows, g)
    cnt = torch.tensor([rows], dtype=torch.int32, device="cuda")
    ffn = torch.zeros(BN + 1, D, dtype=torch.bfloat16, device="cuda")
    err = K.error_word("cuda")
    ms = _events(lambda: K.fused_ffn_scatter(hp, ln, wg, wu, wd, r, cnt, ffn, BN, 1e-6, err=err),
                 iters)
    K.raise_device_error(err)
    return _report("ffn", ms, 3 * I * D * 2, 2 * rows * 3 * I * D, {"rows": rows})


def bench_lm_head(dims, rows, iters, g):
    D, V = dims.hidden, dims.vocab
    B1, N = max(1, rows // 32), 32
    h = torch.randn(B1 * N, D, generator=g).to(torch.bfloat16).cuda()
    nw = torch.ones(D, dtype=torch.bfloat16, device="cuda")
    w = (torch.randn(V, D, generator=g) * 0.02).to(torch.bfloat16).cuda()
    err = K.error_word("cuda")
    ms = _events(lambda: K.final_norm_lm_head(h, nw, w, B1, N, 1e-6, 1, err=err), iters)
    K.raise_device_error(err)
    return _report("lm_head", ms, V * D * 2 + B1 * N * V * 2, 2 * B1 * N * V * D,
                   {"rows": B1 * N})


def bench_sample(dims, rows, iters, g):
    """Greedy top-p sampling of a verify step's logits (256 rows x V, bf16) on the GPU
    sampler; for context, the time of the full-vocabulary torch.sort alone, the first of
    the reference sampler's five full-size passes (fastdllm_model_executor.py:141)."""
    V = dims.vocab
    x = (torch.randn(rows, V, generator=g) * 2.0).to(torch.bfloat16).cuda()
    ms = _events(lambda: K.sample_top_p_greedy(x, 0.95), iters)
    sort_ms = _events(lambda: torch.sort(x, descending=True, dim=-1), iters)
    return _report("sample", ms, rows * V * 2, 0, {"rows": rows, "vocab": V,
                                                   "torch_sort_ms": round(sort_ms, 4)})


def bench_forward(dims, args):
    """Whole verify forward (main + 7 drafts, configuration-0 noise, fold ~0.6) with
    ``--layers`` decoder layers of the named shape; per-kernel times from the library's
    event profiler."""
    import dataclasses
    from .folded import SpecFoldB200FastDLLMV2Generation
    from . import synthetic as syn
    if args.layers:
        dims = dataclasses.replace(dims, layers=args.layers)
    B1, N = args.branches, 32
    model = syn.build_model(dims, family="fastdllm", dtype=torch.bfloat16, seed=0, device="cuda")
    cache = syn.random_prefix_cache(dims, args.prefix, dtype=torch.bfloat16, seed=1, device="cuda")
    syn.inject_hidden(model, syn.config0_hidden(dims, B1, N, dtype=torch.bfloat16,
                                                frac_recompute=1.0 - args.fold).cuda())
    gen = SpecFoldB200FastDLLMV2Generation(model_executor=syn.StandinExecutor(model), delta=0.1)
    gen.tile_weights = not args.untiled
    ids = torch.zeros(B1, N, dtype=torch.int64, device="cuda")
    for _ in range(3):
        gen._batched_block_forward(ids, cache)
    torch.cuda.synchronize()
    gen._fold_draft_positions = gen._fold_draft_recomputed = 0
    _lib.profile_begin(args.iters * (dims.layers * 9 + 4))
    ms = _events(lambda: gen._batched_block_forward(ids, cache), args.iters, warmup=0)
    prof = _lib.profile_end()
    out = {"kernel": "forward", "ms": round(ms, 4), "layers": dims.layers, "prefix": args.prefix,
           "fold_ratio": round(gen.fold_ratio, 4),
           "per_kernel_ms": {k: round(v[0] / args.iters, 4) for k, v in prof.items() if v[1]}}
    print(json.dumps(out), flush=True)


def bench_sweep(args):
    """The folded-attention / fused-QKV sweep at the Llama-style 8B shape (hidden 4096,
    32 q / 8 kv heads, head_dim 128, RoPE theta 5e5, bf16): prefix length x fold ratio x
    branch budget B (B1 = B + 1 branches of N = 32), configuration-0 noise (a 1 - fold
    share of the draft rows gets the large noise and is recomputed).  One decoder layer
    per configuration; per-kernel CUDA-event times from the library's profiler, with the
    algorithmic bytes and FLOPs of each kernel:

    * qkv: weights + the recomputed rows' input and output; 2 R (H + 2 Hkv) hd D FLOPs;
    * attention (prefix pass + rows pass): the prefix K/V once + the block's q / k / v;
      4 R H hd (P + N) FLOPs for the R recomputed rows plus 4 (BN - R) H hd N for the
      folded rows' in-block keys;
    * gate: the layer input, the parents' rows and the normalised recomputed rows."""
    import dataclasses
    from .folded import SpecFoldB200NLDGeneration
    from . import synthetic as syn
    dims = dataclasses.replace(SHAPES["llama8b"], layers=1)
    D, H, Hkv, hd = dims.hidden, dims.heads, dims.kv_heads, dims.head_dim
    N = 32
    model = syn.build_model(dims, family="nld", dtype=torch.bfloat16, seed=0, device="cuda")
    gen = SpecFoldB200NLDGeneration(model_executor=syn.StandinExecutor(model), delta=0.1)
    prefixes = [int(x) for x in args.sweep_prefix.split(",")]
    folds = [float(x) for x in args.sweep_fold.split(",")]
    budgets = [int(x) for x in args.sweep_b.split(",")]
    for P in prefixes:
        cache = syn.random_prefix_cache(dims, P, dtype=torch.bfloat16, seed=1, device="cuda")
        for B in budgets:
            B1 = B + 1
            for fold in folds:
                syn.inject_hidden(model, syn.config0_hidden(
                    dims, B1, N, dtype=torch.bfloat16, frac_recompute=1.0 - fold).cuda())
                ids = torch.zeros(B1, N, dtype=torch.int64, device="cuda")
                for _ in range(3):
                    gen._batched_block_forward(ids, cache)
                torch.cuda.synchronize()
                gen._fold_draft_positions = gen._fold_draft_recomputed = 0
                _lib.profile_begin(args.iters * 16)
                for _ in range(args.iters):
                    gen._batched_block_forward(ids, cache)
                torch.cuda.synchronize()
                prof = _lib.profile_end()
                BN = B1 * N
                R = (gen._fold_draft_recomputed + args.iters * N) / args.iters
                n_out = (H + 2 * Hkv) * hd
                work = {
                    "qkv": (n_out * D * 2 + R * D * 2 + R * n_out * 2, 2 * R * n_out * D),
                    "attention": (2 * P * Hkv * hd * 2 + BN * (H + 2 * Hkv) * hd * 2 + BN * H * hd * 2,
                                  4 * R * H * hd * (P + N) + 4 * (BN - R) * H * hd * N),
                    "gate": (2 * BN * D * 2 + R * D * 2, 0),
                }
                out = {"sweep": "llama8b", "prefix": P, "B": B, "B1": B1, "fold_target": fold,
                       "fold_ratio": round(gen.fold_ratio, 4) if B > 0 else None,
                       "recomputed_rows": round(R, 1)}
                for k, (nb, nf) in work.items():
                    t_ms, calls = prof.get(k, (0.0, 0))
                    if not calls:
                        continue
                    per = t_ms / calls / 1e3
                    out[k] = {"us": round(per * 1e6, 2), "gbs": round(nb / per / 1e9, 1),
                              "tflops": round(nf / per / 1e12, 2)}
                print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", required=True,
                    choices=["qkv", "o_proj", "ffn", "lm_head", "all_gemm", "forward", "sample",
                             "sweep"])
    ap.add_argument("--shape", default="qwen7b", choices=sorted(SHAPES))
    ap.add_argument("--rows", type=int, default=122)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--layers", type=int, default=0, help="forward: layer count override")
    ap.add_argument("--prefix", type=int, default=1024, help="forward: prefix length")
    ap.add_argument("--fold", type=float, default=0.6, help="forward: draft fold fraction")
    ap.add_argument("--branches", type=int, default=8, help="forward: B1 (main + drafts)")
    ap.add_argument("--untiled", action="store_true",
                    help="forward: plain row-major weights instead of the tile layout")
    ap.add_argument("--sweep-prefix", default="1024,4096,16384,32768")
    ap.add_argument("--sweep-fold", default="0,0.3,0.6,0.9")
    ap.add_argument("--sweep-b", default="1,4,7")
    args = ap.parse_args()
    _lib.check(_lib.load().sf_check_device(), "device")
    if args.kernel == "sweep":
        bench_sweep(args)
        return
    dims = SHAPES[args.shape]
    g = torch.Generator().manual_seed(args.seed)
    if args.kernel == "forward":
        bench_forward(dims, args)
        return
    if args.kernel == "sample":
        bench_sample(dims, 256 if args.rows == 122 else args.rows, args.iters, g)
        return
    todo = ["qkv", "o_proj", "ffn", "lm_head"] if args.kernel == "all_gemm" else [args.kernel]
    for k in todo:
        rows = 256 if k in ("o_proj", "lm_head") and args.kernel == "all_gemm" else args.rows
        {"qkv": bench_qkv, "o_proj": bench_o_proj, "ffn": bench_ffn,
         "lm_head": bench_lm_head}[k](dims, rows, args.iters, g)


if __name__ == "__main__":
    main()
