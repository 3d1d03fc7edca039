"""Benchmark of the B200 folded multi-branch verify forward.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload (the benchmark's Qwen2.5-7B-shape configuration): 28 layers, hidden 3584,
28 q / 4 kv heads, head_dim 128, MLP 18944, vocab 152064, bf16, random-init N(0, 0.02);
one verify step = ``_batched_block_forward`` over the main block + 7 drafts (B1 = 8,
N = 32) against a 1024-token prefix cache, delta = 0.1.  Draft rows follow the
configuration-0 recipe (main hidden + noise; 40% of draft rows recompute at layer 0),
which gives the fold ratio reported in the JSON line.  Weights (15 GB) far exceed L2,
so every step streams them from HBM; no flush is needed.

One step = one verify forward.  ``value`` = verify steps/s of the whole job (N GPUs
run independent request streams, data-parallel, no collective on the hot path), with
inputs resident in HBM; ``e2e`` = the same through the public call with the block's
token ids copied from pinned host memory and the argmax token ids of every verified
position (the greedy decode result the caller consumes) copied back each step.

``--impl reference`` times the reference's PyTorch folded forward (restated in
oracle/folded_oracle.py and pinned bit-exact to the reference) on this machine's host
cores: one decoder layer plus the LM head of the same shape, extrapolated to 28 layers.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s + folded verify-step µs, 7B Qwen2 shape, B=7 D=8 S=3"
UNIT = "verify-steps/s"
SHAPE = "qwen7b"
P_PREFIX = 1024
B1, N = 8, 32
DELTA = 0.1
FRAC_RECOMPUTE = 0.4


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def max_over_ranks(values, device):
    """Element-wise max of per-rank timings (device-timed on each rank); identity at N=1."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return list(values)
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def weak_scaling_value(ws, steps, ms):
    """Whole-job verify steps per second: every rank runs `steps` steps of its own
    stream (data-parallel replicas, no collective on the path); ms = max over ranks."""
    return ws * steps / (ms / 1e3)


# ----------------------------------------------------------------------------- workload
def build_workload(device, dtype=torch.bfloat16, layers=None, seed=0):
    from specfold_b200 import synthetic as syn
    dims = syn.SHAPES[SHAPE]
    if layers is not None:
        import dataclasses
        dims = dataclasses.replace(dims, layers=layers)
    model = syn.build_model(dims, family="fastdllm", dtype=dtype, seed=seed, device=str(device))
    cache = syn.random_prefix_cache(dims, P_PREFIX, dtype=dtype, seed=seed + 1, device=str(device))
    hidden = syn.config0_hidden(dims, B1, N, dtype=dtype, seed=seed + 3,
                                frac_recompute=FRAC_RECOMPUTE)
    model.token_embedding = model.model.embed_tokens      # kept for the decode leg
    syn.inject_hidden(model, hidden.to(device))
    ids = torch.zeros(B1, N, dtype=torch.int64)
    return dims, model, cache, ids


# decode leg: the end-to-end configuration of the 7B shape -- 1024-token random prompts,
# 512 generated tokens each, block length 32, draft graph B=7 D=8 S=3, delta 0.1,
# threshold 0.9 -- on random-init weights with the seeded per-position logit bias that
# stands in for a trained model's confidence (specfold_b200.synthetic.decode_bias)
DECODE_PROMPT, DECODE_NEW = 1024, 512
MASK_ID, STOP_ID = 151665, 151645


def decode_leg(gen, model, dims, streams, rank, device):
    """Decode `streams` independent sequences on this rank; returns the stats of the
    timed ones (after one short warm-up sequence) and their device time in ms."""
    from specfold_b200 import synthetic as syn
    from specfold_b200.decode import FastDLLMV2Decoder
    model.model.embed_tokens = model.token_embedding
    total = DECODE_PROMPT + DECODE_NEW + 2 * N
    graph = syn.synthetic_draft_graph()

    def decoder(seed, new):
        bias = syn.decode_bias(dims.vocab, DECODE_PROMPT, total, seed=1000 + seed,
                               frac_strong=0.6, exclude=(MASK_ID, STOP_ID))
        return FastDLLMV2Decoder(gen, block_length=N, small_block_size=8, threshold=0.9,
                                 top_p=0.95, max_new_tokens=new, mask_id=MASK_ID,
                                 stop_token=STOP_ID, calibration_graph=graph, logit_bias=bias,
                                 capacity=total)

    def prompt(seed):
        return syn.decode_prompt(dims.vocab, DECODE_PROMPT, seed=2000 + seed,
                                 exclude=(MASK_ID, STOP_ID)).tolist()

    decoder(-1, 2 * N).generate_with_draft_speculation(prompt(-1), device=device)   # warm-up
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    runs = []
    torch.cuda.synchronize(device)
    e0.record(stream)
    for k in range(streams):
        seed = rank * 1000 + k
        _, st = decoder(seed, DECODE_NEW).generate_with_draft_speculation(prompt(seed), device=device)
        runs.append(st)
    e1.record(stream)
    torch.cuda.synchronize(device)
    return runs, e0.elapsed_time(e1)


def profiled_traffic(kind):
    """DRAM bytes (read + write) per launch of the kernel `kind`, from the committed ncu
    summary profiles/roofline_traffic.txt (lines `kind: bytes`), or None."""
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "profiles",
                        "roofline_traffic.txt")
    try:
        for line in open(path):
            line = line.split("#", 1)[0].strip()
            if ":" in line:
                k, v = line.split(":", 1)
                if k.strip() == kind:
                    return int(float(v.strip()))
    except OSError:
        pass
    return None


def algorithmic_bytes(dims, P):
    """Bytes one verify step must move: every weight once + the prefix K/V once."""
    w = dims.weight_bytes(2)
    kv = dims.layers * 2 * 2 * P * dims.kv_heads * dims.head_dim
    return w, kv


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        # nvidia-smi's start-up (driver / NVML initialisation) costs host CPU: wait for its
        # first sample, so that it is not competing with the launches of the timed region
        deadline = time.monotonic() + 5.0
        while self.proc is not None and time.monotonic() < deadline:
            if os.path.getsize(self.path) > 0 or self.proc.poll() is not None:
                break
            time.sleep(0.02)
        time.sleep(0.15)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        if not self.path or not os.path.exists(self.path):
            return out
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        os.unlink(self.path)
        if sm:
            out.update(sm_mhz=statistics.median(sm), sm_max_mhz=max(mx), samples=len(sm))
        out["reasons"] = sorted(reasons)
        return out


# ----------------------------------------------------------------------------- arms
def run_b200(args):
    from specfold_b200 import SpecFoldB200FastDLLMV2Generation, _lib
    from specfold_b200.synthetic import StandinExecutor

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev)
    _lib.check(_lib.load().sf_check_device(), "device")
    dims, model, cache, ids = build_workload(dev)
    gen = SpecFoldB200FastDLLMV2Generation(model_executor=StandinExecutor(model), delta=DELTA)
    ids_dev = ids.to(dev)
    torch.cuda.synchronize()

    def barrier():
        if ws > 1:
            import torch.distributed as dist
            dist.barrier()

    # warm-up (also packs the weights and sizes the workspace)
    for _ in range(args.warmup):
        gen._batched_block_forward(ids_dev, cache)
    torch.cuda.synchronize()
    gen._fold_draft_positions = 0
    gen._fold_draft_recomputed = 0

    # ---- device-resident timed region (no instrumentation inside it)
    launches0 = _lib.launch_count()
    stream = torch.cuda.current_stream(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        torch.cuda.synchronize()
        t0.record(stream)
        for _ in range(args.steps):
            gen._batched_block_forward(ids_dev, cache)
        t1.record(stream)
        torch.cuda.synchronize()
        barrier()
    launches = _lib.launch_count() - launches0
    ms = t0.elapsed_time(t1)
    fold_ratio = gen.fold_ratio
    recomputed_rows = (gen._fold_draft_recomputed + args.steps * dims.layers * N) / (
        args.steps * dims.layers)

    # ---- the same steps again with a CUDA-event pair around every kernel launch (on the
    # launching stream): per-kernel durations for the roofline and the breakdown.  Kept
    # out of the timed region above because recording ~600 events per step slows the
    # host enough to leave gaps between kernels.
    _lib.profile_begin(args.steps * (dims.layers * 9 + 4))
    for _ in range(args.steps):
        gen._batched_block_forward(ids_dev, cache)
    torch.cuda.synchronize()
    prof = _lib.profile_end()

    # ---- end to end through the public call with host buffers
    host_ids = ids.pin_memory()
    host_out = torch.empty(B1, N, dtype=torch.int64).pin_memory()
    for _ in range(2):
        d = host_ids.to(dev, non_blocking=True)
        host_out.copy_(gen._batched_block_forward(d, cache).argmax(-1), non_blocking=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        d = host_ids.to(dev, non_blocking=True)
        host_out.copy_(gen._batched_block_forward(d, cache).argmax(-1), non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1)

    # ---- decode tok/s: whole sequences through the decode loop (prefill, verify steps,
    # draft construction, sampling, block commits), device-timed, max over ranks
    decode = None
    dec_ms = 0.0
    if args.decode_streams > 0:
        barrier()
        runs, dec_ms = decode_leg(gen, model, dims, args.decode_streams, rank, dev)
        barrier()
    # ---- max over ranks
    ms, e2e_ms, dec_ms = max_over_ranks([ms, e2e_ms, dec_ms], dev)
    if args.decode_streams > 0:
        tok = sum(r["tokens_generated"] for r in runs)
        calls = sum(r["model_calls"] for r in runs)
        verify = sum(sum(1 for k, _ in r["steps"] if k == "forward") for r in runs)
        hits = sum(r["draft_hits"] for r in runs)
        fr = [r["fold_ratio"] for r in runs]
        decode = {"tok_s": round(ws * tok / (dec_ms / 1e3), 2), "unit": "tok/s",
                  "streams": ws * args.decode_streams, "prompt": DECODE_PROMPT,
                  "new_tokens": DECODE_NEW, "tokens_per_stream": tok / len(runs),
                  "ms_per_stream": round(dec_ms / len(runs), 2),
                  "model_calls_per_stream": calls / len(runs),
                  "verify_calls_per_stream": verify / len(runs),
                  "draft_hits_per_stream": hits / len(runs),
                  "tokens_per_verify_call": round(tok / max(verify, 1), 3),
                  "fold_ratio": round(sum(fr) / len(fr), 4),
                  "timing": "CUDA events around whole sequences on the launching stream "
                            "(the loop synchronises every step), max over ranks",
                  "workload": "1024-token random prompt, 512 new tokens, block 32, small "
                              "block 8, graph B=7 D=8 S=3, delta 0.1, threshold 0.9, seeded "
                              "per-position logit bias (60% strong)"}
    step_ms = ms / args.steps
    value = weak_scaling_value(ws, args.steps, ms)
    e2e_value = weak_scaling_value(ws, args.steps, e2e_ms)

    hbm, tflops, src = peaks()
    wbytes, kvbytes = algorithmic_bytes(dims, P_PREFIX)
    # dominant kernel: the chained layer tail, one launch per layer -- o_proj + residual
    # (split-K reduction fused into the norm), post-attention RMSNorm, gate/up + SwiGLU,
    # down (SF_CHAIN=2, the default: (H*hd + 3*I) x D bf16 weights), or the FFN alone
    # (SF_CHAIN=1: 3 x I x D), or gate/up alone when not chained
    if prof.get("ffn", (0.0, 0))[1]:
        gu_bytes = 3 * 2 * dims.inter * dims.hidden
        if int(os.environ.get("SF_CHAIN", "2")) >= 2:
            dom, dom_name = "ffn", ("layer tail chain (tcgen05 o_proj + residual, RMSNorm, "
                                    "gate/up + SwiGLU, down; one launch)")
            gu_bytes += 2 * dims.heads * dims.head_dim * dims.hidden
        else:
            dom, dom_name = "ffn", "ffn chain (RMSNorm + tcgen05 gate/up + SwiGLU + down, one launch)"
    else:
        dom, dom_name = "gate_up", "gate_up (tcgen05 swap-AB GEMM + SwiGLU)"
        gu_bytes = 2 * 2 * dims.inter * dims.hidden
    gu_ms, gu_calls = prof.get(dom, (0.0, 0))
    gu_avg_s = gu_ms / max(gu_calls, 1) / 1e3
    achieved = gu_bytes / gu_avg_s / 1e9 if gu_avg_s > 0 else 0.0
    traffic = profiled_traffic("layer_tail" if "layer tail" in dom_name else dom)
    step_achieved = (wbytes + kvbytes) / (step_ms / 1e3) / 1e9
    clocks = clk.summary()
    kernels = {k: {"ms_per_step": round(v[0] / args.steps, 4), "calls_per_step": v[1] / args.steps}
               for k, v in prof.items() if v[1]}

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline(budget_s=args.cpu_budget)

    line = {
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4),
        "verify_step_us": round(step_ms * 1e3, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init N(0,0.02) weights of the named shape; seeded "
                "configuration-0 draft noise)",
        "config": {"workload": "folded verify step, Qwen2.5-7B shape, B1=8 (main + 7 drafts), "
                               "N=32, prefix 1024, delta 0.1",
                   "shape": SHAPE, "B1": B1, "N": N, "prefix": P_PREFIX, "delta": DELTA,
                   "fold_ratio": round(fold_ratio, 4),
                   "recomputed_rows_per_layer": round(recomputed_rows, 1),
                   "parallelism": f"dp{ws} (independent streams, no collectives)",
                   "l2": "inputs larger than L2 (15 GB of weights streamed per step)"},
        "decode": decode,
        "e2e": {"value": round(e2e_value, 4), "unit": UNIT,
                "ms_per_step": round(e2e_ms / args.steps, 4),
                "h2d_bytes_per_step": B1 * N * 8, "d2h_bytes_per_step": B1 * N * 8},
        "roofline": {"bound": "hbm", "kernel": dom_name,
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "peak_source": src,
                     "algorithmic_bytes_per_launch": gu_bytes,
                     "launch_ms": round(gu_avg_s * 1e3, 4), "traffic": traffic,
                     "step_bytes": wbytes + kvbytes,
                     "step_achieved_gbs": round(step_achieved, 1),
                     "step_frac": round(step_achieved / hbm, 4)},
        "kernels": kernels,
        "gpu_launches": int(launches),
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def cpu_model_name() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class CpuReference:
    """Reference PyTorch folded forward (oracle restatement) on the host cores: one
    decoder layer of the 7B shape at the bench inputs plus the LM head.  A step is
    extrapolated as layers x (t(layer + head) - t(head)) + t(head), each term the median
    of the same number of samples after one warm-up, at a given thread count -- the same
    procedure in both arms of the benchmark."""

    def __init__(self):
        from specfold_b200 import synthetic as syn
        self.all_threads = os.cpu_count() or 1
        self.layers_full = syn.SHAPES[SHAPE].layers
        self.dims, self.model, self.cache, self.ids = build_workload("cpu", layers=1)
        self.x = torch.randn(B1 * N, self.dims.hidden).to(torch.bfloat16)

    def _full(self):
        from oracle import folded_oracle as orc
        t = time.perf_counter()
        orc.folded_forward(self.model, self.ids, self.cache, DELTA)
        return time.perf_counter() - t

    def _head(self):
        t = time.perf_counter()
        self.model.lm_head(self.model.model.norm(self.x))
        return time.perf_counter() - t

    @torch.no_grad()
    def measure(self, threads: int, samples: int, budget_s: float):
        torch.set_num_threads(threads)
        self._full(), self._head()                                  # warm
        full, head, start = [], [], time.perf_counter()
        while len(full) < samples and (not full or time.perf_counter() - start < budget_s):
            full.append(self._full())
            head.append(self._head())
        f, h = statistics.median(full), statistics.median(head)
        step = self.layers_full * max(f - h, 1e-6) + h
        return {"step_s": round(step, 4), "value": round(1.0 / step, 6), "threads": threads,
                "samples": len(full), "layer_s": round(f - h, 5), "lm_head_s": round(h, 5)}

    def describe(self, allc, one=None):
        out = {"value": allc["value"], "unit": UNIT, "cores": allc["threads"], "kind": "port",
               "cpu_model": cpu_model_name(), "step_s_extrapolated": allc["step_s"],
               "all_threads": allc,
               "sample": f"1 decoder layer + LM head of the 7B shape at the bench inputs "
                         f"(bf16, P={P_PREFIX}), medians of {allc['samples']} samples each "
                         f"after one warm-up, extrapolated to {self.layers_full} layers"}
        if one is not None:
            out["one_thread"] = one
        return out


def cpu_baseline(budget_s=30.0):
    ref = CpuReference()
    allc = ref.measure(ref.all_threads, 5, budget_s / 2)
    one = ref.measure(1, 3, budget_s / 2)
    torch.set_num_threads(ref.all_threads)
    return ref.describe(allc, one)


def run_reference(args):
    ws, rank, local = dist_env()
    if rank != 0:
        return
    ref = CpuReference()
    allc = ref.measure(ref.all_threads, max(args.steps, 5), args.cpu_budget)
    one = ref.measure(1, 3, args.cpu_budget)
    cpu = ref.describe(allc, one)
    step_s = allc["step_s"]
    line = {
        "metric": METRIC, "value": cpu["value"], "unit": UNIT, "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_s * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "impl": "reference", "data": "synthetic",
        "config": {"workload": "folded verify step, Qwen2.5-7B shape, B1=8 (main + 7 drafts), "
                               "N=32, prefix 1024, delta 0.1",
                   "note": "host cores; 1 layer + LM head timed per step, extrapolated to 28"},
        "cpu_baseline": cpu,
        "e2e": {"value": cpu["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _import_reference(root):
    """The reference's folded generators from an installed copy (baseline/_ref): the
    package __init__ modules import the vendored NLD model and the executors, which the
    folded forwards do not use, so the packages are registered as bare namespaces first
    and the two NLD modules nld_folded imports are stubbed."""
    import importlib
    import types
    for name in ("specfold", "specfold.generate", "specfold.model_cache",
                 "specfold.model_cache.nemotron_labs_diffusion"):
        mod = types.ModuleType(name)
        mod.__path__ = [os.path.join(root, *name.split("."))]
        sys.modules[name] = mod
    ex = types.ModuleType("specfold.generate.nld_model_executor")
    ex.NLDModelExecutor = object
    sys.modules[ex.__name__] = ex
    mdl = types.ModuleType("specfold.model_cache.nemotron_labs_diffusion.modeling_nemotron_labs_diffusion")
    mdl._get_num_transfer_tokens = mdl._get_transfer_index = None
    sys.modules[mdl.__name__] = mdl
    sys.path.insert(0, root)
    return importlib.import_module("specfold.generate.fastdllm_v2_folded")


def run_triton_reference(args):
    """The reference's own fused generator, SpecFoldTritonFastDLLMV2Generation
    (specfold/generate/fastdllm_v2_folded.py:226-370, its Triton kernels JIT-compiled for
    this GPU), timed at the benchmark workload on one GPU: the kernel-level bar for the
    B200 path.  Needs the reference installed under baseline/_ref (pip --target); prints
    an "unavailable" line otherwise.  Not the driver's reference arm (that is the CPU
    path, --impl reference)."""
    ws, rank, local = dist_env()
    if rank != 0:
        return
    root = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(root, "specfold")):
        print(json.dumps({"impl": "reference-triton", "unavailable": "baseline/_ref not installed"}))
        return
    fd = _import_reference(root)
    from specfold_b200.synthetic import StandinExecutor
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dims, model, cache, ids = build_workload(dev)
    gen = object.__new__(fd.SpecFoldTritonFastDLLMV2Generation)
    gen.model_executor = StandinExecutor(model)
    gen.delta = DELTA
    gen.fold_bucket = None
    gen._fold_stats = []
    ids = ids.to(dev)
    with torch.no_grad():
        for _ in range(args.warmup):
            gen._batched_block_forward(ids, cache)
        torch.cuda.synchronize()
        gen._fold_draft_positions = gen._fold_draft_recomputed = 0
        stream = torch.cuda.current_stream(dev)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            torch.cuda.synchronize()
            t0.record(stream)
            for _ in range(args.steps):
                gen._batched_block_forward(ids, cache)
            t1.record(stream)
            torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    print(json.dumps({
        "metric": METRIC, "impl": "reference-triton", "value": round(args.steps / (ms / 1e3), 4),
        "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "dtype": "bf16",
        "fold_ratio": round(gen.fold_ratio, 4),
        "config": {"workload": "folded verify step, Qwen2.5-7B shape, B1=8 (main + 7 drafts), "
                               "N=32, prefix 1024, delta 0.1",
                   "generator": "SpecFoldTritonFastDLLMV2Generation (reference, Triton)"},
        "clocks": clk.summary()}), flush=True)


def run_tp(args):
    """The 14B tensor-parallel configuration: a Llama-style 14B-shape model, tensor
    parallel over all torchrun ranks (heads and the intermediate dimension sharded, o_proj
    and down partials summed over NVLink: peer memory by default, NCCL with
    SF_TP_TRANSPORT=nccl), one verify stream, prefix 2048.  Strong scaling:
    the whole group serves one stream; value = verify steps/s of that stream."""
    from specfold_b200 import SpecFoldB200NLDGeneration, _lib
    from specfold_b200 import synthetic as syn
    import datetime
    import torch.distributed as dist

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    _lib.check(_lib.load().sf_check_device(), "device")
    dims = syn.SHAPES["llama14b"]
    P = 2048
    model = syn.build_model(dims, family="nld", dtype=torch.bfloat16, seed=0, device=str(dev))
    cache = syn.random_prefix_cache(dims, P, dtype=torch.bfloat16, seed=1, device=str(dev))
    hidden = syn.config0_hidden(dims, B1, N, dtype=torch.bfloat16, seed=3,
                                frac_recompute=FRAC_RECOMPUTE)
    syn.inject_hidden(model, hidden.to(dev))
    gen = SpecFoldB200NLDGeneration(model_executor=syn.StandinExecutor(model), delta=DELTA)
    transport = "one GPU"
    if ws > 1:
        gen.set_tensor_parallel(rank, ws)
        transport = ("NCCL all-reduce" if gen._tp_transport == "nccl"
                     else "peer memory (NVLink loads, flag handshake)")
    ids = torch.zeros(B1, N, dtype=torch.int64, device=dev)
    for _ in range(args.warmup):
        gen._batched_block_forward(ids, cache)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0.record(stream)
        for _ in range(args.steps):
            gen._batched_block_forward(ids, cache)
        t1.record(stream)
        torch.cuda.synchronize()
        if ws > 1:
            dist.barrier()
    ms = max_over_ranks([t0.elapsed_time(t1)], dev)[0]
    # per-kernel breakdown (direct launches with CUDA events around each, outside the timed
    # region; the all-reduces and their residual / scatter kernels are "tp_reduce")
    _lib.profile_begin(args.steps * (dims.layers * 12 + 4))
    for _ in range(args.steps):
        gen._batched_block_forward(ids, cache)
    torch.cuda.synchronize()
    prof = _lib.profile_end()
    kernels = {k: {"ms_per_step": round(v[0] / args.steps, 4), "calls_per_step": v[1] / args.steps}
               for k, v in prof.items() if v[1]}
    step_ms = ms / args.steps
    hbm, _, src = peaks()
    wbytes, kvbytes = algorithmic_bytes(dims, P)
    # per GPU: its shard of the layers + the replicated LM head + its kv heads
    head = 2 * dims.vocab * dims.hidden
    per_gpu = (wbytes - head) / ws + head + kvbytes / ws
    line = {
        "metric": "folded verify-step, 14B Llama shape, tensor parallel", "value": round(args.steps / (ms / 1e3), 4),
        "unit": UNIT, "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step_ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init 14B shape)",
        "config": {"workload": "folded verify step, Llama-style 14B shape, B1=8, N=32, prefix 2048, "
                               "delta 0.1", "shape": "llama14b", "prefix": P,
                   "parallelism": f"tp{ws} (heads / intermediate sharded; fp32 partials of o_proj "
                                  f"and down summed over {transport})",
                   "fold_ratio": round(gen.fold_ratio, 4)},
        "roofline": {"bound": "hbm", "per_gpu_bytes": int(per_gpu),
                     "achieved": round(per_gpu / (step_ms / 1e3) / 1e9, 1), "peak": hbm,
                     "unit": "GB/s", "peak_source": src,
                     "frac": round(per_gpu / (step_ms / 1e3) / 1e9 / hbm, 4)},
        "kernels": kernels,
        "clocks": clk.summary(),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ws > 1:
        gen.close_tensor_parallel()
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference", "reference-triton"], default="b200")
    ap.add_argument("--cpu-budget", type=float, default=30.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--decode-streams", type=int, default=2,
                    help="sequences each rank decodes for the decode tok/s figure (0: skip)")
    ap.add_argument("--tp", action="store_true",
                    help="the 14B tensor-parallel configuration over all ranks instead")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.tp and args.impl == "b200":
        run_tp(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.impl == "reference-triton":
        run_triton_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
