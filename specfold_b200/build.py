"""Builds libspecfold_b200.so (the C-ABI library) in-tree with nvcc for sm_100a.

    python -m specfold_b200.build [--verbose]

The library links the CUDA runtime statically and resolves the driver entry point it
needs (cuTensorMapEncodeTiled) at run time, so it depends on nothing beyond libcuda.
"""

from __future__ import annotations

import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libspecfold_b200.so")
SOURCES = ["gate.cu", "gemm.cu", "gemm_tc.cu", "attention.cu", "attention_tc.cu",
           "attention_rows_mma.cu", "attention_rows_tc.cu", "merge.cu", "tp.cu", "capi.cu", "ffn_static.cu", "sample.cu",
           "draft.cu"]
HEADERS = ["sf_common.cuh", "sf_kernels.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    return "nvcc"


def _digest() -> str:
    h = hashlib.sha256()
    for name in SOURCES + HEADERS:
        with open(os.path.join(CSRC, name), "rb") as f:
            h.update(f.read())
    with open(os.path.join(INCLUDE, "specfold_b200.h"), "rb") as f:
        h.update(f.read())
    h.update(" ".join(ARCH).encode())
    return h.hexdigest()


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> str:
    os.makedirs(LIBDIR, exist_ok=True)
    stamp = LIB + ".sha256"
    digest = _digest()
    if not force and os.path.exists(LIB) and os.path.exists(stamp):
        with open(stamp) as f:
            if f.read().strip() == digest:
                return LIB
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
                    "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]
    if ptxas_verbose:
        flags += ["-Xptxas", "-v"]
    objs = [os.path.join(LIBDIR, src.replace(".cu", ".o")) for src in SOURCES]
    cmds = [[nvcc(), "-c", os.path.join(CSRC, src), "-o", obj] + flags
            for src, obj in zip(SOURCES, objs)]
    if verbose:
        for cmd in cmds:
            print(" ".join(cmd), flush=True)
    # translation units compile independently: one nvcc per core
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=max(1, min(len(cmds), os.cpu_count() or 1))) as pool:
        for r in list(pool.map(lambda c: subprocess.run(c, capture_output=ptxas_verbose), cmds)):
            if ptxas_verbose:
                sys.stdout.write(r.stdout.decode() + r.stderr.decode())
            if r.returncode != 0:
                if not ptxas_verbose:
                    raise subprocess.CalledProcessError(r.returncode, r.args)
                raise subprocess.CalledProcessError(r.returncode, r.args, r.stdout, r.stderr)
    cmd = [nvcc(), "-shared", "-o", LIB] + objs + ARCH + ["-cudart", "static", "-Xcompiler", "-fPIC",
                                                          "-ldl"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    for o in objs:
        os.remove(o)
    with open(stamp, "w") as f:
        f.write(digest)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv,
                ptxas_verbose="--ptxas" in sys.argv))
