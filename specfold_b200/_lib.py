"""ctypes binding of libspecfold_b200.so (declarations: include/specfold_b200.h).

There is no fallback: if the library is missing or was built for another
architecture, every entry point raises.  Build it with ``python -m specfold_b200.build``.
"""

from __future__ import annotations

import ctypes as C
import os
import threading

from . import build as _build

_LOCK = threading.Lock()
_LIB = None

c_void_p, c_int, c_float, c_int64, c_size_t = C.c_void_p, C.c_int, C.c_float, C.c_int64, C.c_size_t

SF_DTYPE_F32 = 0
SF_DTYPE_BF16 = 1
DEV_ERR_BITS = {1: "barrier wait timed out", 2: "index out of range", 4: "parent chain too deep",
                8: "TMEM allocation failed"}


class SfLayer(C.Structure):
    _fields_ = [(n, c_void_p) for n in ("w_qkv", "b_qkv", "ln1_w", "w_o", "ln2_w", "w_gate",
                                        "w_up", "w_down", "prefix_k", "prefix_v")]


class SfVerifyArgs(C.Structure):
    _fields_ = [
        ("dtype", c_int), ("B1", c_int), ("N", c_int), ("D", c_int), ("H", c_int),
        ("Hkv", c_int), ("hd", c_int), ("I", c_int), ("V", c_int), ("L", c_int), ("P", c_int),
        ("kv_head_stride", c_int64), ("bucket", c_int),
        ("delta", c_float), ("eps", c_float), ("scale", c_float), ("shift_logits", c_int),
        ("weights_tiled", c_int),
        ("layers", C.POINTER(SfLayer)), ("final_norm_w", c_void_p), ("lm_w", c_void_p),
        ("par_idx", c_void_p), ("hidden_in", c_void_p), ("cos", c_void_p), ("sin", c_void_p),
        ("q_scale", c_void_p), ("logits", c_void_p), ("count_slab", c_void_p),
        ("segcnt_slab", c_void_p), ("rec_slab", c_void_p), ("ws", c_void_p),
        ("ws_bytes", c_size_t), ("err", c_void_p), ("stream", c_void_p),
        ("tp_comm", c_void_p), ("tp_size", c_int),
        ("P_dev", c_void_p), ("commit", c_int), ("tp_peers", c_void_p), ("prefill", c_int),
    ]


# name -> (restype, argtypes); mirrors include/specfold_b200.h
_SIGS = {
    "sf_last_error": (C.c_char_p, []),
    "sf_abi_version": (c_int, []),
    "sf_check_device": (c_int, []),
    "sf_residual_delta_gate": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_void_p, c_void_p, c_float, c_int, c_int, c_int, c_int,
                                       c_float, c_void_p, c_void_p]),
    "sf_src_resolve": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "sf_workspace_bytes": (c_size_t, [c_int] * 7),
    "sf_workspace_init": (c_int, [c_void_p, c_size_t, c_void_p]),
    "sf_fused_ln_qkv_rope_scatter": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                             c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                             c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
                                             c_void_p, c_size_t, c_void_p, c_void_p]),
    "sf_flash_attn_gqa": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_int64, c_void_p,
                                  c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_int, c_int, c_float, c_int, c_int, c_int, c_int, c_int,
                                  c_void_p, c_size_t, c_void_p, c_void_p]),
    "sf_attn_workspace_bytes": (c_size_t, [c_int] * 6),
    "sf_chain_correction_gqa": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                        c_int, c_float, c_int, c_int, c_int, c_void_p,
                                        c_void_p]),
    "sf_o_proj_residual": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                   c_int, c_void_p, c_size_t, c_void_p, c_void_p]),
    "sf_fused_ffn_scatter": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                     c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p,
                                     c_void_p, c_float, c_int, c_int, c_void_p, c_size_t,
                                     c_void_p, c_void_p]),
    "sf_fused_ffn_scatter_static": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                            c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                            c_float, c_int, c_int, c_void_p, c_void_p]),
    "sf_combine": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                           c_void_p, c_void_p]),
    "sf_final_norm_lm_head": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_int, c_int, c_int, c_int, c_float, c_int, c_void_p,
                                      c_size_t, c_void_p, c_void_p]),
    "sf_kv_append": (c_int, [c_int, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int64,
                             c_int, c_int, c_int, c_int, c_void_p]),
    "sf_sample_top_p_greedy": (c_int, [c_int, c_void_p, c_int64, c_int, c_int64, c_float,
                                       c_void_p, c_void_p, c_void_p]),
    "sf_draft_workspace_bytes": (c_size_t, [c_int, c_int]),
    "sf_draft_blocks": (c_int, [c_int, c_void_p, c_int64, c_int, c_int, c_int, c_int, c_void_p,
                                c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_void_p,
                                c_void_p, c_void_p, c_size_t, c_void_p]),
    "sf_weight_tiles_bytes": (c_size_t, [c_int] * 4),
    "sf_parent_map": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "sf_tp_unique_id": (c_int, [c_void_p, c_int]),
    "sf_tp_comm_init": (c_int, [c_void_p, c_int, c_int, C.POINTER(c_void_p)]),
    "sf_tp_comm_destroy": (c_int, [c_void_p]),
    "sf_tp_exchange_bytes": (c_size_t, [c_int, c_int]),
    "sf_tp_peers_init": (c_int, [c_int, c_int, C.POINTER(c_void_p), c_int, c_int,
                                 C.POINTER(c_void_p)]),
    "sf_tp_peers_destroy": (c_int, [c_void_p]),
    "sf_tp_ipc_export": (c_int, [c_void_p, c_void_p, c_int, C.POINTER(c_size_t)]),
    "sf_tp_ipc_open": (c_int, [c_void_p, c_int, C.POINTER(c_void_p)]),
    "sf_tp_ipc_close": (c_int, [c_void_p]),
    "sf_release_graphs": (c_int, []),
    "sf_pack_weight_tiles": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                                     c_void_p]),
    "sf_launch_count": (C.c_longlong, []),
    "sf_profile_begin": (c_int, [c_int]),
    "sf_profile_end": (c_int, []),
    "sf_profile_kinds": (c_int, []),
    "sf_profile_name": (C.c_char_p, [c_int]),
    "sf_profile_kind": (c_int, [c_int, C.POINTER(C.c_double), C.POINTER(c_int)]),
    "sf_verify_workspace_bytes": (c_size_t, [c_int] * 10),
    "sf_folded_verify_forward": (c_int, [C.POINTER(SfVerifyArgs)]),
}


def library_path() -> str:
    return _build.LIB


def load(build_if_missing: bool = False):
    """The loaded library; raises if it is not built (or builds it when asked)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        path = library_path()
        if not os.path.exists(path):
            if not build_if_missing:
                raise RuntimeError(
                    f"libspecfold_b200.so not found at {path}; build it with "
                    "`python -m specfold_b200.build` (the CUDA path has no fallback)")
            _build.build()
        lib = C.CDLL(path)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
        return lib


def exported_symbols():
    return list(_SIGS)


class SpecFoldError(RuntimeError):
    pass


def check(status: int, what: str = "") -> None:
    if status != 0:
        msg = load().sf_last_error().decode(errors="replace")
        raise SpecFoldError(f"{what or 'specfold_b200'} failed (status {status}): {msg}")


def describe_device_error(bits: int) -> str:
    return ", ".join(v for k, v in DEV_ERR_BITS.items() if bits & k) or f"code {bits}"


def profile_begin(capacity: int) -> None:
    check(load().sf_profile_begin(int(capacity)), "profile_begin")


def profile_end() -> dict:
    """{kind name: (total ms, calls)} of the launches timed since profile_begin."""
    lib = load()
    check(lib.sf_profile_end(), "profile_end")
    out = {}
    for k in range(lib.sf_profile_kinds()):
        ms, calls = C.c_double(), c_int()
        check(lib.sf_profile_kind(k, C.byref(ms), C.byref(calls)), "profile_kind")
        out[lib.sf_profile_name(k).decode()] = (ms.value, calls.value)
    return out


def launch_count() -> int:
    return int(load().sf_launch_count())
