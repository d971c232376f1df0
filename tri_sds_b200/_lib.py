"""ctypes binding of libtsds.so (the C ABI declared in include/tsds.h).

The library is built in-tree (``python -m tri_sds_b200.build``).  There is
no fallback: a missing or unloadable library raises at first use, and every
non-zero status becomes a RuntimeError naming the entry point.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("TSDS_LIB", os.path.join(_HERE, "libtsds.so"))

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_Z = ctypes.c_size_t
_L = ctypes.c_int64

PHASE_GEMM, PHASE_NORM, PHASE_PEER = 0, 1, 2
# the library's default of tsds_set_gemm_dp_rows (tests restore it)
GEMM_DP_ROWS_DEFAULT = 128
GEMM_DP_SLACK_DEFAULT = 100
EPI_STORE, EPI_RESIDUAL, EPI_SWIGLU, EPI_STORE_F32, EPI_QKROPE = 0, 1, 2, 4, 5


class FusedPhase(ctypes.Structure):
    """tsds_fused_phase (include/tsds.h)."""
    _fields_ = [("kind", _I), ("epi", _I), ("x", _P), ("ldx", _I), ("K", _I), ("w", _P), ("n_out", _I),
                ("res_ld", _I), ("res", _P), ("out", _P), ("ldo", _I), ("eps", _F)]


class QkRope(ctypes.Structure):
    """tsds_qk_rope (include/tsds.h)."""
    _fields_ = [("q_norm_w", _P), ("k_norm_w", _P), ("cos", _P), ("sin", _P), ("positions", _P), ("starts", _P),
                ("q_out", _P), ("k_cache", _P), ("v_cache", _P), ("T", _I), ("Hq", _I), ("Hkv", _I), ("S", _I),
                ("rope_len", _I), ("eps", _F)]


class PeerGroup(ctypes.Structure):
    """tsds_peer_group (include/tsds.h)."""
    _fields_ = [("bufs", _P), ("rank", _I), ("tp", _I), ("max_elems", _I)]


# name -> (restype, argtypes); mirrors include/tsds.h
SIGNATURES = {
    "tsds_status_string": (ctypes.c_char_p, [_I]),
    "tsds_abi_version": (_I, []),
    "tsds_launch_count": (ctypes.c_int64, []),
    "tsds_set_pdl": (None, [_I]),
    "tsds_embed": (_I, [_P, _I, _P, _P, _I, _I, _I, _P]),
    "tsds_rms_norm": (_I, [_P, _P, _P, _I, _I, _I, _I, _F, _P]),
    "tsds_prep_chain": (_I, [_P, _I, _I, _I, _P, _P, _P]),
    "tsds_qk_norm_rope_kv": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _F, _P]),
    "tsds_linear_workspace_bytes": (_Z, [_I, _I, _I]),
    "tsds_linear_workspace_header_bytes": (_Z, []),
    "tsds_set_wait_limit_ns": (None, [ctypes.c_ulonglong]),
    "tsds_get_wait_limit_ns": (ctypes.c_ulonglong, []),
    "tsds_set_gemv_max_rows": (None, [_I]),
    "tsds_get_gemv_max_rows": (_I, []),
    "tsds_set_gemv_splitk": (None, [_I]),
    "tsds_get_gemv_splitk": (_I, []),
    "tsds_set_gemm_ctas_per_sm": (None, [_I]),
    "tsds_set_gemm_pair_rows": (None, [_I]),
    "tsds_get_gemm_pair_rows": (_I, []),
    "tsds_set_gemm_dp_rows": (None, [_I]),
    "tsds_get_gemm_dp_rows": (_I, []),
    "tsds_set_gemm_dp_slack": (None, [_I]),
    "tsds_get_gemm_dp_slack": (_I, []),
    "tsds_tc_gemm_plan": (_I, [_I, _I, _I, _I, _P]),
    "tsds_linear": (_I, [_P, _I, _P, _P, _I, _I, _I, _I, _P, _Z, _P]),
    "tsds_linear_residual": (_I, [_P, _I, _P, _P, _P, _I, _I, _I, _I, _P, _Z, _P]),
    "tsds_linear_residual_norm": (_I, [_P, _I, _P, _P, _P, _I, _I, _I, _I, _P, _P, _I, _F, _P, _Z, _P]),
    "tsds_linear_swiglu": (_I, [_P, _I, _P, _P, _I, _I, _I, _I, _P, _Z, _P]),
    "tsds_linear_bias": (_I, [_P, _I, _P, _P, _P, _I, _I, _I, _I, _P, _Z, _P]),
    "tsds_logits_topk": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _P]),
    "tsds_tree_state_bytes": (_Z, [_I]),
    "tsds_tree_init": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I, _P]),
    "tsds_tree_step": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _I, _P]),
    "tsds_tree_finalize": (_I, [_P, _I, _I, _P, _P, _P, _P, _P, _P, _P, _I, _P]),
    "tsds_accept_tree": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "tsds_accept_tree_rule": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "tsds_tree_commit": (_I, [_P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _I, _P, _I, _I, _P, _P]),
    "tsds_eagle_inputs": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "tsds_attention_workspace_bytes": (_Z, [_I, _I, _I, _I, _I, _I, _I]),
    "tsds_verify_attention": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _F, _P, _Z, _P, _P]),
    "tsds_set_attention_tc": (None, [_I]),
    "tsds_get_attention_tc": (_I, []),
    "tsds_verify_attention_paged": (_I, [_P, _P, _P, _P, _P, _P, _I, _P, _L, _P, _L, _I, _I, _I, _I, _I, _I, _I,
                                         _I, _F, _P, _Z, _P, _P]),
    "tsds_qk_norm_rope_kv_paged": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _L, _I, _F, _P,
                                        _P]),
    "tsds_tree_commit_paged": (_I, [_P, _L, _P, _P, _P, _P, _I, _P, _P, _I, _I, _P, _I, _P]),
    "tsds_attention_plan": (_I, [_I, _I, _I, _I, _I, _I, _I, _P]),
    "tsds_table_rows": (_I, [_P, _L, _P, _P, _I, _I, _P, _P]),
    "tsds_verify_attention_noalloc_limit": (_Z, []),
    "tsds_verify_attention_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _F, _P]),
    "tsds_verify_attention_noalloc_status": (_I, [_P]),
    "tsds_lm_head_workspace_bytes": (_Z, [_I, _I]),
    "tsds_lm_head_argmax": (_I, [_P, _I, _P, _P, _P, _I, _P, _I, _I, _I, _P, _Z, _P]),
    "tsds_linear_f32": (_I, [_P, _I, _P, _P, _I, _I, _I, _I, _P, _Z, _P]),
    "tsds_residual_add_f32": (_I, [_P, _P, _I, _I, _P]),
    "tsds_argmax_merge": (_I, [_P, _P, _I, _I, ctypes.c_int64, _P, _I, _P]),
    "tsds_gather_shards": (_I, [_P, _P, _I, _I, _I, _P]),
    "tsds_fused_layer_workspace_bytes": (_Z, [_I]),
    "tsds_fused_layer_workspace_header_bytes": (_Z, []),
    "tsds_fused_layer_grid": (_I, [_I, _P]),
    "tsds_fused_layer": (_I, [_P, _I, _I, _P, _P, _P, _Z, _P]),
    "tsds_peer_buffer_bytes": (_Z, [_I, _Z]),
    "tsds_peer_slot_offset": (_Z, [_I, _I]),
    "tsds_peer_exchange_offset": (_Z, [_I]),
    "tsds_peer_lm_gather": (_I, [_P, _I, _I, _I, _Z, _I, _I, ctypes.c_int64, ctypes.c_int64, _P, _I, _P, _P, _P]),
    "tsds_peer_handle_bytes": (_Z, []),
    "tsds_peer_alloc": (_I, [_Z, ctypes.POINTER(_P)]),
    "tsds_peer_free": (_I, [_P]),
    "tsds_peer_export": (_I, [_P, _P]),
    "tsds_peer_import": (_I, [_P, ctypes.POINTER(_P)]),
    "tsds_peer_close": (_I, [_P]),
    "tsds_peer_allreduce_residual": (_I, [_P, _P, _I, _I, _I, _I, _I, _I, _P, _P]),
    "tsds_accept_greedy": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _P]),
    "tsds_gather_ids": (_I, [_P, _P, _P, _P, _P, _I, _I, _P]),
}

_lib = None
_lock = threading.Lock()


def load():
    """Load libtsds.so once and attach the ABI signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libtsds.so not found at {LIB_PATH}: build it with `python -m tri_sds_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


def call(name: str, *args) -> None:
    """Call an int-returning entry point; raise on a non-zero status."""
    lib = load()
    st = getattr(lib, name)(*args)
    if st != 0:
        msg = lib.tsds_status_string(st).decode()
        raise RuntimeError(f"{name} failed: status {st} ({msg})")


def query(name: str, *args):
    return getattr(load(), name)(*args)
