"""ctypes binding of ``libdsv4attn.so`` (the C ABI declared in include/dsv4attn.h).

The library is built in-tree by ``tt-deepseek-v4_b200/build.py``.  There is no
fallback: if the library is missing or cannot be loaded every op raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdsv4attn.so")

DSA_OK = 0
DSA_ERR_ARG = -1
DSA_KEYS_READY = 1  # dsa_indexer_score_ex flag
DSA_ERR_CUDA = -2
DSA_ERR_UNSUPPORTED = -3
DSA_ERR_TIMEOUT = -4
DSA_ERR_WORKSPACE = -5

P = ctypes.c_void_p
I32 = ctypes.c_int
I64 = ctypes.c_int64
F32 = ctypes.c_float
SZ = ctypes.c_size_t

DSA_BESIDE_PREVIOUS = 1  # dsa_layer_prologue flag


class CompressorArgs(ctypes.Structure):
    """dsa_compressor_args (include/dsv4attn.h)."""
    _fields_ = [("kv_row", P), ("score_row", P), ("ld_row", I64), ("ape", P), ("kv_state", P),
                ("score_state", P), ("gamma", P), ("kv_cache", P), ("cache_bstride", I64), ("cache_rows", I64),
                ("slot_offset", I32), ("d", I32), ("rope_dim", I32), ("ratio", I32), ("overlap", I32),
                ("rotate", I32)]


# name -> (restype, argtypes); must match include/dsv4attn.h
PROTOTYPES = {
    "dsa_version": (I32, []),
    "dsa_last_error": (ctypes.c_char_p, []),
    "dsa_set_wait_limit": (I32, [ctypes.c_longlong]),
    "dsa_get_wait_limit": (ctypes.c_longlong, []),
    "dsa_linear": (I32, [P, I64, P, P, I64, I32, I32, I32, I32, I32, P, P, I32, P, I32, I32, I32, P, P]),
    "dsa_linear_packed_bytes": (ctypes.c_size_t, [I32, I32, I32]),
    "dsa_linear_pack": (I32, [P, I32, I32, I32, P, ctypes.c_size_t, P]),
    "dsa_act_quant_block": (I32, [P, P, P, P, I64, I64, I64, I64, I32, F32, F32, P]),
    "dsa_kv_window_write": (I32, [P, P, P, P, I32, I32, I32, I64, I32, I32, P]),
    "dsa_kv_norm_rope_window_write": (I32, [P, I64, P, F32, P, P, I32, P, P, I64, I32, P, I64, P, I32, I32,
                                            I32, P, P]),
    "dsa_head_norm_rope": (I32, [P, I64, P, I64, I32, I32, I32, I32, P, F32, I32, F32, P, P, I32, P, I32, P, P]),
    "dsa_fold_index_mask": (I32, [P, P, I64, P, P]),
    "dsa_compressor_step": (I32, [P, P, I64, P, P, P, P, P, P, I32, P, I64, I64, I32, P, P,
                                  I32, I32, I32, I32, I32, I32, I32, F32, P]),
    "dsa_window_indices": (I32, [P, P, I64, I32, I32, P]),
    "dsa_indexer_score": (I32, [P, P, P, P, P, I32, I32, I32, I32, I64, I64, P]),
    "dsa_indexer_score_ex": (I32, [P, P, P, P, P, I32, I32, I32, I32, I64, I64, I32, P]),
    "dsa_indexer_score_dyn": (I32, [P, P, P, P, P, I32, I32, I32, I32, I64, I64, I32, P, P]),
    "dsa_layer_prologue": (I32, [ctypes.POINTER(CompressorArgs), ctypes.POINTER(CompressorArgs), P, P, I32, F32, P,
                                  P, P, P, P, I64, I32, P, P, I32, I32, I32, P, I64, I32, ctypes.c_uint, P]),
    "dsa_indexer_score_newest": (I32, [P, P, I64, P, P, P, I64, I32, I32, P]),
    "dsa_indexer_topk": (I32, [P, I64, P, P, P, I64, I32, I32, I32, I32, I32, I32, P]),
    "dsa_indexer_topk_workspace_size": (SZ, [I32, I32, I32]),
    "dsa_indexer_topk_ws": (I32, [P, I64, P, P, P, I64, I32, I32, I32, I32, I32, I32, P, SZ, P]),
    "dsa_indexer_topk_newest": (I32, [P, I64, P, P, P, I64, I32, I32, I32, I32, I32, I32, P, P, I64, P, P, SZ,
                                       P]),
    "dsa_advance_positions": (I32, [P, P, I32, I32, I32, P]),
    "dsa_topk_merge": (I32, [P, P, I32, P, P, I64, I32, I32, I32, P]),
    "dsa_shard_active": (I32, [P, P, I32, I32, I32, P]),
    "dsa_prefill_positions": (I32, [I32, I32, I32, I32, I32, I32, P, P, I64, P]),
    "dsa_topk_wide_workspace_size": (SZ, [I32, I32]),
    "dsa_topk_wide": (I32, [P, I64, P, I64, P, P, P, I64, I32, I32, I32, I32, I32, I32, I64, P, SZ, P, P]),
    "dsa_shard_local_indices": (I32, [P, I64, I32, P, I64, I32, I32, I32, I32, I32, P, I64, I32, P]),
    "dsa_sparse_attn_workspace_size": (SZ, [I32, I32, I32, I32, I32]),
    "dsa_sparse_attn": (I32, [P, P, I64, I64, P, I64, P, P, P, I32, I32, I32, I32, I32, F32, P, SZ, P, P]),
    "dsa_sparse_attn_ex": (I32, [P, P, I64, I64, P, I64, P, P, P, I32, I32, I32, I32, I32, F32, P, SZ, I32,
                                 ctypes.c_uint, P, P]),
    "dsa_sparse_attn_noalloc": (I32, [P, P, I64, I64, P, I64, P, P, P, I32, I32, I32, I32, I32, F32, P, P]),
    "dsa_sparse_attn_partial": (I32, [P, P, I64, I64, P, I64, P, P, I32, I32, I32, I32, I32, F32, P, SZ, P, P]),
    "dsa_lse_combine": (I32, [P, P, P, P, I32, I32, I32, I32, P]),
    "dsa_lse_combine_strided": (I32, [P, I64, P, I64, P, P, I32, I32, I32, I32, P]),
    "dsa_set_trace": (I32, [P, SZ]),
    "dsa_p2p_alloc": (I32, [SZ, P]),
    "dsa_p2p_free": (I32, [P]),
    "dsa_p2p_handle_size": (SZ, []),
    "dsa_p2p_export": (I32, [P, P, P]),
    "dsa_p2p_import": (I32, [P, P]),
    "dsa_p2p_close": (I32, [P]),
    "dsa_p2p_publish": (I32, [P, SZ, P, P, P, I32, P, P]),
    "dsa_p2p_wait": (I32, [P, I32, P, P, P]),
    "dsa_counter_bump": (I32, [P, P]),
}

_lock = threading.Lock()
_lib = None


class NativeLibraryError(RuntimeError):
    pass


def lib():
    """Load (once) and return the ctypes handle; raises if the .so is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise NativeLibraryError(
                    f"dsv4attn native library not found at {LIB_PATH}; "
                    "build it with `python tt-deepseek-v4_b200/build.py` (nvcc, sm_100a)")
            h = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in PROTOTYPES.items():
                fn = getattr(h, name)
                fn.restype = res
                fn.argtypes = args
            _lib = h
    return _lib


def last_error() -> str:
    msg = lib().dsa_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    """Map a C status to the reference's Python error conventions:
    ValueError for shape/argument problems (inference.py:3036-3044,
    4394-4397), RuntimeError for device failures (4949-4952)."""
    if rc == DSA_OK:
        return
    msg = last_error() or f"status {rc}"
    if rc in (DSA_ERR_ARG, DSA_ERR_WORKSPACE, DSA_ERR_UNSUPPORTED):
        raise ValueError(f"{what}: {msg}")
    if rc == DSA_ERR_TIMEOUT:
        raise TimeoutError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg}")


def exported_symbols():
    return sorted(PROTOTYPES)
