"""ctypes binding of the C ABI declared in ``include/ai_attn.h``.

The shared library ``_ai_attn.so`` is built in-tree by
``autoindexer_b200.build`` (``nvcc -gencode arch=compute_100a,code=sm_100a``).
There is no fallback: if the library is missing or cannot be loaded every
attention call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

__all__ = [
    "LIB_PATH",
    "AiTensor4",
    "AiAttnLayout",
    "AiAttnFwdArgs",
    "AiAttnBwdArgs",
    "AiAttnDecodeArgs",
    "DTYPE_BF16",
    "DTYPE_F16",
    "DTYPE_F32",
    "EXPORTED_SYMBOLS",
    "lib",
    "check",
]

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ai_attn.so")

DTYPE_BF16, DTYPE_F16, DTYPE_F32 = 0, 1, 2
# AiProfKind, in order.
PROF_KINDS = ("prerot", "fwd", "fwd_fill", "delta", "dq", "dkdv", "bwd_fill", "simt", "decode")
ABI_VERSION = 9
BWD_DQ, BWD_DKDV = 1, 2

# Every function include/ai_attn.h declares.
EXPORTED_SYMBOLS = (
    "ai_attn_abi_version",
    "ai_attn_fwd_tile_rows",
    "ai_attn_kv_tile_rows",
    "ai_attn_fwd",
    "ai_attn_fwd_workspace",
    "ai_attn_bwd_workspace",
    "ai_attn_bwd",
    "ai_attn_bwd_noalloc",
    "ai_attn_decode_workspace",
    "ai_attn_decode",
    "ai_attn_profile_enable",
    "ai_attn_profile_read",
    "ai_attn_read_status",
    "ai_attn_selftest_wait",
    "ai_attn_strerror",
    "ai_attn_positions_from_ops_sizes",
    "ai_attn_positions_from_ops",
    "ai_attn_prep_sizes",
    "ai_attn_prep",
    "ai_index_fwd",
    "ai_index_bwd",
    "ai_index_rows_sizes",
    "ai_index_rows",
)

_i32p = ctypes.POINTER(ctypes.c_int32)
_f32p = ctypes.POINTER(ctypes.c_float)


class AiTensor4(ctypes.Structure):
    _fields_ = [
        ("ptr", ctypes.c_void_p),
        ("stride_b", ctypes.c_int64),
        ("stride_h", ctypes.c_int64),
        ("stride_t", ctypes.c_int64),
    ]


class AiAttnLayout(ctypes.Structure):
    _fields_ = [
        ("n_blocks", ctypes.c_int32),
        ("blocks", ctypes.c_void_p),
        ("row_blocks", ctypes.c_void_p),
        ("row_cov", ctypes.c_void_p),
        ("key_info", ctypes.c_void_p),
        ("n_keys", ctypes.c_int64),
        ("q_pos", ctypes.c_void_p),
        ("k_own", ctypes.c_void_p),
        ("rope_cos", ctypes.c_void_p),
        ("rope_sin", ctypes.c_void_p),
        ("rope_cs16", ctypes.c_void_p),
        ("n_pos", ctypes.c_int32),
        ("fwd_tile", ctypes.c_int32),
        ("fwd_items", ctypes.c_void_p),
        ("n_fwd_items", ctypes.c_int32),
        ("n_fwd_abs_items", ctypes.c_int32),
        ("kv_tile", ctypes.c_int32),
        ("kv_items", ctypes.c_void_p),
        ("n_kv_items", ctypes.c_int32),
        ("n_kv_abs_items", ctypes.c_int32),
        ("all_rows_owned", ctypes.c_int32),
        ("n_fwd_short_items", ctypes.c_int32),
        ("kv_chunks", ctypes.c_void_p),
        ("n_kv_chunks", ctypes.c_int32),
        ("n_kv_partials", ctypes.c_int32),
        ("kv_reduce", ctypes.c_void_p),
        ("n_kv_reduce", ctypes.c_int32),
        ("kv_cost_max", ctypes.c_int32),
        ("kv_cost_total", ctypes.c_int32),
        ("blk_cls", ctypes.c_void_p),
        ("chunk_cls", ctypes.c_void_p),
        ("n_chunk_cls", ctypes.c_int32),
        ("rot_classes", ctypes.c_void_p),
        ("n_rot_classes", ctypes.c_int32),
        ("n_fwd_abs_short_items", ctypes.c_int32),
    ]


class AiAttnFwdArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32),
        ("seq_len", ctypes.c_int32),
        ("num_q_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("q", AiTensor4),
        ("k", AiTensor4),
        ("v", AiTensor4),
        ("out", AiTensor4),
        ("lse", ctypes.c_void_p),
        ("layout", AiAttnLayout),
        ("status", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
    ]


class AiAttnBwdArgs(ctypes.Structure):
    _fields_ = [
        ("fwd", AiAttnFwdArgs),
        ("dout", AiTensor4),
        ("dq", AiTensor4),
        ("dk", AiTensor4),
        ("dv", AiTensor4),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("fwd_rotated", ctypes.c_int32),
        ("parts", ctypes.c_int32),
    ]


class AiAttnDecodeArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32),
        ("kv_len", ctypes.c_int32),
        ("num_q_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("q", AiTensor4),
        ("k", AiTensor4),
        ("v", AiTensor4),
        ("out", AiTensor4),
        ("key_rows", ctypes.c_void_p),
        ("key_rows_stride_b", ctypes.c_int64),
        ("key_ok", ctypes.c_void_p),
        ("key_ok_stride_b", ctypes.c_int64),
        ("rope_cs16", ctypes.c_void_p),
        ("n_pos", ctypes.c_int32),
        ("status", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
    ]


class AiIndexArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32),
        ("seq_len", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("q", AiTensor4),
        ("k", AiTensor4),
        ("n_rows", ctypes.c_int32),
        ("rows", ctypes.c_void_p),
        ("targets", ctypes.c_void_p),
        ("n_keys", ctypes.c_int64),
        ("key_rows", ctypes.c_void_p),
        ("key_ok", ctypes.c_void_p),
        ("rope_cos", ctypes.c_void_p),
        ("rope_sin", ctypes.c_void_p),
        ("n_pos", ctypes.c_int32),
        ("logits", ctypes.c_void_p),
        ("lse", ctypes.c_void_p),
        ("loss", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
    ]


class AiIndexBwdArgs(ctypes.Structure):
    _fields_ = [
        ("fwd", AiIndexArgs),
        ("dloss", ctypes.c_void_p),
        ("dq", AiTensor4),
        ("dk", AiTensor4),
    ]


class AiPrepList(ctypes.Structure):
    _fields_ = [
        ("n_blocks", ctypes.c_int32),
        ("boundary", ctypes.c_void_p),
        ("n_query", ctypes.c_int64),
        ("query_pos", ctypes.c_void_p),
        ("n_keys", ctypes.c_int64),
        ("key_pos", ctypes.c_void_p),
        ("attn_mask", ctypes.c_void_p),
        ("abs_mask", ctypes.c_void_p),
    ]


class AiIndexRowsOut(ctypes.Structure):
    _fields_ = [
        ("rows", ctypes.c_void_p),
        ("key_rows", ctypes.c_void_p),
        ("key_ok", ctypes.c_void_p),
        ("rel_lo", ctypes.c_int64),
        ("rel_hi", ctypes.c_int64),
    ]


class AiPrepSizes(ctypes.Structure):
    _fields_ = [
        ("n_blocks", ctypes.c_int32),
        ("n_fwd_items", ctypes.c_int32),
        ("n_kv_items", ctypes.c_int32),
        ("n_kv_chunks", ctypes.c_int32),
        ("n_kv_reduce", ctypes.c_int32),
        ("n_chunk_cls", ctypes.c_int32),
        ("n_rot_classes", ctypes.c_int32),
        ("n_keys", ctypes.c_int64),
        ("p_min", ctypes.c_int64),
        ("p_max", ctypes.c_int64),
    ]


class AiPrepTables(ctypes.Structure):
    _fields_ = [
        ("blocks", ctypes.c_void_p),
        ("row_blocks", ctypes.c_void_p),
        ("row_cov", ctypes.c_void_p),
        ("key_info", ctypes.c_void_p),
        ("q_pos", ctypes.c_void_p),
        ("k_own", ctypes.c_void_p),
        ("fwd_items", ctypes.c_void_p),
        ("kv_items", ctypes.c_void_p),
        ("kv_chunks", ctypes.c_void_p),
        ("kv_reduce", ctypes.c_void_p),
        ("blk_cls", ctypes.c_void_p),
        ("chunk_cls", ctypes.c_void_p),
        ("rot_classes", ctypes.c_void_p),
        ("n_kv_partials", ctypes.c_int32),
        ("kv_cost_max", ctypes.c_int32),
        ("kv_cost_total", ctypes.c_int32),
        ("n_fwd_abs_items", ctypes.c_int32),
        ("n_fwd_short_items", ctypes.c_int32),
        ("n_fwd_abs_short_items", ctypes.c_int32),
        ("n_kv_abs_items", ctypes.c_int32),
        ("all_rows_owned", ctypes.c_int32),
        ("pairs_per_head", ctypes.c_int64),
    ]


_lock = threading.Lock()
_lib = None


def _bind(handle):
    P = ctypes.POINTER
    handle.ai_attn_abi_version.restype = ctypes.c_int
    handle.ai_attn_abi_version.argtypes = []
    for name in ("ai_attn_fwd_tile_rows", "ai_attn_kv_tile_rows"):
        fn = getattr(handle, name)
        fn.restype = ctypes.c_int
        fn.argtypes = [ctypes.c_int, ctypes.c_int]
    handle.ai_attn_fwd.restype = ctypes.c_int
    handle.ai_attn_fwd.argtypes = [P(AiAttnFwdArgs), ctypes.c_void_p]
    handle.ai_attn_fwd_workspace.restype = ctypes.c_int
    handle.ai_attn_fwd_workspace.argtypes = [P(AiAttnFwdArgs), P(ctypes.c_size_t)]
    handle.ai_attn_bwd_workspace.restype = ctypes.c_int
    handle.ai_attn_bwd_workspace.argtypes = [P(AiAttnBwdArgs), P(ctypes.c_size_t)]
    handle.ai_attn_bwd.restype = ctypes.c_int
    handle.ai_attn_bwd.argtypes = [P(AiAttnBwdArgs), ctypes.c_void_p]
    handle.ai_attn_bwd_noalloc.restype = ctypes.c_int
    handle.ai_attn_bwd_noalloc.argtypes = [P(AiAttnBwdArgs), ctypes.c_void_p]
    handle.ai_attn_decode_workspace.restype = ctypes.c_int
    handle.ai_attn_decode_workspace.argtypes = [P(AiAttnDecodeArgs), P(ctypes.c_size_t)]
    handle.ai_attn_decode.restype = ctypes.c_int
    handle.ai_attn_decode.argtypes = [P(AiAttnDecodeArgs), ctypes.c_void_p]
    handle.ai_attn_read_status.restype = ctypes.c_int
    handle.ai_attn_read_status.argtypes = [ctypes.c_void_p, ctypes.c_void_p, P(ctypes.c_int32)]
    handle.ai_attn_strerror.restype = ctypes.c_char_p
    handle.ai_attn_strerror.argtypes = [ctypes.c_int]
    handle.ai_attn_profile_enable.restype = ctypes.c_int
    handle.ai_attn_profile_enable.argtypes = [ctypes.c_int]
    handle.ai_attn_profile_read.restype = ctypes.c_int
    handle.ai_attn_profile_read.argtypes = [P(ctypes.c_float), P(ctypes.c_int32)]
    handle.ai_attn_selftest_wait.restype = ctypes.c_int
    handle.ai_attn_selftest_wait.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p]
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    handle.ai_attn_positions_from_ops_sizes.restype = ctypes.c_int
    handle.ai_attn_positions_from_ops_sizes.argtypes = [vp, i32, P(i32), P(i64), P(i64)]
    handle.ai_attn_positions_from_ops.restype = ctypes.c_int
    handle.ai_attn_positions_from_ops.argtypes = [vp, i32, vp, vp, vp, vp, vp, vp]
    handle.ai_attn_prep_sizes.restype = ctypes.c_int
    handle.ai_attn_prep_sizes.argtypes = [P(AiPrepList), i32, vp, i32, i32, i32, i32, P(AiPrepSizes)]
    handle.ai_attn_prep.restype = ctypes.c_int
    handle.ai_attn_prep.argtypes = [P(AiPrepList), i32, vp, i32, i32, i32, i32, P(AiPrepTables)]
    handle.ai_index_fwd.restype = ctypes.c_int
    handle.ai_index_fwd.argtypes = [P(AiIndexArgs), vp]
    handle.ai_index_bwd.restype = ctypes.c_int
    handle.ai_index_bwd.argtypes = [P(AiIndexBwdArgs), vp]
    handle.ai_index_rows_sizes.restype = ctypes.c_int
    handle.ai_index_rows_sizes.argtypes = [P(AiPrepList), vp, P(i32), P(i64), vp]
    handle.ai_index_rows.restype = ctypes.c_int
    handle.ai_index_rows.argtypes = [P(AiPrepList), vp, i64, P(AiIndexRowsOut)]
    return handle


def lib():
    """The loaded C library (loaded once).  Raises if it is missing."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"autoindexer_b200: CUDA library {LIB_PATH} is not built; "
                        "run `python -m autoindexer_b200.build` (nvcc, sm_100a)")
                handle = _bind(ctypes.CDLL(LIB_PATH))
                ver = handle.ai_attn_abi_version()
                if ver != ABI_VERSION:
                    raise RuntimeError(f"autoindexer_b200: library ABI {ver} != expected {ABI_VERSION}; rebuild it")
                _lib = handle
    return _lib


def strerror(code: int) -> str:
    return lib().ai_attn_strerror(int(code)).decode()


def check(code: int, what: str) -> None:
    if code != 0:
        raise RuntimeError(f"{what} failed ({code}): {strerror(code)}")
