"""ctypes binding of ``libtfa_sm100.so`` (the C ABI in ``include/tfa.h``).

Loading is explicit and loud: if the library is missing or cannot be loaded, every
caller gets an ``ImportError``/``RuntimeError``; there is no fallback implementation.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "libtfa_sm100.so"

TFA_OK = 0
STATUS_NAMES = {
    0: "TFA_OK",
    -1: "TFA_ERR_NULL_POINTER",
    -2: "TFA_ERR_HEAD_DIM",
    -3: "TFA_ERR_GQA",
    -4: "TFA_ERR_BLOCK_SIZE",
    -5: "TFA_ERR_LAYOUT",
    -6: "TFA_ERR_SHAPE",
    -7: "TFA_ERR_WORKSPACE",
    -8: "TFA_ERR_TENSOR_MAP",
    -9: "TFA_ERR_CUDA",
    -10: "TFA_ERR_DEVICE",
    -11: "TFA_ERR_KERNEL",
    -12: "TFA_ERR_STATIC_WORKSPACE_LIMIT",
}

# Every symbol declared in include/tfa.h.
EXPORTED_SYMBOLS = (
    "tfa_plan",
    "tfa_workspace_size",
    "tfa_fwd",
    "tfa_fwd_timed",
    "tfa_fwd_static_workspace",
    "tfa_read_static_workspace_error",
    "tfa_read_device_error",
    "tfa_device_sm_count",
    "tfa_status_string",
    "tfa_gather_kv",
    "tfa_kv_cache_update",
)

_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_vp = ctypes.c_void_p


class TfaFwdParams(ctypes.Structure):
    """Mirror of ``struct tfa_fwd_params``."""

    _fields_ = [
        ("q", _vp),
        ("q_stride", _i64 * 3),
        ("k", _vp),
        ("k_stride", _i64 * 4),
        ("v", _vp),
        ("v_stride", _i64 * 4),
        ("out", _vp),
        ("out_stride", _i64 * 3),
        ("softmax_lse", _vp),
        ("cu_seqlens_q", _vp),
        ("seqused_k", _vp),
        ("block_table", _vp),
        ("block_table_stride0", _i64),
        ("batch", _i64),
        ("total_q", _i64),
        ("num_q_heads", _i64),
        ("num_kv_heads", _i64),
        ("head_dim", _i64),
        ("block_size", _i64),
        ("num_blocks", _i64),
        ("max_seqlen_q", _i64),
        ("max_seqlen_k", _i64),
        ("causal", _i32),
        ("window_left", _i32),
        ("window_right", _i32),
        ("softmax_scale", ctypes.c_float),
        ("num_splits", _i32),
    ]


class TfaPlanInfo(ctypes.Structure):
    """Mirror of ``struct tfa_plan_info``."""

    _fields_ = [
        ("kernel", _i32),
        ("rows_per_tile", _i32),
        ("q_tiles", _i32),
        ("max_splits", _i32),
        ("split_cap", _i32),
        ("num_items", _i32),
        ("grid", _i32),
        ("combine", _i32),
        ("workspace_bytes", ctypes.c_uint64),
        ("item_list", _i32),
        ("pages", _i32),
    ]


_lock = threading.Lock()
_lib = None


def lib_path() -> Path:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load (once) and return the library, with argument types declared."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not _LIB_PATH.exists():
            raise ImportError(
                f"{_LIB_PATH.name} is not built; run `python -m toy_flash_attn._build` "
                "(or __graft_entry__.build()) first"
            )
        lib = ctypes.CDLL(str(_LIB_PATH))
        P = ctypes.POINTER
        lib.tfa_plan.argtypes = [P(TfaFwdParams), ctypes.c_int, P(TfaPlanInfo)]
        lib.tfa_plan.restype = ctypes.c_int
        lib.tfa_workspace_size.argtypes = [P(TfaFwdParams), ctypes.c_int]
        lib.tfa_workspace_size.restype = ctypes.c_size_t
        lib.tfa_fwd.argtypes = [P(TfaFwdParams), _vp, ctypes.c_size_t, _vp]
        lib.tfa_fwd.restype = ctypes.c_int
        lib.tfa_fwd_timed.argtypes = [P(TfaFwdParams), _vp, ctypes.c_size_t, _vp, _vp, _vp]
        lib.tfa_fwd_timed.restype = ctypes.c_int
        lib.tfa_fwd_static_workspace.argtypes = [P(TfaFwdParams), _vp]
        lib.tfa_fwd_static_workspace.restype = ctypes.c_int
        lib.tfa_read_static_workspace_error.argtypes = [_vp, P(ctypes.c_int)]
        lib.tfa_read_static_workspace_error.restype = ctypes.c_int
        lib.tfa_read_device_error.argtypes = [_vp, _vp, P(ctypes.c_int)]
        lib.tfa_read_device_error.restype = ctypes.c_int
        lib.tfa_device_sm_count.argtypes = [ctypes.c_int]
        lib.tfa_device_sm_count.restype = ctypes.c_int
        lib.tfa_status_string.argtypes = [ctypes.c_int]
        lib.tfa_status_string.restype = ctypes.c_char_p
        lib.tfa_gather_kv.argtypes = [P(TfaFwdParams), _vp, _vp, _vp, _vp, _vp]
        lib.tfa_gather_kv.restype = ctypes.c_int
        lib.tfa_kv_cache_update.argtypes = [
            _vp, P(_i64), _vp, P(_i64), _vp, P(_i64), _vp, P(_i64), _vp,
            _i64, _i64, _i64, _i64, _i64, _vp, _vp,
        ]
        lib.tfa_kv_cache_update.restype = ctypes.c_int
        _lib = lib
        return lib


def check(status: int, what: str) -> None:
    if status != TFA_OK:
        name = STATUS_NAMES.get(status, str(status))
        msg = load().tfa_status_string(status).decode()
        raise RuntimeError(f"{what} failed: {name} ({msg})")
