"""ctypes binding of libexl3b.so, the sm_100a C-ABI library (declared in include/exl3b.h).

Loading fails loudly: there is no CPU or eager fallback for any op of this package.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("EXL3B_LIB", os.path.join(_HERE, "libexl3b.so"))

EXL3B_OK = 0
EXL3B_DECLINED = 1
EXL3B_BAD_ARG = 2
EXL3B_WORKSPACE = 3
EXL3B_TOO_LARGE = 4

c_u16p = ctypes.c_void_p
c_vp = ctypes.c_void_p
i32, i64, f32, sz = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t

EXL3B_MAX_TP = 8
EXL3B_IPC_HANDLE_BYTES = 72


class KvLayout(ctypes.Structure):
    """exl3b_kv_layout of include/exl3b.h: cache strides in bytes, scale strides in floats."""
    _fields_ = [("cache_block", ctypes.c_int64), ("cache_slot", ctypes.c_int64), ("cache_head", ctypes.c_int64),
                ("scale_block", ctypes.c_int64), ("scale_slot", ctypes.c_int64), ("scale_head", ctypes.c_int64)]


class TpComm(ctypes.Structure):
    """exl3b_tp_comm of include/exl3b.h."""
    _fields_ = [("tp_size", ctypes.c_int), ("tp_rank", ctypes.c_int), ("max_blocks", ctypes.c_int),
                ("max_rows", ctypes.c_int), ("buffers", ctypes.c_void_p * EXL3B_MAX_TP)]


# name -> (restype, argtypes); every symbol include/exl3b.h declares
SIGNATURES = {
    "exl3b_version": (i32, []),
    "exl3b_status_string": (ctypes.c_char_p, [i32]),
    "exl3b_decode_states": (i32, [c_vp, c_vp, i64, i32, c_vp]),
    "exl3b_dequant": (i32, [c_vp, i32, i32, i32, i32, i32, i32, c_vp, i64, c_vp]),
    "exl3b_had128": (i32, [c_vp, i64, c_vp, i64, i64, i64, c_vp, c_vp, f32, c_vp]),
    "exl3b_linear_workspace_bytes": (sz, [i32, i32, i32, i64]),
    "exl3b_linear": (i32, [c_vp, i32, i32, c_vp, i32, i32, i32, c_vp, c_vp, c_vp, i64, c_vp, sz, c_vp]),
    "exl3b_linear_grouped": (i32, [c_vp, i32, i32, i32, ctypes.POINTER(c_vp), ctypes.POINTER(i32), i32, i32,
                                   ctypes.POINTER(c_vp), ctypes.POINTER(c_vp), ctypes.POINTER(c_vp), i64, c_vp, sz,
                                   c_vp]),
    "exl3b_linear_grouped_rmsnorm": (i32, [c_vp, i32, i32, i32, ctypes.POINTER(c_vp), ctypes.POINTER(i32), i32, i32,
                                           c_vp, f32, ctypes.POINTER(c_vp), ctypes.POINTER(c_vp),
                                           ctypes.POINTER(c_vp), i64, c_vp, sz, c_vp]),
    "exl3b_linear_workspace_error": (i32, [c_vp, ctypes.POINTER(i32), c_vp]),
    "exl3b_gemm_workspace_bytes": (sz, [i32, i32]),
    "exl3b_gemm": (i32, [c_vp, i32, i32, c_vp, i32, i32, i32, c_vp, c_vp, c_vp, i64, c_vp, sz, c_vp]),
    "exl3b_decode_ceiling": (i32, [i32, i32, c_vp, i32, c_vp, c_vp, c_vp]),
    "exl3b_linear_supported": (i32, [i32, i32, i32, i32, i32]),
    "exl3b_fp8_embedding": (i32, [c_vp, i64, i64, c_vp, i32, i64, c_vp, c_vp]),
    "exl3b_linear_noalloc": (i32, [c_vp, i32, i32, c_vp, i32, i32, i32, c_vp, c_vp, c_vp, i64, c_vp]),
    "exl3b_linear_noalloc_error": (i32, [ctypes.POINTER(i32), c_vp]),
    "exl3b_kv_int8_write": (i32, [c_vp, c_vp, i32, i64, i32, i32, i64, i64, i64, i64, c_vp, c_vp, c_vp, c_vp, c_vp,
                                  i32, c_vp, c_vp]),
    "exl3b_kv_int8_write_rope": (i32, [c_vp, i64, c_vp, i64, i64, i32, i32, c_vp, c_vp, i64, c_vp, c_vp, c_vp, c_vp,
                                       c_vp, i32, c_vp, c_vp]),
    "exl3b_kv_int4_write": (i32, [c_vp, c_vp, i32, i64, i32, i32, i64, i64, i64, i64, c_vp, c_vp, c_vp, c_vp, c_vp,
                                  i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, i32, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "exl3b_tp_comm_bytes": (sz, [i32, i32, i32]),
    "exl3b_ipc_get_handle": (i32, [c_vp, c_vp]),
    "exl3b_ipc_open_handle": (i32, [c_vp, ctypes.POINTER(c_vp)]),
    "exl3b_ipc_close": (i32, [c_vp]),
    "exl3b_linear_tp": (i32, [c_vp, i32, i32, c_vp, i32, i32, i32, c_vp, c_vp, c_vp, i64, c_vp, sz,
                              ctypes.POINTER(TpComm), c_vp]),
    "exl3b_kv_attn_workspace_bytes": (sz, [i32, i32, i32, i32, i32]),
    "exl3b_kv_int8_gather": (i32, [c_vp, c_vp, i32, i32, i32, c_vp, i64, c_vp, c_vp, c_vp]),
    "exl3b_kv_int4_gather": (i32, [c_vp, c_vp, i32, i32, i32, c_vp, i64, i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "exl3b_kv_int8_attn": (i32, [c_vp, c_vp, i32, i32, i32, i32, c_vp, c_vp, c_vp, c_vp, i32, c_vp, i64, c_vp, c_vp,
                                 i32, i32, i32, f32, c_vp, sz, c_vp, c_vp]),
    "exl3b_kv_int4_attn": (i32, [c_vp, c_vp, i32, i32, i32, i32, c_vp, c_vp, c_vp, c_vp, i32, c_vp, i64, c_vp, c_vp,
                                 i32, i32, i32, f32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, sz, c_vp, c_vp]),
    "exl3b_rmsnorm": (i32, [c_vp, i64, c_vp, i64, c_vp, c_vp, i64, i32, i32, f32, c_vp]),
    "exl3b_rope_neox": (i32, [c_vp, i64, c_vp, i64, i32, i32, i32, c_vp, c_vp, i64, c_vp]),
    "exl3b_silu_mul": (i32, [c_vp, i64, c_vp, i64, i32, i32, c_vp]),
}

_lib = None
_lock = threading.Lock()


class Exl3bError(RuntimeError):
    """A call into libexl3b returned a non-zero status."""

    def __init__(self, fn: str, status: int, text: str):
        super().__init__(f"{fn}: status {status}: {text}")
        self.status = status


def lib() -> ctypes.CDLL:
    """The loaded library (loaded once).  Raises ImportError when it is missing."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"libexl3b.so not found at {LIB_PATH}; build it with "
                        "`python qwen38-27b-exl3-rdna4_b200/build.py` (nvcc, sm_100a). "
                        "exl3rocm has no fallback path.")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def check(fn: str, status: int) -> None:
    if status != EXL3B_OK:
        text = lib().exl3b_status_string(status).decode()
        raise Exl3bError(fn, status, text)


def call(fn: str, *args) -> None:
    check(fn, getattr(lib(), fn)(*args))
