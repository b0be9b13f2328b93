"""ctypes binding of the C ABI declared in include/apex_attn.h.

The shared library is built in-tree next to this file (``libapex_attn.so``) by
``apex-tune-results_b200/build.py``. There is no fallback: if the library is missing the
import of :mod:`apex_attn` still works, but every call raises ``RuntimeError`` naming
the missing file, so a CUDA-less or stale checkout fails loudly instead of silently
computing attention some other way.
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_NAME = "libapex_attn.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

# Status codes, mirrored from include/apex_attn.h.
OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_UNSUPPORTED_HEAD_DIM = -2
ERR_UNSUPPORTED_DTYPE = -3
ERR_BAD_LAYOUT = -4
ERR_BAD_SCALE = -5
ERR_NO_DEVICE = -6
ERR_UNSUPPORTED_ARCH = -7
ERR_TENSOR_MAP = -8
ERR_LAUNCH = -9
ERR_DEVICE_TIMEOUT = -10
ERR_TOO_LARGE = -11
ERR_CUDA = -12

DTYPE_BF16 = 0
DTYPE_FP16 = 1

class FwdArgs(ctypes.Structure):
    """Mirror of apex_attn_fwd_args (include/apex_attn.h)."""
    _fields_ = [("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
                ("o", ctypes.c_void_p), ("lse", ctypes.c_void_p), ("batch", ctypes.c_int),
                ("heads_q", ctypes.c_int), ("heads_kv", ctypes.c_int), ("seqlen", ctypes.c_int),
                ("head_dim", ctypes.c_int), ("dtype", ctypes.c_int), ("causal", ctypes.c_int),
                ("window_left", ctypes.c_int), ("sm_scale", ctypes.c_float),
                ("strides", ctypes.c_longlong * 12)]


class BwdArgs(ctypes.Structure):
    """Mirror of apex_attn_bwd_args (include/apex_attn.h)."""
    _fields_ = [("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
                ("o", ctypes.c_void_p), ("dout", ctypes.c_void_p), ("lse", ctypes.c_void_p),
                ("dq", ctypes.c_void_p), ("dk", ctypes.c_void_p), ("dv", ctypes.c_void_p),
                ("batch", ctypes.c_int), ("heads_q", ctypes.c_int), ("heads_kv", ctypes.c_int),
                ("seqlen", ctypes.c_int), ("head_dim", ctypes.c_int), ("dtype", ctypes.c_int),
                ("causal", ctypes.c_int), ("window_left", ctypes.c_int),
                ("sm_scale", ctypes.c_float), ("strides", ctypes.c_longlong * 24)]


class VarlenArgs(ctypes.Structure):
    """Mirror of apex_attn_varlen_args (include/apex_attn.h)."""
    _fields_ = [("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
                ("o", ctypes.c_void_p), ("lse", ctypes.c_void_p), ("cu_seqlens", ctypes.c_void_p),
                ("batch", ctypes.c_int), ("heads_q", ctypes.c_int), ("heads_kv", ctypes.c_int),
                ("total", ctypes.c_int), ("max_seqlen", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("dtype", ctypes.c_int), ("causal", ctypes.c_int), ("window_left", ctypes.c_int),
                ("sm_scale", ctypes.c_float), ("strides", ctypes.c_longlong * 8)]


class BwdVarlenArgs(ctypes.Structure):
    """Mirror of apex_attn_bwd_varlen_args (include/apex_attn.h)."""
    _fields_ = [("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
                ("o", ctypes.c_void_p), ("dout", ctypes.c_void_p), ("lse", ctypes.c_void_p),
                ("dq", ctypes.c_void_p), ("dk", ctypes.c_void_p), ("dv", ctypes.c_void_p),
                ("cu_seqlens", ctypes.c_void_p), ("batch", ctypes.c_int), ("heads_q", ctypes.c_int),
                ("heads_kv", ctypes.c_int), ("total", ctypes.c_int), ("max_seqlen", ctypes.c_int),
                ("head_dim", ctypes.c_int), ("dtype", ctypes.c_int), ("causal", ctypes.c_int),
                ("window_left", ctypes.c_int), ("sm_scale", ctypes.c_float),
                ("strides", ctypes.c_longlong * 16)]


# Every symbol the header declares: (name, restype, argtypes).
_c_ll_p = ctypes.POINTER(ctypes.c_longlong)
SYMBOLS = {
    "apex_attn_fwd": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
         ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
         ctypes.c_float, _c_ll_p, ctypes.c_void_p],
    ),
    "apex_attn_fwd_ex": (ctypes.c_int, [ctypes.POINTER(FwdArgs), ctypes.c_void_p]),
    "apex_attn_fwd_varlen": (ctypes.c_int, [ctypes.POINTER(VarlenArgs), ctypes.c_void_p]),
    "apex_attn_fwd_noalloc": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
         ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
         ctypes.c_float, _c_ll_p, ctypes.c_void_p],
    ),
    "apex_attn_bwd_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "apex_attn_bwd": (ctypes.c_int, [ctypes.POINTER(BwdArgs), ctypes.c_void_p, ctypes.c_size_t,
                                     ctypes.c_void_p]),
    "apex_attn_bwd_varlen": (ctypes.c_int, [ctypes.POINTER(BwdVarlenArgs), ctypes.c_void_p,
                                            ctypes.c_size_t, ctypes.c_void_p]),
    "apex_attn_bwd_workspace_bytes_mode": (ctypes.c_size_t, [ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                             ctypes.c_int, ctypes.c_int]),
    "apex_attn_bwd_mode": (ctypes.c_int, [ctypes.POINTER(BwdArgs), ctypes.c_int, ctypes.c_void_p,
                                          ctypes.c_size_t, ctypes.c_void_p]),
    "apex_attn_bwd_varlen_mode": (ctypes.c_int, [ctypes.POINTER(BwdVarlenArgs), ctypes.c_int,
                                                 ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "apex_attn_num_sms_hint": (ctypes.c_int, [ctypes.c_int]),
    "apex_attn_set_forward_kernel": (ctypes.c_int, [ctypes.c_int]),
    "apex_attn_forward_kernel_for": (ctypes.c_int, [ctypes.c_int] * 7),
    "apex_attn_device_status": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    "apex_attn_noalloc_status": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    "apex_attn_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_int, ctypes.c_void_p]),
    "apex_attn_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "apex_attn_version": (ctypes.c_int, []),
    "apex_attn_supports_head_dim": (ctypes.c_int, [ctypes.c_int]),
}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Loads (once) and returns the library with argtypes configured."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"apex_attn native library not found at {LIB_PATH}; build it with "
                    "`python apex-tune-results_b200/build.py` (there is no non-CUDA fallback)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SYMBOLS.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def strerror(code: int) -> str:
    return load().apex_attn_strerror(int(code)).decode()


def check(code: int, what: str = "apex_attn") -> None:
    if code != OK:
        raise RuntimeError(f"{what} failed: {strerror(code)} (status {code})")
