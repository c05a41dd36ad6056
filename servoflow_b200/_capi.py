"""ctypes binding of libsfb200.so (the C ABI declared in include/sfb200.h).

The shared library is built in-tree (servoflow_b200/_lib/libsfb200.so) by
``servoflow_b200.build.build_library()``. Loading fails loudly when it is
missing: there is no Python or CPU fallback for any op.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libsfb200.so")

SFB_OK = 0
SFB_ERR_INVALID = -1
SFB_ERR_DTYPE = -2
SFB_ERR_SHAPE = -3
SFB_ERR_ALIGN = -4
SFB_ERR_WORKSPACE = -5
SFB_ERR_LAUNCH = -6
SFB_ERR_UNSUPPORTED = -7
SFB_ERR_CUDA = -8
SFB_ERR_DEVICE_TIMEOUT = -9
SFB_ERR_RANGE = -10
SFB_ERR_IO = -11

SFB_F32, SFB_F16, SFB_BF16, SFB_I8, SFB_I32, SFB_BOOL = 0, 1, 2, 3, 5, 6


class AttnArgs(ctypes.Structure):
    """Mirror of ``sfb_attn_args`` (include/sfb200.h)."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("q_stride", ctypes.c_int64 * 3),
        ("k_stride", ctypes.c_int64 * 3),
        ("v_stride", ctypes.c_int64 * 3),
        ("out_stride", ctypes.c_int64 * 3),
        ("batch", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("heads_kv", ctypes.c_int32),
        ("seq_q", ctypes.c_int32),
        ("seq_k", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("is_causal", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("kv_len", ctypes.c_void_p),
        ("key_mask", ctypes.c_void_p),
        ("key_mask_stride_b", ctypes.c_int64),
        ("num_splits", ctypes.c_int32),
        ("v_dtype", ctypes.c_int32),
        ("attn_mask_dtype", ctypes.c_int32),
        ("attn_mask", ctypes.c_void_p),
        ("attn_mask_stride", ctypes.c_int64 * 2),
    ]


class SfbError(RuntimeError):
    """A non-zero status returned through the C ABI."""

    def __init__(self, status: int, what: str, detail: bool = False):
        self.status = status
        extra = ""
        if detail or status in (SFB_ERR_LAUNCH, SFB_ERR_CUDA, SFB_ERR_IO):
            extra = " — " + lib().sfb_last_error().decode("utf-8", errors="replace")   # may quote file bytes
        super().__init__(f"{what}: {status_string(status)} (status {status}){extra}")


_lib = None
_lock = threading.Lock()


def _declare(lib: ctypes.CDLL) -> None:
    c = ctypes
    lib.sfb_status_string.restype = c.c_char_p
    lib.sfb_status_string.argtypes = [c.c_int]
    lib.sfb_last_error.restype = c.c_char_p
    lib.sfb_last_error.argtypes = []
    lib.sfb_version.restype = c.c_char_p
    lib.sfb_version.argtypes = []
    lib.sfb_device_error.restype = c.c_int
    lib.sfb_device_error.argtypes = [c.POINTER(c.c_int), c.c_int]
    lib.sfb_attention_fwd.restype = c.c_int
    lib.sfb_attention_fwd.argtypes = [c.POINTER(AttnArgs), c.c_void_p]
    lib.sfb_attention_bhsd.restype = c.c_int
    lib.sfb_attention_bhsd.argtypes = [c.c_void_p, c.c_void_p, c.c_void_p, c.c_void_p,
                                       c.c_int32, c.c_int32, c.c_int32, c.c_int32, c.c_int32,
                                       c.c_int32, c.c_int32, c.c_void_p, c.c_float, c.c_int32,
                                       c.c_void_p]
    lib.sfb_w8a16_linear.restype = c.c_int
    lib.sfb_w8a16_linear.argtypes = [c.c_void_p, c.c_int64, c.c_void_p, c.c_void_p, c.c_void_p,
                                     c.c_void_p, c.c_int64, c.c_void_p, c.c_int64, c.c_int32,
                                     c.c_int32, c.c_int32, c.c_int32, c.c_int32, c.c_int32,
                                     c.c_void_p]
    lib.sfb_w8a16_mlp_workspace_bytes.restype = c.c_size_t
    lib.sfb_w8a16_mlp_workspace_bytes.argtypes = [c.c_int32, c.c_int32]
    lib.sfb_w8a16_mlp.restype = c.c_int
    lib.sfb_w8a16_mlp.argtypes = [c.c_void_p, c.c_int64, c.c_void_p, c.c_void_p, c.c_void_p,
                                  c.c_void_p, c.c_void_p, c.c_void_p, c.c_void_p, c.c_int64,
                                  c.c_void_p, c.c_int64, c.c_int32, c.c_int32, c.c_int32, c.c_int32,
                                  c.c_int32, c.c_int32, c.c_void_p, c.c_size_t, c.c_void_p]
    lib.sfb_dequantize_int8.restype = c.c_int
    lib.sfb_dequantize_int8.argtypes = [c.c_void_p, c.c_void_p, c.c_int32, c.c_int64, c.c_void_p,
                                        c.c_int32, c.c_int64, c.c_int64, c.c_void_p]


def lib() -> ctypes.CDLL:
    """Loads libsfb200.so once; raises ImportError if it was not built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"{LIB_PATH} is missing: build it with "
                        "`python -c 'import servoflow_b200.build as b; b.build_library()'`")
                h = ctypes.CDLL(LIB_PATH)
                _declare(h)
                _lib = h
    return _lib


def status_string(status: int) -> str:
    return lib().sfb_status_string(int(status)).decode()


def check(status: int, what: str, detail: bool = False) -> None:
    """Raises SfbError for a non-zero status; detail=True appends the library's
    message for the call (calls that record one on every failure)."""
    if status != SFB_OK:
        raise SfbError(status, what, detail)
