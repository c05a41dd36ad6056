"""ctypes wrapper of the CPU oracle (oracle/libsfo_oracle.so) and of the
reference's own CUDA ops (oracle/_ref/libsfref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / --impl reference legs, never by the product path.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libsfo_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libsfref.so")
REFERENCE_TREE = "/root/reference"

_f = ctypes.c_float
_i = ctypes.c_int
_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
_lib = None
_ref = None


def build(force: bool = False) -> None:
    """make -C oracle (and the reference shim when the reference tree exists)."""
    if force or not os.path.exists(ORACLE_SO) or \
            os.path.getmtime(ORACLE_SO) < os.path.getmtime(os.path.join(HERE, "sfo_oracle.c")):
        subprocess.run(["make", "-C", HERE, "libsfo_oracle.so"], check=True, capture_output=True)
    if os.path.isdir(REFERENCE_TREE) and (force or not os.path.exists(REF_SO)):
        subprocess.run(["make", "-C", HERE, "ref", f"REF={REFERENCE_TREE}"], check=True,
                       capture_output=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        h = ctypes.CDLL(ORACLE_SO)
        h.sfo_attention.restype = None
        h.sfo_attention.argtypes = [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _i, _vp, _vp, _i]
        h.sfo_dequant_int8.restype = None
        h.sfo_dequant_int8.argtypes = [_vp, _vp, _i64, _vp, _i64, _i64, _i]
        h.sfo_round_f16.restype = _f
        h.sfo_round_f16.argtypes = [_f]
        h.sfo_round_bf16.restype = _f
        h.sfo_round_bf16.argtypes = [_f]
        h.sfo_num_threads.restype = _i
        h.sfo_w8a16_linear.restype = None
        h.sfo_w8a16_linear.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i]
        _lib = h
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_vp) if a is not None else None


def attention(q, k, v, scale=0.0, causal=False, kv_len=None, key_mask=None, nthreads=0):
    """Oracle attention on float32 numpy arrays [B, H, L, D] (K/V [B, Hkv, Lk, D])."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    B, H, Lq, D = q.shape
    Hkv, Lk = k.shape[1], k.shape[2]
    if D > 256:
        raise ValueError("oracle supports head_dim <= 256")
    out = np.empty_like(q)
    kl = None if kv_len is None else np.ascontiguousarray(kv_len, dtype=np.int32)
    km = None if key_mask is None else np.ascontiguousarray(key_mask, dtype=np.uint8)
    lib().sfo_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(out), B, H, Hkv, Lq, Lk, D, float(scale),
                        1 if causal else 0, _ptr(kl), _ptr(km), int(nthreads))
    return out


def dequant_int8(q, scale, round_mode=0):
    """round_mode 0: fp32; 1: fp16 (reference behaviour); 2: bf16."""
    q = np.ascontiguousarray(q, dtype=np.int8)
    s = np.ascontiguousarray(scale, dtype=np.float32).reshape(-1)
    rows = q.shape[0]
    cols = q.size // rows
    out = np.empty(q.shape, dtype=np.float32)
    lib().sfo_dequant_int8(_ptr(q), _ptr(s), s.size, _ptr(out), rows, cols, int(round_mode))
    return out


def w8a16_linear(x, q, scale, bias=None, residual=None, act=0, nthreads=0):
    """Oracle int8-weight linear layer: float32 x [M, K], int8 q [N, K]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.ascontiguousarray(q, dtype=np.int8)
    s = np.ascontiguousarray(scale, dtype=np.float32)
    M, K = x.shape
    N = q.shape[0]
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    r = None if residual is None else np.ascontiguousarray(residual, dtype=np.float32)
    y = np.empty((M, N), np.float32)
    lib().sfo_w8a16_linear(_ptr(x), _ptr(q), _ptr(s), _ptr(b), _ptr(r), _ptr(y), M, N, K, int(act),
                           int(nthreads))
    return y


def num_threads() -> int:
    return lib().sfo_num_threads()


def ref_lib():
    """The reference's own attention/dequant CUDA code (None if not built)."""
    global _ref
    if _ref is None and os.path.exists(REF_SO):
        h = ctypes.CDLL(REF_SO)
        h.sfref_attention.restype = _i
        h.sfref_attention.argtypes = [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _i, _vp]
        h.sfref_dequantize.restype = _i
        h.sfref_dequantize.argtypes = [_vp, _vp, ctypes.c_long, _vp, ctypes.c_long, ctypes.c_long, _vp]
        _ref = h
    return _ref
