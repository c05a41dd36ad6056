"""ctypes wrapper of the CPU oracle (oracle/libsfo_oracle.so) and of the
reference's own CUDA ops (oracle/_ref/libsfref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / --impl reference legs, never by the product path.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libsfo_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libsfref.so")
REF_FA2_SO = os.path.join(HERE, "_ref", "libsfref_fa2.so")
BINDING_SO = os.path.join(HERE, "_ref", "libsfb_binding_test.so")
# The reference project's root, where its sources can be compiled (set by the
# caller; no default). Without it the prebuilt oracle/_ref libraries, if any,
# are used as they are.
REF_ENV = "SFB_REFERENCE_TREE"

_f = ctypes.c_float
_i = ctypes.c_int
_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
_lib = None
_ref = None
_ref_fa2 = None


def build(force: bool = False) -> None:
    """make -C oracle; with $SFB_REFERENCE_TREE set, also the reference's own
    CUDA attention/dequant (libsfref.so) and FlashAttention-2 (libsfref_fa2.so,
    built only when missing: it takes minutes)."""
    if force or not os.path.exists(ORACLE_SO) or \
            os.path.getmtime(ORACLE_SO) < os.path.getmtime(os.path.join(HERE, "sfo_oracle.c")):
        subprocess.run(["make", "-C", HERE, "libsfo_oracle.so"], check=True, capture_output=True)
    tree = os.environ.get(REF_ENV, "")
    if not tree:
        if not os.path.exists(REF_SO):
            print(f"oracle: {REF_ENV} unset, the reference's own kernels are not built", file=sys.stderr)
        return
    if not os.path.isdir(os.path.join(tree, "src")):
        raise FileNotFoundError(f"{REF_ENV}={tree} is not the reference project's root")
    if force or not os.path.exists(REF_SO):
        subprocess.run(["make", "-C", HERE, "ref", f"REF={tree}"], check=True, capture_output=True)
    if not os.path.exists(REF_FA2_SO):
        subprocess.run(["make", "-C", HERE, "ref-fa2", f"REF={tree}"], check=True, capture_output=True)


def build_binding(force: bool = False) -> None:
    """With $SFB_REFERENCE_TREE set: the servoflow-side binding
    (integration/sfb_servoflow.hpp) compiled against the reference's headers,
    linked to libsfb200.so (build that first). Rebuilt when its sources change."""
    tree = os.environ.get(REF_ENV, "")
    if not tree:
        return
    srcs = [os.path.join(HERE, "..", "tests", "binding", "binding_test.cpp"),
            os.path.join(HERE, "..", "integration", "sfb_servoflow.hpp"),
            os.path.join(HERE, "..", "include", "sfb200.h")]
    if force or not os.path.exists(BINDING_SO) or \
            os.path.getmtime(BINDING_SO) < max(os.path.getmtime(f) for f in srcs):
        if os.path.exists(BINDING_SO):
            os.remove(BINDING_SO)
        subprocess.run(["make", "-C", HERE, "binding", f"REF={tree}"], check=True, capture_output=True)


def binding_lib():
    """The compiled servoflow-side binding (None if not built)."""
    if not os.path.exists(BINDING_SO):
        return None
    h = ctypes.CDLL(BINDING_SO)
    h.sfbind_last_message.restype = ctypes.c_char_p
    h.sfbind_attention.restype = _i
    h.sfbind_attention.argtypes = [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _i, _i, _vp,
                                   _f, _i, _vp]
    h.sfbind_dequantize.restype = _i
    h.sfbind_dequantize.argtypes = [_vp, _vp, _i, ctypes.c_long, _vp, _i, ctypes.c_long, ctypes.c_long, _vp]
    return h


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        h = ctypes.CDLL(ORACLE_SO)
        h.sfo_attention.restype = None
        h.sfo_attention.argtypes = [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _i, _vp, _vp, _i, _vp]
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


def attention(q, k, v, scale=0.0, causal=False, kv_len=None, key_mask=None, nthreads=0,
              attn_mask=None):
    """Oracle attention on float32 numpy arrays [B, H, L, D] (K/V [B, Hkv, Lk, D]).
    attn_mask: an additive float mask broadcastable to [B, 1, Lq, Lk]."""
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
    am = None
    if attn_mask is not None:
        am = np.ascontiguousarray(np.broadcast_to(np.asarray(attn_mask, dtype=np.float32),
                                                  (B, 1, Lq, Lk)).reshape(B, Lq, Lk))
    lib().sfo_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(out), B, H, Hkv, Lq, Lk, D, float(scale),
                        1 if causal else 0, _ptr(kl), _ptr(km), int(nthreads), _ptr(am))
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


def ref_fa2_lib():
    """The reference's FlashAttention-2 forward, hdim 64 (None if not built)."""
    global _ref_fa2
    if _ref_fa2 is None and os.path.exists(REF_FA2_SO):
        try:
            h = ctypes.CDLL(REF_FA2_SO)
        except OSError as e:                      # a stale or partial build
            print(f"oracle: cannot load {REF_FA2_SO}: {e}", file=sys.stderr)
            return None
        h.sfref_fa2_workspace_bytes.restype = ctypes.c_long
        h.sfref_fa2_workspace_bytes.argtypes = [_i, _i, _i]
        h.sfref_fa2_attention.restype = _i
        h.sfref_fa2_attention.argtypes = [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _i, _vp,
                                          ctypes.c_long, _vp]
        _ref_fa2 = h
    return _ref_fa2
