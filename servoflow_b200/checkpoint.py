"""RDT-1B checkpoints: safetensors inspection, the reference converter's key
mapping, config.json and loading into an RDT1B model, through the C ABI
(sfb_safetensors_inspect, sfb_checkpoint_key, sfb_rdt1b_config_from_json,
sfb_rdt1b_load_checkpoint). Mirrors the reference's loader API:
SafeTensorsLoader::inspect (include/servoflow/loader/safetensors.h:53),
RDT1BConfig::from_json (src/models/rdt1b/config.cpp:10) and load_rdt1b
(src/models/rdt1b/rdt1b.cpp:379-394).
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

from . import _capi
from .rdt1b import RDT1B, RDT1BConfig, _declare, default_config

DTYPE_NAMES = {0: "F32", 1: "F16", 2: "BF16", 3: "I8", 4: "I4", 5: "I32", 6: "BOOL"}


class TensorInfo(ctypes.Structure):
    """Mirror of ``sfb_tensor_info`` (include/sfb200.h)."""

    _fields_ = [("name", ctypes.c_char * 256), ("dtype", ctypes.c_int32), ("ndim", ctypes.c_int32),
                ("shape", ctypes.c_int64 * 8), ("data_begin", ctypes.c_uint64),
                ("data_end", ctypes.c_uint64)]


def _lib():
    lib = _capi.lib()
    if not getattr(lib, "_ckpt_declared", False):
        c = ctypes
        lib.sfb_safetensors_inspect.argtypes = [c.c_char_p, c.POINTER(TensorInfo), c.c_int32,
                                                c.POINTER(c.c_int32), c.POINTER(c.c_uint64)]
        lib.sfb_safetensors_inspect.restype = c.c_int
        lib.sfb_checkpoint_key.argtypes = [c.c_char_p, c.c_char_p, c.c_int32]
        lib.sfb_checkpoint_key.restype = c.c_int
        lib._ckpt_declared = True
    _declare(lib)
    return lib


def inspect(path: str) -> list:
    """Tensor entries of a .safetensors file, sorted by name, without reading
    the data: dicts with name, dtype (safetensors spelling), shape and
    data_offsets (relative to the data section)."""
    lib = _lib()
    count, off = ctypes.c_int32(), ctypes.c_uint64()
    _capi.check(lib.sfb_safetensors_inspect(str(path).encode(), None, 0, ctypes.byref(count), ctypes.byref(off)),
                f"inspect {path}", detail=True)
    arr = (TensorInfo * max(1, count.value))()
    _capi.check(lib.sfb_safetensors_inspect(str(path).encode(), arr, count.value, ctypes.byref(count), None),
                f"inspect {path}", detail=True)
    return [dict(name=t.name.decode("utf-8", errors="replace"), dtype=DTYPE_NAMES[t.dtype],
                 shape=tuple(t.shape[:t.ndim]),
                 data_offsets=(t.data_begin, t.data_end)) for t in arr[:count.value]]


def checkpoint_key(name: str) -> Optional[str]:
    """The converter's ServoFlow name for an HF RDTRunner weight name, or None
    for an entry the converter drops."""
    buf = ctypes.create_string_buffer(1024)
    rc = _lib().sfb_checkpoint_key(name.encode(), buf, len(buf))
    if rc < 0:
        _capi.check(rc, f"checkpoint_key {name}")
    return buf.value.decode() if rc == 1 else None


def config_from_json(path: str, **overrides) -> RDT1BConfig:
    """RDT1BConfig from a checkpoint's config.json (converter or HF format)."""
    lib = _lib()
    cfg = RDT1BConfig()
    _capi.check(lib.sfb_rdt1b_config_from_json(str(path).encode(), ctypes.byref(cfg)), f"config {path}",
                detail=True)
    for k, v in overrides.items():
        setattr(cfg, k, v)
    return cfg


def load_rdt1b(checkpoint_dir: str, max_sessions: int = 1, **overrides) -> RDT1B:
    """A model from a checkpoint directory: config.json when present (else the
    defaults), then every *.safetensors shard; every parameter must be found."""
    cfg_path = os.path.join(checkpoint_dir, "config.json")
    if os.path.exists(cfg_path):
        cfg = config_from_json(cfg_path, max_sessions=max_sessions, **overrides)
    else:
        cfg = default_config(max_sessions=max_sessions, **overrides)
    model = RDT1B(cfg)
    try:
        model.load_checkpoint(checkpoint_dir)
    except Exception:
        model.close()
        raise
    return model
