"""Python handle on the Octo policy runtime of libsfb200 (C ABI sfb_octo_*),
mirroring the reference's OctoModel (include/servoflow/models/octo/octo.h:
87-132): encode() for encode_condition, denoise_step(), and sample() for the
flow-matching sampler. torch tensors supply device memory and streams only."""
from __future__ import annotations

import ctypes

import torch

from . import _capi
from .rdt1b import _copy_d2d, _sh


class OctoConfig(ctypes.Structure):
    """Mirror of ``sfb_octo_config`` (include/sfb200.h)."""

    _fields_ = [(n, ctypes.c_int32) for n in (
        "num_layers", "hidden", "heads", "head_dim", "intermediate", "action_dim", "action_horizon",
        "head_hidden", "seq_len", "max_sessions", "num_steps", "readout_token")] + [
        ("weight_std", ctypes.c_float)]


_FUNCS = ("default_config", "create", "destroy", "encode", "set_condition", "denoise_step", "sample",
          "timesteps", "param", "graph_kernels")


def _declare(lib):
    c = ctypes
    if getattr(lib, "_octo_declared", False):
        return
    lib.sfb_octo_default_config.argtypes = [c.POINTER(OctoConfig)]
    lib.sfb_octo_create.argtypes = [c.POINTER(OctoConfig), c.c_uint64, c.POINTER(c.c_void_p)]
    lib.sfb_octo_destroy.argtypes = [c.c_void_p]
    lib.sfb_octo_encode.argtypes = [c.c_void_p, c.c_int32, c.c_void_p, c.c_void_p, c.c_void_p]
    lib.sfb_octo_set_condition.argtypes = [c.c_void_p, c.c_int32, c.c_void_p, c.c_void_p]
    lib.sfb_octo_denoise_step.argtypes = [c.c_void_p, c.c_int32, c.c_void_p, c.c_float, c.c_void_p,
                                          c.c_void_p]
    lib.sfb_octo_sample.argtypes = [c.c_void_p, c.c_int32, c.c_void_p, c.c_void_p, c.c_int32, c.c_void_p]
    lib.sfb_octo_timesteps.argtypes = [c.c_void_p, c.c_void_p, c.c_int32]
    lib.sfb_octo_param.argtypes = [c.c_void_p, c.c_char_p, c.POINTER(c.c_void_p), c.POINTER(c.c_int64),
                                   c.POINTER(c.c_int32)]
    lib.sfb_octo_graph_kernels.argtypes = [c.c_void_p, c.c_int32, c.POINTER(c.c_int64)]
    for f in _FUNCS:
        getattr(lib, "sfb_octo_" + f).restype = c.c_int
    lib._octo_declared = True


def default_config(**overrides) -> OctoConfig:
    """OctoConfig defaults (Octo-Small: hidden 384, 12 layers, 6 heads)."""
    lib = _capi.lib()
    _declare(lib)
    cfg = OctoConfig()
    _capi.check(lib.sfb_octo_default_config(ctypes.byref(cfg)), "octo default_config")
    for k, v in overrides.items():
        setattr(cfg, k, v)
    return cfg


class Octo:
    """Model handle: encode() once per observation, sample() per action chunk."""

    _DT = {_capi.SFB_BF16: torch.bfloat16, _capi.SFB_F32: torch.float32, _capi.SFB_I8: torch.int8}

    def __init__(self, cfg: OctoConfig, seed: int = 0):
        self.lib = _capi.lib()
        _declare(self.lib)
        self.cfg = cfg
        h = ctypes.c_void_p()
        _capi.check(self.lib.sfb_octo_create(ctypes.byref(cfg), seed, ctypes.byref(h)), "octo create")
        self.h = h

    def close(self):
        if self.h:
            self.lib.sfb_octo_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def encode(self, tokens=None, features=None, sessions: int | None = None, stream=None):
        """encode_condition: the backbone over tokens bf16 [B, seq_len, hidden]
        (None: the reference's 0.1 fill for `sessions` sessions); the output
        tokens go to `features` when given."""
        B = tokens.shape[0] if tokens is not None else (sessions or 1)
        _capi.check(self.lib.sfb_octo_encode(self.h, B, tokens.data_ptr() if tokens is not None else None,
                                             features.data_ptr() if features is not None else None,
                                             _sh(stream)), "octo encode")

    def set_condition(self, context, stream=None):
        """context bf16 [B, hidden] (or [B, 1, hidden])."""
        _capi.check(self.lib.sfb_octo_set_condition(self.h, context.shape[0], context.data_ptr(), _sh(stream)),
                    "octo set_condition")

    def denoise_step(self, x_t, t: float, velocity, stream=None):
        _capi.check(self.lib.sfb_octo_denoise_step(self.h, x_t.shape[0], x_t.data_ptr(), float(t),
                                                   velocity.data_ptr(), _sh(stream)), "octo denoise_step")

    def sample(self, noise, out, use_graph=True, stream=None):
        _capi.check(self.lib.sfb_octo_sample(self.h, noise.shape[0], noise.data_ptr(), out.data_ptr(),
                                             1 if use_graph else 0, _sh(stream)), "octo sample")

    def timesteps(self):
        n = self.cfg.num_steps + 1
        arr = (ctypes.c_float * n)()
        _capi.check(self.lib.sfb_octo_timesteps(self.h, ctypes.cast(arr, ctypes.c_void_p), n), "octo timesteps")
        return list(arr)

    def graph_kernels(self, sessions: int = 1) -> int:
        n = ctypes.c_int64()
        _capi.check(self.lib.sfb_octo_graph_kernels(self.h, sessions, ctypes.byref(n)), "octo graph_kernels")
        return n.value

    def param(self, name: str) -> torch.Tensor:
        """A copy (on the GPU) of a model parameter."""
        ptr, n, dt = ctypes.c_void_p(), ctypes.c_int64(), ctypes.c_int32()
        _capi.check(self.lib.sfb_octo_param(self.h, name.encode(), ctypes.byref(ptr), ctypes.byref(n),
                                            ctypes.byref(dt)), f"octo param {name}")
        out = torch.empty(n.value, dtype=self._DT[dt.value], device="cuda")
        torch.cuda.synchronize()
        _copy_d2d(out.data_ptr(), ptr.value, n.value * out.element_size())
        return out


def _main(argv=None):
    """Octo-Small latency run, the counterpart of the reference's
    examples/octo_inference.cpp: encode (backbone over the reference's 0.1
    tokens) then `--iters` samples of `num_steps` flow-matching steps in one
    graph; device-timed medians in ms, one line of JSON."""
    import argparse
    import json
    import statistics

    ap = argparse.ArgumentParser(description=_main.__doc__)
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args(argv)
    dev = torch.device("cuda:0")
    m = Octo(default_config(), seed=1)
    noise = torch.randn(1, m.cfg.action_horizon, m.cfg.action_dim, device=dev)
    act = torch.empty_like(noise)
    stream = torch.cuda.current_stream()

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.iters)]
        for a, b in ev:
            a.record(stream); fn(); b.record(stream)
        torch.cuda.synchronize()
        return statistics.median(a.elapsed_time(b) for a, b in ev)

    enc = timed(lambda: m.encode())
    smp = timed(lambda: m.sample(noise, act))
    print(json.dumps({"encode_ms": enc, "sample_ms": smp, "sample_graph_kernels": m.graph_kernels(1),
                      "finite": bool(torch.isfinite(act).all())}))
    m.close()


if __name__ == "__main__":
    _main()
