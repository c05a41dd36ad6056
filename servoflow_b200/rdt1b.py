"""Python handle on the RDT-1B denoising runtime of libsfb200 (C ABI
sfb_rdt1b_*). torch tensors supply device memory and streams only."""
from __future__ import annotations

import ctypes

import torch

from . import _capi


class RDT1BConfig(ctypes.Structure):
    """Mirror of ``sfb_rdt1b_config`` (include/sfb200.h)."""

    _fields_ = [(n, ctypes.c_int32) for n in (
        "num_layers", "hidden", "heads", "action_dim", "horizon", "state_dim", "lang_dim", "img_dim",
        "max_lang_len", "img_len", "max_sessions", "num_steps", "ctrl_freq")] + [
        ("weight_std", ctypes.c_float)]


def _declare(lib):
    c = ctypes
    if getattr(lib, "_rdt_declared", False):
        return
    lib.sfb_rdt1b_default_config.argtypes = [c.POINTER(RDT1BConfig)]
    lib.sfb_rdt1b_create.argtypes = [c.POINTER(RDT1BConfig), c.c_uint64, c.POINTER(c.c_void_p)]
    lib.sfb_rdt1b_destroy.argtypes = [c.c_void_p]
    lib.sfb_rdt1b_encode.argtypes = [c.c_void_p, c.c_int32, c.c_void_p, c.c_void_p, c.c_void_p,
                                     c.c_void_p, c.c_void_p]
    lib.sfb_rdt1b_forward.argtypes = [c.c_void_p, c.c_int32, c.c_void_p, c.c_float, c.c_void_p,
                                      c.c_void_p]
    lib.sfb_rdt1b_sample.argtypes = [c.c_void_p, c.c_int32, c.c_void_p, c.c_void_p, c.c_int32,
                                     c.c_void_p]
    lib.sfb_rdt1b_param.argtypes = [c.c_void_p, c.c_char_p, c.POINTER(c.c_void_p),
                                    c.POINTER(c.c_int64), c.POINTER(c.c_int32)]
    lib.sfb_rdt1b_schedule.argtypes = [c.c_void_p, c.c_void_p, c.c_void_p, c.c_void_p, c.c_void_p,
                                       c.c_int32]
    lib.sfb_rdt1b_graph_kernels.argtypes = [c.c_void_p, c.c_int32, c.POINTER(c.c_int64)]
    lib.sfb_rdt1b_set_path.argtypes = [c.c_void_p, c.c_int32]
    lib.sfb_rdt1b_profile_dense.argtypes = [c.c_void_p, c.c_float, c.c_int32, c.POINTER(c.c_int32),
                                            c.POINTER(c.c_double), c.POINTER(c.c_float), c.c_void_p]
    lib.sfb_rdt1b_tick.argtypes = [c.c_void_p, c.c_int32, c.c_uint64, c.c_void_p, c.c_void_p, c.c_void_p,
                                   c.c_void_p, c.c_void_p, c.c_void_p, c.c_void_p]
    lib.sfb_rdt1b_invalidate_condition.argtypes = [c.c_void_p]
    lib.sfb_rdt1b_tick_stats.argtypes = [c.c_void_p, c.POINTER(c.c_int64), c.POINTER(c.c_int64)]
    lib.sfb_rdt1b_config_from_json.argtypes = [c.c_char_p, c.POINTER(RDT1BConfig)]
    lib.sfb_rdt1b_load_safetensors.argtypes = [c.c_void_p, c.c_char_p, c.POINTER(c.c_int64),
                                               c.POINTER(c.c_int64)]
    lib.sfb_rdt1b_load_checkpoint.argtypes = [c.c_void_p, c.c_char_p, c.POINTER(c.c_int64),
                                              c.POINTER(c.c_int64)]
    lib.sfb_rdt1b_params_missing.argtypes = [c.c_void_p, c.POINTER(c.c_int64), c.c_char_p, c.c_int32]
    for f in ("default_config", "create", "destroy", "encode", "forward", "sample", "param",
              "schedule", "graph_kernels", "set_path", "tick", "invalidate_condition", "tick_stats", "config_from_json", "load_safetensors", "load_checkpoint",
              "params_missing"):
        getattr(lib, "sfb_rdt1b_" + f).restype = c.c_int
    lib._rdt_declared = True


def default_config(**overrides) -> RDT1BConfig:
    lib = _capi.lib()
    _declare(lib)
    cfg = RDT1BConfig()
    _capi.check(lib.sfb_rdt1b_default_config(ctypes.byref(cfg)), "default_config")
    for k, v in overrides.items():
        setattr(cfg, k, v)
    return cfg


def _sh(stream):
    return torch.cuda.current_stream().cuda_stream if stream is None else int(stream.cuda_stream)


class RDT1B:
    """Model handle: encode() once per control tick, sample() per chunk."""

    _DT = {_capi.SFB_BF16: torch.bfloat16, _capi.SFB_F32: torch.float32, _capi.SFB_I8: torch.int8}

    def __init__(self, cfg: RDT1BConfig, seed: int = 0):
        self.lib = _capi.lib()
        _declare(self.lib)
        self.cfg = cfg
        h = ctypes.c_void_p()
        _capi.check(self.lib.sfb_rdt1b_create(ctypes.byref(cfg), seed, ctypes.byref(h)), "rdt1b create")
        self.h = h

    def close(self):
        if self.h:
            self.lib.sfb_rdt1b_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def encode(self, lang, lang_len, img, state, stream=None):
        B = lang.shape[0]
        _capi.check(self.lib.sfb_rdt1b_encode(self.h, B, lang.data_ptr(), lang_len.data_ptr(),
                                              img.data_ptr(), state.data_ptr(), _sh(stream)),
                    "rdt1b encode")

    def forward(self, x_t, t: float, out, stream=None):
        _capi.check(self.lib.sfb_rdt1b_forward(self.h, x_t.shape[0], x_t.data_ptr(), float(t),
                                               out.data_ptr(), _sh(stream)), "rdt1b forward")

    def sample(self, noise, out, use_graph=True, stream=None):
        _capi.check(self.lib.sfb_rdt1b_sample(self.h, noise.shape[0], noise.data_ptr(), out.data_ptr(),
                                              1 if use_graph else 0, _sh(stream)), "rdt1b sample")

    def sample_host(self, noise, out, stream=None):
        """sample() from host noise into host actions (pinned CPU tensors keep
        the copies asynchronous); the copies run inside the same call."""
        assert not noise.is_cuda and not out.is_cuda
        _capi.check(self.lib.sfb_rdt1b_sample(self.h, noise.shape[0], noise.data_ptr(), out.data_ptr(),
                                              1, _sh(stream)), "rdt1b sample")

    def tick(self, frame_id: int, state, noise, actions, lang=None, lang_len=None, img=None,
             stream=None) -> None:
        """One control tick (sfb_rdt1b_tick): re-encodes lang/img only when
        frame_id changed, then denoises noise into actions. Every tensor may
        live on the host (pinned) or the device."""
        p = lambda t: None if t is None else t.data_ptr()
        _capi.check(self.lib.sfb_rdt1b_tick(self.h, noise.shape[0], int(frame_id), p(lang), p(lang_len), p(img),
                                            p(state), p(noise), p(actions), _sh(stream)), "tick")

    def invalidate_condition(self) -> None:
        _capi.check(self.lib.sfb_rdt1b_invalidate_condition(self.h), "invalidate_condition")

    def tick_stats(self):
        """(ticks, encodes) run on this handle."""
        t, e = ctypes.c_int64(), ctypes.c_int64()
        _capi.check(self.lib.sfb_rdt1b_tick_stats(self.h, ctypes.byref(t), ctypes.byref(e)), "tick_stats")
        return t.value, e.value

    def set_path(self, path: int) -> None:
        """One-session execution path (sfb_rdt1b_set_path): 0 the persistent
        kernel runs every projection and attention as stages, 1 one kernel per
        projection, norm and attention (default), 2 the persistent kernel
        between cross-attention kernels."""
        _capi.check(self.lib.sfb_rdt1b_set_path(self.h, int(path)), "set_path")

    def profile_dense(self, t: float = 999.0):
        """[(algorithmic bytes, microseconds)] of each persistent-kernel launch of
        one session-0 network evaluation at timestep t (sfb_rdt1b_profile_dense;
        synchronises the current stream)."""
        import torch
        n = ctypes.c_int32()
        stream = torch.cuda.current_stream().cuda_stream
        rc = self.lib.sfb_rdt1b_profile_dense(self.h, float(t), 0, ctypes.byref(n), None, None, stream)
        if rc not in (0, _capi.SFB_ERR_SHAPE):
            _capi.check(rc, "profile_dense")
        b = (ctypes.c_double * n.value)()
        us = (ctypes.c_float * n.value)()
        _capi.check(self.lib.sfb_rdt1b_profile_dense(self.h, float(t), n.value, ctypes.byref(n), b, us, stream),
                    "profile_dense")
        return list(zip(b, us))

    def graph_kernels(self, sessions: int = 1) -> int:
        """Kernel launches in the captured sampling graph for `sessions`."""
        n = ctypes.c_int64()
        _capi.check(self.lib.sfb_rdt1b_graph_kernels(self.h, sessions, ctypes.byref(n)), "graph_kernels")
        return n.value

    def param_ptr(self, name: str):
        """(device pointer, element count, SFB dtype code) of a parameter, no copy."""
        ptr, n, dt = ctypes.c_void_p(), ctypes.c_int64(), ctypes.c_int32()
        _capi.check(self.lib.sfb_rdt1b_param(self.h, name.encode(), ctypes.byref(ptr), ctypes.byref(n),
                                             ctypes.byref(dt)), f"param {name}")
        return ptr.value, n.value, dt.value

    def param(self, name: str) -> torch.Tensor:
        """A copy (on the GPU) of a model parameter."""
        ptr, n, dt = ctypes.c_void_p(), ctypes.c_int64(), ctypes.c_int32()
        _capi.check(self.lib.sfb_rdt1b_param(self.h, name.encode(), ctypes.byref(ptr), ctypes.byref(n),
                                             ctypes.byref(dt)), f"param {name}")
        out = torch.empty(n.value, dtype=self._DT[dt.value], device="cuda")
        torch.cuda.synchronize()
        _copy_d2d(out.data_ptr(), ptr.value, n.value * out.element_size())
        return out

    def load_safetensors(self, path: str):
        """Writes the parameters one .safetensors file provides (float
        projection weights are quantised to int8 per output channel on the
        device); returns (tensors loaded, entries ignored)."""
        loaded, ignored = ctypes.c_int64(), ctypes.c_int64()
        _capi.check(self.lib.sfb_rdt1b_load_safetensors(self.h, str(path).encode(), ctypes.byref(loaded),
                                                        ctypes.byref(ignored)), f"load {path}", detail=True)
        return loaded.value, ignored.value

    def load_checkpoint(self, checkpoint_dir: str):
        """Loads every *.safetensors of a checkpoint directory; raises if a
        model parameter is in none of them. Returns (loaded, ignored)."""
        loaded, ignored = ctypes.c_int64(), ctypes.c_int64()
        _capi.check(self.lib.sfb_rdt1b_load_checkpoint(self.h, str(checkpoint_dir).encode(),
                                                       ctypes.byref(loaded), ctypes.byref(ignored)),
                    f"load checkpoint {checkpoint_dir}", detail=True)
        return loaded.value, ignored.value

    def params_missing(self):
        """(number of parameters no load has written, the first one's name)."""
        n, buf = ctypes.c_int64(), ctypes.create_string_buffer(256)
        _capi.check(self.lib.sfb_rdt1b_params_missing(self.h, ctypes.byref(n), buf, 256), "params_missing")
        return n.value, buf.value.decode()

    def schedule(self):
        n = self.cfg.num_steps
        arrs = [(ctypes.c_float * n)() for _ in range(4)]
        _capi.check(self.lib.sfb_rdt1b_schedule(self.h, *[ctypes.cast(a, ctypes.c_void_p) for a in arrs], n),
                    "schedule")
        return [list(a) for a in arrs]


def _copy_d2d(dst: int, src: int, nbytes: int) -> None:
    lib = _capi.lib()
    if not hasattr(lib, "_copy_declared"):
        lib.sfb_copy_device.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
        lib.sfb_copy_device.restype = ctypes.c_int
        lib._copy_declared = True
    _capi.check(lib.sfb_copy_device(dst, src, nbytes), "copy")
