"""CPU tests of the Octo path: the oracle's pieces against their definitions
in the reference, the default configuration, and the C-ABI argument checks
(no device needed)."""
import ctypes

import numpy as np
import torch
import torch.nn.functional as F

from oracle import octo_ref
from servoflow_b200 import _capi
from servoflow_b200.octo import _declare, default_config


def test_timesteps_follow_schedule_linspace():
    """Schedule::linspace (flow_matching.cpp:10-17) in fp32: 1 → 0 in n steps."""
    ts = octo_ref.timesteps(10)
    assert len(ts) == 11 and ts[0] == 1.0 and ts[-1] == 0.0
    for i, t in enumerate(ts):
        alpha = np.float32(i) / np.float32(10)
        assert t == np.float32(1.0) + alpha * np.float32(-1.0)
        assert t.dtype == np.float32
    assert all(ts[i + 1] < ts[i] for i in range(10))


def test_layer_norm_matches_torch():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(5, 384, generator=g) * 3 + 1
    w, b = torch.randn(384, generator=g), torch.randn(384, generator=g)
    ref = F.layer_norm(x, (384,), w, b, eps=1e-5)
    assert torch.allclose(octo_ref.layer_norm(x, w, b), ref, atol=1e-5, rtol=1e-5)


class _Cfg:
    num_layers, hidden, heads, intermediate = 1, 128, 2, 256
    action_dim, action_horizon, head_hidden, seq_len, num_steps, readout_token = 7, 4, 64, 8, 3, -1


def test_oracle_head_input_and_euler():
    """The head concatenates [x_t | 0.1 × 128 | context] (octo.cpp:150-160)
    and the sampler adds dt·v per step (flow_matching.cpp:69-74)."""
    cfg = _Cfg()
    w = octo_ref.random_weights(cfg, seed=1)
    assert w["head.fc1.weight"].shape == (64, 28 + 128 + 128)
    ref = octo_ref.RefOcto(w, cfg)
    x = torch.randn(2, 4, 7)
    cond = torch.randn(2, 128)
    inp = torch.cat([x.reshape(2, -1), torch.full((2, 128), 0.1), cond], 1)
    h = F.gelu(inp @ w["head.fc1.weight"].t() + w["head.fc1.bias"], approximate="tanh")
    h = F.gelu(h @ w["head.fc2.weight"].t() + w["head.fc2.bias"], approximate="tanh")
    v = (h @ w["head.fc3.weight"].t() + w["head.fc3.bias"]).view(2, 4, 7)
    assert torch.equal(ref.head(x, cond), v)
    ts = octo_ref.timesteps(3)
    xs = x.clone()
    for i in range(3):
        xs = xs + float(ts[i + 1] - ts[i]) * ref.head(xs, cond)
    assert torch.equal(ref.sample(x, cond), xs)


def test_oracle_encode_readout_is_the_reference_fill():
    cfg = _Cfg()
    ref = octo_ref.RefOcto(octo_ref.random_weights(cfg, seed=2), cfg)
    out, cond = ref.encode(None, sessions=2)
    assert out.shape == (2, 8, 128) and torch.equal(cond, torch.full((2, 128), 0.1))
    cfg.readout_token = 3
    out, cond = ref.encode(torch.randn(2, 8, 128))
    assert torch.equal(cond, out[:, 3])


def test_default_config_is_octo_small():
    """OctoConfig defaults (include/servoflow/models/octo/config.h:17-38) and
    the sampler's 10 steps (sampler.h:24)."""
    c = default_config()
    assert (c.num_layers, c.hidden, c.heads, c.head_dim, c.intermediate) == (12, 384, 6, 64, 1536)
    assert (c.action_dim, c.action_horizon, c.head_hidden, c.seq_len) == (7, 4, 256, 64)
    assert (c.max_sessions, c.num_steps, c.readout_token) == (1, 10, -1)


def test_api_argument_checks_without_a_gpu():
    lib = _capi.lib()
    _declare(lib)
    h = ctypes.c_void_p()
    cfg = default_config()
    assert lib.sfb_octo_create(None, 0, ctypes.byref(h)) == _capi.SFB_ERR_INVALID
    assert lib.sfb_octo_create(ctypes.byref(cfg), 0, None) == _capi.SFB_ERR_INVALID
    for bad in (dict(head_dim=32), dict(head_dim=48, heads=8), dict(hidden=400), dict(heads=5),
                dict(num_layers=0), dict(intermediate=100), dict(head_hidden=0), dict(max_sessions=0),
                dict(num_steps=0),
                dict(seq_len=0), dict(readout_token=64), dict(action_dim=0)):
        c = default_config(**bad)
        assert lib.sfb_octo_create(ctypes.byref(c), 0, ctypes.byref(h)) == _capi.SFB_ERR_SHAPE, bad
    x = ctypes.c_void_p(1)
    assert lib.sfb_octo_encode(None, 1, x, x, None) == _capi.SFB_ERR_INVALID
    assert lib.sfb_octo_set_condition(None, 1, x, None) == _capi.SFB_ERR_INVALID
    assert lib.sfb_octo_denoise_step(None, 1, x, 0.5, x, None) == _capi.SFB_ERR_INVALID
    assert lib.sfb_octo_sample(None, 1, x, x, 1, None) == _capi.SFB_ERR_INVALID
    assert lib.sfb_octo_timesteps(None, None, 11) == _capi.SFB_ERR_INVALID
    assert lib.sfb_octo_destroy(None) == _capi.SFB_ERR_INVALID
    n = ctypes.c_int64()
    assert lib.sfb_octo_graph_kernels(None, 1, ctypes.byref(n)) == _capi.SFB_ERR_INVALID
