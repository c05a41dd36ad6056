"""CPU oracle of the Octo policy path (fp32, PyTorch on CPU).

TEST INFRASTRUCTURE ONLY (tests/ and bench.py's CPU legs; never the product).

A restatement of the reference's Octo model, evaluated on the exact weights
of a libsfb200 Octo model (int8 weights dequantised as q·s, padding sliced
off):

* OctoBlock::forward (src/models/octo/octo.cpp:46-122): pre-LN residual
  block, LayerNorm eps 1e-5 (octo.cpp:56,102), QKV packed as
  [Q heads | K heads | V heads] (unpack_qkv, src/backend/cuda/ops/
  attention.cu:203-237), SDPA with scale 1/sqrt(head_dim) and no mask (the
  reference's attention drops the mask, attention.cu:30), GELU in its tanh
  form (cuBLASLt's GELU epilogue, cuda_backend.cu:383-387).
* OctoDiffusionHead::forward (octo.cpp:144-177): [x_t flattened | 0.1 × 128
  | context] → fc1 GELU → fc2 GELU → fc3; t is not used (octo.cpp:147-148).
* OctoModel::encode_condition (octo.cpp:196-224): blocks over `seq_len`
  tokens (0.1 when none are given); readout = 0.1 fill.
* FlowMatchingSampler::sample (src/sampling/flow_matching.cpp:25-93) with
  Schedule::linspace (flow_matching.cpp:10-17): fp32 timesteps
  t_i = 1 + (i / n)·(0 − 1), x ← x + (t_{i+1} − t_i)·v with the product
  rounded before the sum.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

TIME_DIM = 128
FILL = 0.1


def timesteps(num_steps: int):
    """Schedule::linspace() in fp32 (flow_matching.cpp:10-17)."""
    n = np.float32(num_steps)
    out = []
    for i in range(num_steps + 1):
        alpha = np.float32(i) / n
        out.append(np.float32(np.float32(1.0) + alpha * np.float32(0.0 - 1.0)))
    return out


def layer_norm(x, g, b, eps=1e-5):
    mu = x.mean(-1, keepdim=True)
    var = (x - mu).pow(2).mean(-1, keepdim=True)
    return (x - mu) / torch.sqrt(var + eps) * g + b


class RefOcto:
    """fp32 Octo on CPU over a weight dict {name: float32 tensor}.

    store: None computes every tensor in fp32. A torch dtype rounds each
    tensor the model stores (block input and residual stream, LayerNorm
    outputs, QKV, attention output, fc1 output, the head's input and hidden
    layers) to that type, where the reference stores fp16 tensors and the
    runtime bf16 ones; the arithmetic between stores stays fp32."""

    def __init__(self, weights: dict, cfg, store=None):
        self.w = weights
        self.c = cfg
        self.store = store

    def r(self, x):
        return x if self.store is None else x.to(self.store).float()

    def lin(self, x, name, act=None):
        y = x @ self.w[name + ".weight"].t() + self.w[name + ".bias"]
        return F.gelu(y, approximate="tanh") if act == "gelu" else y

    def block(self, x, l):
        c, w = self.c, self.w
        B, S, D = x.shape
        H = c.heads
        p = f"blocks.{l}."
        r = self.r
        h = r(layer_norm(x, w[p + "norm1.weight"], w[p + "norm1.bias"]))
        qkv = r(self.lin(h, p + "attn.qkv")).view(B, S, 3, H, D // H)
        q, k, v = (qkv[:, :, i].transpose(1, 2) for i in range(3))
        with torch.nn.attention.sdpa_kernel(torch.nn.attention.SDPBackend.MATH):
            o = r(F.scaled_dot_product_attention(q, k, v))
        x = r(x + self.lin(o.transpose(1, 2).reshape(B, S, D), p + "attn.proj"))
        h = r(layer_norm(x, w[p + "norm2.weight"], w[p + "norm2.bias"]))
        return r(x + self.lin(r(self.lin(h, p + "mlp.fc1", "gelu")), p + "mlp.fc2"))

    def backbone(self, tokens):
        x = self.r(tokens)
        for l in range(self.c.num_layers):
            x = self.block(x, l)
        return x

    def encode(self, tokens=None, sessions: int = 1):
        """(backbone output, condition) as encode_condition with readout_token."""
        c = self.c
        if tokens is None:
            tokens = torch.full((sessions, c.seq_len, c.hidden), FILL)
        out = self.backbone(tokens)
        if c.readout_token < 0:
            cond = self.r(torch.full((tokens.shape[0], c.hidden), FILL))
        else:
            cond = out[:, c.readout_token]
        return out, cond

    def head(self, x_t, cond):
        B = x_t.shape[0]
        r = self.r
        inp = r(torch.cat([x_t.reshape(B, -1), torch.full((B, TIME_DIM), FILL), cond.reshape(B, -1)], 1))
        h = r(self.lin(r(self.lin(inp, "head.fc1", "gelu")), "head.fc2", "gelu"))
        return self.lin(h, "head.fc3").view_as(x_t)

    def sample(self, noise, cond):
        ts = timesteps(self.c.num_steps)
        x = noise.clone().float()
        for i in range(self.c.num_steps):
            v = self.head(x, cond)
            dt = float(np.float32(ts[i + 1] - ts[i]))
            x = x + (dt * v)                      # fp32 product, then the sum
        return x


def load_weights(model, cfg) -> dict:
    """Every parameter of a servoflow_b200.octo.Octo as fp32 CPU tensors, the
    padded head weights cut to their valid blocks."""
    D, Fd, Hh = cfg.hidden, cfg.intermediate, cfg.head_hidden
    Hp = (Hh + 63) // 64 * 64                     # the model pads the head's hidden width to 64
    HA = cfg.action_dim * cfg.action_horizon
    kin = HA + TIME_DIM + D
    kin_pad = (kin + 63) // 64 * 64
    out_pad = (HA + 127) // 128 * 128
    w = {}

    def lin(name, n, k, nv=None, kv=None):
        q = model.param(name + ".weight_q").view(n, k).float().cpu()
        s = model.param(name + ".weight_scale").float().cpu()
        full = q * s[:, None]
        w[name + ".weight"] = full[: nv or n, : kv or k]
        w[name + ".bias"] = model.param(name + ".bias").float().cpu()[: nv or n]
        w[name + ".weight_full"] = full
        w[name + ".bias_full"] = model.param(name + ".bias").float().cpu()

    for l in range(cfg.num_layers):
        p = f"blocks.{l}."
        for n in ("norm1", "norm2"):
            w[p + n + ".weight"] = model.param(p + n + ".weight").float().cpu()
            w[p + n + ".bias"] = model.param(p + n + ".bias").float().cpu()
        lin(p + "attn.qkv", 3 * D, D); lin(p + "attn.proj", D, D)
        lin(p + "mlp.fc1", Fd, D); lin(p + "mlp.fc2", D, Fd)
    lin("head.fc1", Hp, kin_pad, Hh, kin)
    lin("head.fc2", Hp, Hp, Hh, Hh)
    lin("head.fc3", out_pad, Hp, HA, Hh)
    return w


def random_weights(cfg, seed: int = 0, std: float = 0.02) -> dict:
    """fp32 weights of Octo's shapes (the CPU timing sample; values do not
    matter for timing)."""
    g = torch.Generator().manual_seed(seed)
    D, Fd, Hh = cfg.hidden, cfg.intermediate, cfg.head_hidden
    HA = cfg.action_dim * cfg.action_horizon
    w = {}

    def lin(name, n, k):
        w[name + ".weight"] = torch.randn(n, k, generator=g) * std
        w[name + ".bias"] = torch.randn(n, generator=g) * std

    for l in range(cfg.num_layers):
        p = f"blocks.{l}."
        for n in ("norm1", "norm2"):
            w[p + n + ".weight"] = 1 + torch.randn(D, generator=g) * 0.1
            w[p + n + ".bias"] = torch.randn(D, generator=g) * 0.1
        lin(p + "attn.qkv", 3 * D, D); lin(p + "attn.proj", D, D)
        lin(p + "mlp.fc1", Fd, D); lin(p + "mlp.fc2", D, Fd)
    lin("head.fc1", Hh, HA + TIME_DIM + D); lin("head.fc2", Hh, Hh); lin("head.fc3", HA, Hh)
    return w
