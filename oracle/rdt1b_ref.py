"""CPU oracle of the RDT-1B denoising path (fp32, PyTorch on CPU).

TEST INFRASTRUCTURE ONLY (tests/ and bench.py's CPU legs; never the product).

A restatement of the reference's PyTorch alignment model
(tests/alignment/test_rdt1b_alignment.py:73-210: RmsNorm, timestep embedder,
adaptors, self/cross attention with per-head qk RMSNorm, RDT blocks with
alternating language/image conditions, final layer) — the reference's own
oracle for its C++ model — evaluated on the exact weights of a libsfb200 model
(int8 weights dequantised as q·s). Two additions the reference's model lacks:
the language key-padding mask (keys at or beyond lang_len are masked with
-inf, the torch SDPA boolean-mask convention) and the DPM-Solver++ (2M)
sampler, restated here independently of the C++ code from the published
algorithm (Lu et al., "DPM-Solver++", 2022: data-prediction multistep solver)
over the squaredcos_cap_v2 DDPM schedule (Nichol & Dhariwal, 2021).
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F


def dpm_schedule(num_steps: int, train_steps: int = 1000):
    """(timesteps, a, b, c): step i maps x to a_i·x + b_i·x0_i + c_i·x0_{i-1}."""
    def abar(t):
        return math.cos((t + 0.008) / 1.008 * math.pi / 2) ** 2
    betas = [min(1 - abar((i + 1) / train_steps) / abar(i / train_steps), 0.999)
             for i in range(train_steps)]
    alphas_cumprod = np.cumprod(1.0 - np.array(betas, dtype=np.float64))
    ts = [int(round(x)) for x in np.linspace(0, train_steps - 1, num_steps + 1)[::-1][:-1]]
    alpha = lambda t: math.sqrt(alphas_cumprod[t])
    sigma = lambda t: math.sqrt(1 - alphas_cumprod[t])
    lam = lambda t: math.log(alpha(t) / sigma(t))
    a, b, c = [], [], []
    for i in range(num_steps):
        if i == num_steps - 1:                    # to noise level zero: the x0 estimate
            a.append(0.0); b.append(1.0); c.append(0.0)
            continue
        s, t = ts[i], ts[i + 1]
        h = lam(t) - lam(s)
        first = -alpha(t) * (math.exp(-h) - 1.0)
        if i == 0:                                # first order (DPM-Solver++ 1)
            a.append(sigma(t) / sigma(s)); b.append(first); c.append(0.0)
        else:                                     # second order multistep (2M)
            r = (lam(s) - lam(ts[i - 1])) / h
            a.append(sigma(t) / sigma(s)); b.append(first * (1 + 1 / (2 * r))); c.append(-first / (2 * r))
    return ts, a, b, c


def quantize_rows_int8(w: np.ndarray):
    """Per-output-channel symmetric int8 quantisation of a [N, K] float
    weight, the scheme whose dequantisation q·s is the reference's
    dequantize_int8 (src/backend/cuda/ops/quantization.cu:18-50): in fp32,
    s = max_k |w| / 127 (1 for an all-zero row), q = clip(rint(w / s), ±127)
    with rint rounding half to even. Returns (q int8 [N, K], s float32 [N])."""
    w = np.asarray(w, dtype=np.float32)
    mx = np.abs(w).max(axis=1)
    s = np.where(mx > 0, mx / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint(w / s[:, None]), -127, 127).astype(np.int8)
    return q, s


def rms_norm(x, w, eps=1e-6):
    return x / torch.sqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def sincos(t: float, dim: int = 256):
    half = dim // 2
    freq = torch.exp(-torch.arange(half, dtype=torch.float32) * math.log(10000) / half)
    x = torch.tensor(float(t)) * freq
    return torch.cat([x.cos(), x.sin()])


class RefRDT:
    """fp32 RDT-1B on CPU over a weight dict {name: float32 tensor}."""

    def __init__(self, weights: dict, cfg):
        self.w = weights
        self.c = cfg

    def lin(self, x, name, act=None):
        y = x @ self.w[name + ".weight"].t() + self.w[name + ".bias"]
        if act == "gelu":
            y = F.gelu(y, approximate="tanh")
        elif act == "silu":
            y = F.silu(y)
        return y

    def encode(self, lang, img):
        lang_c = self.lin(self.lin(lang, "lang_adaptor.0", "gelu"), "lang_adaptor.2")
        lang_c = lang_c + self.w["lang_cond_pos_embed"][: lang.shape[1]]
        img_c = self.lin(self.lin(img, "img_adaptor.0", "gelu"), "img_adaptor.2") + self.w["img_cond_pos_embed"]
        return lang_c, img_c

    def attn(self, q, k, v, H, key_len=None):
        B, Sq, D = q.shape
        Sk = k.shape[1]
        q = q.view(B, Sq, H, 64).transpose(1, 2)
        k = k.view(B, Sk, H, 64).transpose(1, 2)
        v = v.view(B, Sk, H, 64).transpose(1, 2)
        mask = None
        if key_len is not None:
            mask = (torch.arange(Sk)[None, :] < key_len[:, None])[:, None, None, :]
        with torch.nn.attention.sdpa_kernel(torch.nn.attention.SDPBackend.MATH):
            o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
        return o.transpose(1, 2).reshape(B, Sq, D)

    def cross_kv_all(self, lang_c, img_c):
        """Every block's cross-attention (K, V): the per-tick cache."""
        return [self.cross_kv(l, lang_c, img_c) for l in range(self.c.num_layers)]

    def forward(self, lang_c, img_c, lang_len, state, x_t, t, kv=None):
        """One network evaluation; kv (optional) is cross_kv_all's cache,
        otherwise each block projects its condition here."""
        c, w = self.c, self.w
        B, T, A = x_t.shape
        D, H = c.hidden, c.heads
        traj = torch.cat([torch.cat([state[:, None, :], x_t], 1), torch.ones(B, T + 1, A)], 2)
        seq = self.lin(self.lin(self.lin(traj, "state_adaptor.0", "gelu"), "state_adaptor.2", "gelu"),
                       "state_adaptor.4")
        temb = self.lin(self.lin(sincos(t), "t_embedder.mlp.0", "silu"), "t_embedder.mlp.2")
        femb = self.lin(self.lin(sincos(c.ctrl_freq), "freq_embedder.mlp.0", "silu"), "freq_embedder.mlp.2")
        x = torch.cat([temb.expand(B, 1, D), femb.expand(B, 1, D), seq], 1) + w["x_pos_embed"].view(-1, D)
        for l in range(c.num_layers):
            k, v = kv[l] if kv is not None else self.cross_kv(l, lang_c, img_c)
            x = self.block(x, l, k, v, lang_len)
        h = rms_norm(x, w["final_layer.norm_final.weight"])
        out = self.lin(self.lin(h, "final_layer.ffn_final.fc1", "gelu"), "final_layer.ffn_final.fc2")
        return out[:, -T:]

    def cross_kv(self, l, lang_c, img_c):
        """Block l's cross-attention K (k-normed) and V over its condition
        (language for even blocks, image for odd; dit_block.cu:288-308)."""
        c, w = self.c, self.w
        p = f"blocks.{l}."
        cond = lang_c if l % 2 == 0 else img_c
        B, D = cond.shape[0], c.hidden
        kv = self.lin(cond, p + "cross_attn.kv").view(B, -1, 2, c.heads, 64)
        k = rms_norm(kv[:, :, 0], w[p + "cross_attn.k_norm.weight"]).reshape(B, -1, D)
        return k, kv[:, :, 1].reshape(B, -1, D)

    def block(self, x, l, k, v, lang_len):
        """RDT block l (dit_block.cu:349-387) on x [B, S, D] with the block's
        cross-attention K/V; language blocks mask keys at or beyond lang_len."""
        c, w = self.c, self.w
        B, D, H = x.shape[0], c.hidden, c.heads
        p = f"blocks.{l}."
        h = rms_norm(x, w[p + "norm1.weight"])
        qkv = self.lin(h, p + "attn.qkv").view(B, -1, 3, H, 64)
        q = rms_norm(qkv[:, :, 0], w[p + "attn.q_norm.weight"]).reshape(B, -1, D)
        kk = rms_norm(qkv[:, :, 1], w[p + "attn.k_norm.weight"]).reshape(B, -1, D)
        vv = qkv[:, :, 2].reshape(B, -1, D)
        x = x + self.lin(self.attn(q, kk, vv, H), p + "attn.proj")
        h = rms_norm(x, w[p + "norm2.weight"])
        q = rms_norm(self.lin(h, p + "cross_attn.q").view(B, -1, H, 64),
                     w[p + "cross_attn.q_norm.weight"]).reshape(B, -1, D)
        x = x + self.lin(self.attn(q, k, v, H, lang_len if l % 2 == 0 else None), p + "cross_attn.proj")
        h = rms_norm(x, w[p + "norm3.weight"])
        return x + self.lin(self.lin(h, p + "ffn.fc1", "gelu"), p + "ffn.fc2")

    def sample(self, lang_c, img_c, lang_len, state, noise, kv=None):
        ts, a, b, cc = dpm_schedule(self.c.num_steps)
        if kv is None:
            kv = self.cross_kv_all(lang_c, img_c)     # once per tick, as the runtime's cache
        x, x0_prev = noise.clone(), torch.zeros_like(noise)
        for i, t in enumerate(ts):
            x0 = self.forward(lang_c, img_c, lang_len, state, x, t, kv)
            x = a[i] * x + b[i] * x0 + cc[i] * x0_prev
            x0_prev = x0
        return x


def load_weights(model, cfg) -> dict:
    """Reads every parameter of a servoflow_b200.rdt1b.RDT1B into fp32 CPU tensors."""
    D = cfg.hidden
    w = {}

    def lin(name, n, k):
        q = model.param(name + ".weight_q").view(n, k).float().cpu()
        s = model.param(name + ".weight_scale").float().cpu()
        w[name + ".weight"] = q * s[:, None]
        w[name + ".bias"] = model.param(name + ".bias").float().cpu()

    def vec(name, shape):
        w[name] = model.param(name).float().cpu().view(*shape)

    lin("lang_adaptor.0", D, cfg.lang_dim); lin("lang_adaptor.2", D, D)
    lin("img_adaptor.0", D, cfg.img_dim); lin("img_adaptor.2", D, D)
    lin("state_adaptor.0", D, 2 * cfg.state_dim); lin("state_adaptor.2", D, D); lin("state_adaptor.4", D, D)
    for e in ("t_embedder", "freq_embedder"):
        lin(e + ".mlp.0", D, 256); lin(e + ".mlp.2", D, D)
    vec("x_pos_embed", (cfg.horizon + 3, D))
    vec("lang_cond_pos_embed", (cfg.max_lang_len, D))
    vec("img_cond_pos_embed", (cfg.img_len, D))
    for l in range(cfg.num_layers):
        p = f"blocks.{l}."
        for n in ("norm1", "norm2", "norm3"):
            vec(p + n + ".weight", (D,))
        lin(p + "attn.qkv", 3 * D, D); lin(p + "attn.proj", D, D)
        vec(p + "attn.q_norm.weight", (64,)); vec(p + "attn.k_norm.weight", (64,))
        lin(p + "cross_attn.q", D, D); lin(p + "cross_attn.kv", 2 * D, D); lin(p + "cross_attn.proj", D, D)
        vec(p + "cross_attn.q_norm.weight", (64,)); vec(p + "cross_attn.k_norm.weight", (64,))
        lin(p + "ffn.fc1", D, D); lin(p + "ffn.fc2", D, D)
    vec("final_layer.norm_final.weight", (D,))
    lin("final_layer.ffn_final.fc1", D, D); lin("final_layer.ffn_final.fc2", cfg.action_dim, D)
    return w


def random_block_weights(cfg, layers, seed: int = 0, std: float = 0.02) -> dict:
    """fp32 weights N(0, std) for the listed blocks only (the CPU timing sample;
    the values do not matter for timing, the shapes are RDT-1B's)."""
    g = torch.Generator().manual_seed(seed)
    D = cfg.hidden
    w = {}

    def lin(name, n, k):
        w[name + ".weight"] = torch.randn(n, k, generator=g) * std
        w[name + ".bias"] = torch.randn(n, generator=g) * std

    for l in layers:
        p = f"blocks.{l}."
        for n in ("norm1", "norm2", "norm3"):
            w[p + n + ".weight"] = 1 + torch.randn(D, generator=g) * std
        lin(p + "attn.qkv", 3 * D, D); lin(p + "attn.proj", D, D)
        lin(p + "cross_attn.q", D, D); lin(p + "cross_attn.kv", 2 * D, D); lin(p + "cross_attn.proj", D, D)
        for n in ("attn.q_norm", "attn.k_norm", "cross_attn.q_norm", "cross_attn.k_norm"):
            w[p + n + ".weight"] = 1 + torch.randn(64, generator=g) * std
        lin(p + "ffn.fc1", D, D); lin(p + "ffn.fc2", D, D)
    return w


def random_weights(cfg, seed: int = 0, std: float = 0.02) -> dict:
    """fp32 weights N(0, std) for the whole network (every name load_weights
    returns) at cfg's shapes: the CPU timing workload, whose values do not
    matter for timing."""
    g = torch.Generator().manual_seed(seed)
    D = cfg.hidden
    w = random_block_weights(cfg, range(cfg.num_layers), seed=seed + 1, std=std)

    def lin(name, n, k):
        w[name + ".weight"] = torch.randn(n, k, generator=g) * std
        w[name + ".bias"] = torch.randn(n, generator=g) * std

    lin("lang_adaptor.0", D, cfg.lang_dim); lin("lang_adaptor.2", D, D)
    lin("img_adaptor.0", D, cfg.img_dim); lin("img_adaptor.2", D, D)
    lin("state_adaptor.0", D, 2 * cfg.state_dim); lin("state_adaptor.2", D, D); lin("state_adaptor.4", D, D)
    for e in ("t_embedder", "freq_embedder"):
        lin(e + ".mlp.0", D, 256); lin(e + ".mlp.2", D, D)
    w["x_pos_embed"] = torch.randn(cfg.horizon + 3, D, generator=g) * std
    w["lang_cond_pos_embed"] = torch.randn(cfg.max_lang_len, D, generator=g) * std
    w["img_cond_pos_embed"] = torch.randn(cfg.img_len, D, generator=g) * std
    w["final_layer.norm_final.weight"] = 1 + torch.randn(D, generator=g) * std
    lin("final_layer.ffn_final.fc1", D, D); lin("final_layer.ffn_final.fc2", cfg.action_dim, D)
    return w
