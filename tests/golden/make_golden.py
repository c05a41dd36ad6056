"""Generates the golden attention fixtures with the reference's own Python
oracle: torch.nn.functional.scaled_dot_product_attention in math mode on CPU
(tests/alignment/test_rdt1b_alignment.py:133-134,148-149 of the reference),
on seeded N(0,1) inputs made the way the reference makes its alignment
inputs (torch.manual_seed + torch.randn, :260-272).

    python tests/golden/make_golden.py

Outputs (committed, small):
  attn_self_f32.npz   — config 1 shape (Lq = Lk = 67, D = 64, scale 1/8, no
                        mask), fp32, 2 of the 32 heads.
  attn_masked_f32.npz — key-padding mask (bool [B, Sk], False → −inf), B = 2,
                        H = 1, Lq = 67, Lk = 144, per-batch valid lengths.
  attn_const.npz      — the constant-input case of the reference's attention
                        bench (benchmarks/bench_attention.cu:50-52): Q = K =
                        V = 0.01, so out = 0.01 whatever the softmax.
The dequant known answers (tests/unit/test_quantization.cpp:9-94) are small
enough to live in dequant_kat.json, written by this script too.
"""
from __future__ import annotations

import json
import os

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))


def sdpa_math(q, k, v, mask=None, scale=None):
    with torch.nn.attention.sdpa_kernel(torch.nn.attention.SDPBackend.MATH):
        return F.scaled_dot_product_attention(q, k, v, attn_mask=mask, scale=scale)


def main():
    torch.manual_seed(42)
    B, H, L, D = 1, 2, 67, 64
    q = torch.randn(B, H, L, D, dtype=torch.float32).double()
    k = torch.randn(B, H, L, D, dtype=torch.float32).double()
    v = torch.randn(B, H, L, D, dtype=torch.float32).double()
    o = sdpa_math(q, k, v, scale=1.0 / 8.0)
    np.savez(os.path.join(HERE, "attn_self_f32.npz"), q=q.float().numpy(), k=k.float().numpy(),
             v=v.float().numpy(), out=o.float().numpy(), scale=np.float32(0.125))

    torch.manual_seed(7)
    B, H, Lq, Lk = 2, 1, 67, 144
    q = torch.randn(B, H, Lq, D, dtype=torch.float32).double()
    k = torch.randn(B, H, Lk, D, dtype=torch.float32).double()
    v = torch.randn(B, H, Lk, D, dtype=torch.float32).double()
    lens = torch.tensor([37, 144], dtype=torch.int32)
    keep = torch.arange(Lk)[None, :] < lens[:, None]
    keep[0, 5] = False            # a hole inside the valid prefix
    o = sdpa_math(q, k, v, mask=keep[:, None, None, :])
    np.savez(os.path.join(HERE, "attn_masked_f32.npz"), q=q.float().numpy(), k=k.float().numpy(),
             v=v.float().numpy(), out=o.float().numpy(), key_mask=keep.numpy().astype(np.uint8),
             scale=np.float32(0.0))

    q = torch.full((1, 2, 16, 64), 0.01, dtype=torch.float32).double()
    o = sdpa_math(q, q, q)
    np.savez_compressed(os.path.join(HERE, "attn_const.npz"), value=np.float32(0.01), out=o.float().numpy())

    kat = {
        "source": "reference tests/unit/test_quantization.cpp:9-94",
        "per_tensor": {"q": [[-10, -5, 0, 5], [10, 20, 30, 40]], "scale": [0.5],
                       "out": [[-5, -2.5, 0, 2.5], [5, 10, 15, 20]], "tol": 1e-2},
        "per_channel": {"q": [[10, 10, 10, 10], [20, 20, 20, 20]], "scale": [0.5, 2.0],
                        "out": [[5, 5, 5, 5], [40, 40, 40, 40]], "tol": 1e-2},
    }
    with open(os.path.join(HERE, "dequant_kat.json"), "w") as f:
        json.dump(kat, f, indent=1)


if __name__ == "__main__":
    main()
