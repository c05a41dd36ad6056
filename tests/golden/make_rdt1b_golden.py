#!/usr/bin/env python3
"""Golden output of the reference's own PyTorch RDT-1B model, for pinning the
CPU oracle network (oracle/rdt1b_ref.py).

The reference's alignment test defines a pure-PyTorch RDT-1B
(tests/alignment/test_rdt1b_alignment.py:73-210 in the reference project:
RmsNorm, sincos timestep embedder, adaptors, self/cross attention with
per-head qk-RMSNorm, RDT blocks alternating language/image conditions, final
layer) and its checkpoint-name loader (load_weights, :213-258). This script
imports that module from a checkout of the reference, builds a small model
(hidden 128 = 2 heads × 64, 2 blocks, short conditions), fills it with seeded
random weights through the reference's own loader, runs one network evaluation
in fp32 on CPU and stores inputs and output in rdt1b_small.npz. The weights are
not stored: `weights()` regenerates them from the seed (tests call it).

    python tests/golden/make_rdt1b_golden.py /path/to/reference
"""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "rdt1b_small.npz")

CFG = {
    "hidden_size": 128, "num_heads": 2, "head_dim": 64, "depth": 2, "action_dim": 16,
    "pred_horizon": 8, "img_cond_len": 12, "img_token_dim": 24, "lang_token_dim": 32,
    "state_token_dim": 16, "max_lang_cond_len": 10, "sincos_dim": 256, "x_seq_len": 11,
}
SEED = 20261201
T_STEP, FREQ = 500, 25


def weights(cfg=CFG, seed=SEED) -> dict:
    """Seeded fp32 weights under the reference checkpoint names."""
    g = torch.Generator().manual_seed(seed)
    D, A = cfg["hidden_size"], cfg["action_dim"]
    sd = {}

    def lin(name, n, k, std=0.08):
        sd[name + ".weight"] = torch.randn(n, k, generator=g) * std
        sd[name + ".bias"] = torch.randn(n, generator=g) * 0.02

    lin("lang_adaptor.0", D, cfg["lang_token_dim"]); lin("lang_adaptor.2", D, D)
    lin("img_adaptor.0", D, cfg["img_token_dim"]); lin("img_adaptor.2", D, D)
    lin("state_adaptor.0", D, 2 * cfg["state_token_dim"]); lin("state_adaptor.2", D, D)
    lin("state_adaptor.4", D, D)
    for e in ("t_embedder", "freq_embedder"):
        lin(e + ".mlp.0", D, cfg["sincos_dim"]); lin(e + ".mlp.2", D, D)
    sd["x_pos_embed"] = torch.randn(1, cfg["x_seq_len"], D, generator=g) * 0.02
    sd["lang_cond_pos_embed"] = torch.randn(1, cfg["max_lang_cond_len"], D, generator=g) * 0.02
    sd["img_cond_pos_embed"] = torch.randn(1, cfg["img_cond_len"], D, generator=g) * 0.02
    for i in range(cfg["depth"]):
        p = f"blocks.{i}."
        for n in ("norm1", "norm2", "norm3"):
            sd[p + n + ".weight"] = 1 + torch.randn(D, generator=g) * 0.1
        lin(p + "attn.qkv", 3 * D, D); lin(p + "attn.proj", D, D)
        lin(p + "cross_attn.q", D, D); lin(p + "cross_attn.kv", 2 * D, D); lin(p + "cross_attn.proj", D, D)
        for n in ("attn.q_norm", "attn.k_norm", "cross_attn.q_norm", "cross_attn.k_norm"):
            sd[p + n + ".weight"] = 1 + torch.randn(64, generator=g) * 0.1
        lin(p + "ffn.fc1", D, D); lin(p + "ffn.fc2", D, D)
    sd["final_layer.norm_final.weight"] = 1 + torch.randn(D, generator=g) * 0.1
    lin("final_layer.ffn_final.fc1", D, D); lin("final_layer.ffn_final.fc2", A, D)
    return sd


def inputs(cfg=CFG, seed=SEED + 1) -> dict:
    g = torch.Generator().manual_seed(seed)
    A, T = cfg["action_dim"], cfg["pred_horizon"]
    return {
        "lang": torch.randn(1, cfg["max_lang_cond_len"], cfg["lang_token_dim"], generator=g),
        "img": torch.randn(1, cfg["img_cond_len"], cfg["img_token_dim"], generator=g),
        "state": torch.randn(1, 1, A, generator=g),
        "noisy": torch.randn(1, T, A, generator=g),
    }


def main(ref_root: str) -> None:
    path = os.path.join(ref_root, "tests", "alignment", "test_rdt1b_alignment.py")
    spec = importlib.util.spec_from_file_location("ref_rdt1b_alignment", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    model = mod.RDT1BRef(CFG).eval()
    mod.load_weights(model, weights(), torch.float32)
    x = inputs()
    with torch.no_grad():
        out = model(x["lang"], x["img"], x["state"], x["noisy"],
                    torch.tensor([T_STEP]), torch.tensor([FREQ]))
    np.savez_compressed(OUT, **{k: v.numpy() for k, v in x.items()}, out=out.numpy(),
                        t=np.array(T_STEP), freq=np.array(FREQ))
    print(f"wrote {OUT}: out {tuple(out.shape)}, |out| mean {out.abs().mean():.4f}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SFB_REFERENCE", ""))
