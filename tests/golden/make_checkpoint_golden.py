#!/usr/bin/env python3
"""Golden manifest of the reference's checkpoint converter, for pinning the
native checkpoint path (sfb_checkpoint_key, sfb_rdt1b_config_from_json,
sfb_rdt1b_load_checkpoint).

`hf_checkpoint()` builds a seeded HuggingFace-format RDTRunner checkpoint of a
small RDT-1B (hidden 256, 4 heads, 2 blocks): backbone tensors under
"model.", the three adaptors, action-normalisation statistics, and entries the
converter drops (EMA shadows, optimizer state, a vision tower). Most tensors
are fp32; a few are stored as fp16/bf16; one weight row is all zeros and one
holds an outlier. This script writes it to a temporary directory, runs the
reference's converter (tools/convert/hf_to_servoflow.py: remap_key,
convert(…, torch.bfloat16), write_servoflow_config) on it, and records in
rdt1b_checkpoint_manifest.json:
  mapping  — remap_key(name) for every HF entry (null = dropped);
  tensors  — dtype, shape and sha256 of every tensor the converter wrote;
  config   — the converter's config.json;  hf_config — the HF config given.
Tests regenerate the checkpoint from the seed, so the tensors themselves are
not stored.

    python tests/golden/make_checkpoint_golden.py /path/to/reference
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import sys
import tempfile

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "rdt1b_checkpoint_manifest.json")
SEED = 20261202

# the small model, in sfb_rdt1b_config field names
CFG = dict(num_layers=2, hidden=256, heads=4, action_dim=32, horizon=8, state_dim=32, lang_dim=64,
           img_dim=64, max_lang_len=10, img_len=12)

# an HF RDTRunner config.json for it (nested "rdt" / "noise_scheduler" keys)
HF_CONFIG = {
    "action_dim": CFG["action_dim"], "pred_horizon": CFG["horizon"], "img_cond_len": CFG["img_len"],
    "img_token_dim": CFG["img_dim"], "lang_token_dim": CFG["lang_dim"],
    "max_lang_cond_len": CFG["max_lang_len"], "state_token_dim": CFG["state_dim"],
    "rdt": {"hidden_size": CFG["hidden"], "depth": CFG["num_layers"], "num_heads": CFG["heads"]},
    "noise_scheduler": {"num_train_timesteps": 1000, "num_inference_timesteps": 5},
}

# stored in a half type in the HF file (exercises the on-device conversions)
HALF = {"model.blocks.1.ffn.fc1.weight": torch.float16, "img_adaptor.2.weight": torch.bfloat16,
        "model.x_pos_embed": torch.bfloat16, "model.blocks.0.norm2.weight": torch.float16}


def hf_checkpoint(seed: int = SEED) -> dict:
    """Seeded HF RDTRunner tensors {name: tensor} for CFG."""
    g = torch.Generator().manual_seed(seed)
    c = CFG
    D, A, S = c["hidden"], c["action_dim"], c["horizon"] + 3
    t = {}

    def lin(name, n, k):
        t[name + ".weight"] = torch.randn(n, k, generator=g) * 0.02
        t[name + ".bias"] = torch.randn(n, generator=g) * 0.02

    def vec(name, *shape, mean=0.0, std=0.02):
        t[name] = mean + torch.randn(*shape, generator=g) * std

    lin("lang_adaptor.0", D, c["lang_dim"]); lin("lang_adaptor.2", D, D)
    lin("img_adaptor.0", D, c["img_dim"]); lin("img_adaptor.2", D, D)
    lin("state_adaptor.0", D, 2 * c["state_dim"]); lin("state_adaptor.2", D, D); lin("state_adaptor.4", D, D)
    for e in ("t_embedder", "freq_embedder"):
        lin(f"model.{e}.mlp.0", D, 256); lin(f"model.{e}.mlp.2", D, D)
    vec("model.x_pos_embed", 1, S, D)
    vec("model.lang_cond_pos_embed", 1, c["max_lang_len"], D)
    vec("model.img_cond_pos_embed", 1, c["img_len"], D)
    for l in range(c["num_layers"]):
        p = f"model.blocks.{l}."
        for n in ("norm1", "norm2", "norm3"):
            vec(p + n + ".weight", D, mean=1.0, std=0.1)
        lin(p + "attn.qkv", 3 * D, D); lin(p + "attn.proj", D, D)
        lin(p + "cross_attn.q", D, D); lin(p + "cross_attn.kv", 2 * D, D); lin(p + "cross_attn.proj", D, D)
        for n in ("attn.q_norm", "attn.k_norm", "cross_attn.q_norm", "cross_attn.k_norm"):
            vec(p + n + ".weight", 64, mean=1.0, std=0.1)
        lin(p + "ffn.fc1", D, D); lin(p + "ffn.fc2", D, D)
    vec("model.final_layer.norm_final.weight", D, mean=1.0, std=0.1)
    lin("model.final_layer.ffn_final.fc1", D, D); lin("model.final_layer.ffn_final.fc2", A, D)
    # quantiser edge cases: an all-zero row, a row with one outlier
    t["model.blocks.0.ffn.fc2.weight"][5].zero_()
    t["model.blocks.1.attn.proj.weight"][7, 3] = 1.5
    # entries the converter keeps without a model parameter, and ones it drops
    vec("action_norm.mean", A); vec("action_norm.std", A, mean=1.0, std=0.1)
    vec("ema_model.blocks.0.norm1.weight", D)
    vec("model.blocks.0.norm1.weight.shadow_params", D)
    vec("optimizer.state.0.exp_avg", 4)
    vec("vision_encoder.patch_embed.weight", 8, 4)
    for name, dt in HALF.items():
        t[name] = t[name].to(dt)
    return {k: v.contiguous() for k, v in t.items()}


def write_hf(directory: str, seed: int = SEED) -> dict:
    """Writes the seeded HF checkpoint (model.safetensors + config.json)."""
    from safetensors.torch import save_file
    t = hf_checkpoint(seed)
    save_file(t, os.path.join(directory, "model.safetensors"))
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(HF_CONFIG, f)
    return t


def sha256(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def main(ref_root: str) -> None:
    from safetensors.torch import load_file
    path = os.path.join(ref_root, "tools", "convert", "hf_to_servoflow.py")
    spec = importlib.util.spec_from_file_location("ref_hf_to_servoflow", path)
    conv = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(conv)
    with tempfile.TemporaryDirectory() as tmp:
        hf_dir, sf_dir = os.path.join(tmp, "hf"), os.path.join(tmp, "sf")
        os.makedirs(hf_dir)
        t = write_hf(hf_dir)
        conv.convert(hf_dir, __import__("pathlib").Path(sf_dir), torch.bfloat16)
        out = load_file(os.path.join(sf_dir, "model.safetensors"))
        with open(os.path.join(sf_dir, "config.json")) as f:
            sf_config = json.load(f)
    manifest = {
        "seed": SEED,
        "cfg": CFG,
        "mapping": {k: conv.remap_key(k) for k in sorted(t)},
        "tensors": {k: {"dtype": str(v.dtype).replace("torch.", ""), "shape": list(v.shape), "sha256": sha256(v)}
                    for k, v in sorted(out.items())},
        "config": sf_config,
        "hf_config": HF_CONFIG,
    }
    with open(OUT, "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    print(f"wrote {OUT}: {len(manifest['tensors'])} converted tensors, "
          f"{sum(v is None for v in manifest['mapping'].values())} dropped")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SFB_REFERENCE", ""))
