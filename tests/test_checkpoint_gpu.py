"""GPU tests of the checkpoint path: a seeded HF RDTRunner checkpoint and the
reference converter's output (both pinned by
tests/golden/rdt1b_checkpoint_manifest.json) load into the runtime. Every
int8 weight and scale must equal the quantiser restated in
oracle/rdt1b_ref.quantize_rows_int8 bit for bit. Every other parameter must
hash-equal the converter's bf16 cast. The loaded model must match the CPU
oracle network by the reference's alignment bar (max |Δ| < 0.05, cosine
> 0.9999)."""
import importlib.util
import json
import os

import numpy as np
import pytest
import torch

from oracle import rdt1b_ref
from servoflow_b200 import _capi
from servoflow_b200 import checkpoint as ckpt
from servoflow_b200.rdt1b import RDT1B

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _gen():
    spec = importlib.util.spec_from_file_location("make_checkpoint_golden",
                                                  os.path.join(GOLDEN, "make_checkpoint_golden.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


gen = _gen()


@pytest.fixture(scope="module")
def manifest():
    with open(os.path.join(GOLDEN, "rdt1b_checkpoint_manifest.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def hf(tmp_path_factory):
    d = tmp_path_factory.mktemp("hf")
    return str(d), gen.write_hf(str(d))


def _quantised(sf):
    return sf.endswith(".weight") and "norm" not in sf


def _check_params(model, manifest, source):
    """source: {servoflow name: the float tensor the loader read}."""
    for sf, t in source.items():
        if sf.startswith("action_norm."):
            continue
        if _quantised(sf):
            base = sf[: -len(".weight")]
            q_ref, s_ref = rdt1b_ref.quantize_rows_int8(t.float().numpy())
            q = model.param(base + ".weight_q").cpu().numpy().reshape(q_ref.shape)
            s = model.param(base + ".weight_scale").cpu().numpy()
            assert np.array_equal(s, s_ref), sf
            assert np.array_equal(q, q_ref), sf
        else:
            p = model.param(sf).cpu()
            assert gen.sha256(p) == manifest["tensors"][sf]["sha256"], sf


def test_load_hf_checkpoint(gpu, hf, manifest):
    d, t = hf
    cfg = ckpt.config_from_json(os.path.join(d, "config.json"))
    model = RDT1B(cfg, seed=7)
    try:
        assert model.params_missing()[0] > 0
        loaded, ignored = model.load_checkpoint(d)
        assert model.params_missing() == (0, "")
        kept = {sf: t[hf_name] for hf_name, sf in manifest["mapping"].items() if sf is not None}
        assert ignored == len(t) - len(kept) + 2          # dropped entries + action_norm.{mean,std}
        assert loaded == len(kept) - 2
        _check_params(model, manifest, kept)
    finally:
        model.close()


@pytest.fixture(scope="module")
def converted(tmp_path_factory, hf, manifest):
    """The reference converter's output, rebuilt from the seed and checked
    against its recorded hashes."""
    from safetensors.torch import save_file
    _, t = hf
    out = {}
    for hf_name, sf in manifest["mapping"].items():
        if sf is None:
            continue
        out[sf] = t[hf_name].to(torch.float32 if sf.startswith("action_norm.") else torch.bfloat16).contiguous()
        assert gen.sha256(out[sf]) == manifest["tensors"][sf]["sha256"], sf
    assert sorted(out) == sorted(manifest["tensors"])
    d = tmp_path_factory.mktemp("sf")
    # two shards, as the converter writes above its shard size
    names = sorted(out)
    save_file({k: out[k] for k in names[::2]}, str(d / "model-00001-of-00002.safetensors"))
    save_file({k: out[k] for k in names[1::2]}, str(d / "model-00002-of-00002.safetensors"))
    (d / "config.json").write_text(json.dumps(manifest["config"]))
    return str(d), out


def test_load_converted_checkpoint_and_run(gpu, converted, manifest):
    d, out = converted
    model = ckpt.load_rdt1b(d, max_sessions=1)
    try:
        _check_params(model, manifest, out)
        cfg = model.cfg
        g = torch.Generator().manual_seed(3)
        lang = torch.randn(1, cfg.max_lang_len, cfg.lang_dim, generator=g).bfloat16()
        img = torch.randn(1, cfg.img_len, cfg.img_dim, generator=g).bfloat16()
        state = torch.randn(1, cfg.state_dim, generator=g).bfloat16()
        lens = torch.tensor([7], dtype=torch.int32)
        noise = torch.randn(1, cfg.horizon, cfg.action_dim, generator=g)
        model.encode(lang.to(gpu), lens.to(gpu), img.to(gpu), state.to(gpu))
        y = torch.empty(1, cfg.horizon, cfg.action_dim, device=gpu)
        model.forward(noise.to(gpu), 599.0, y)
        torch.cuda.synchronize()
        ref = rdt1b_ref.RefRDT(rdt1b_ref.load_weights(model, cfg), cfg)
        lang_c, img_c = ref.encode(lang.float(), img.float())
        r = ref.forward(lang_c, img_c, lens, state.float(), noise, 599)
        a, b = y.cpu().reshape(-1).double(), r.reshape(-1).double()
        max_abs = (a - b).abs().max().item()
        cos = torch.nn.functional.cosine_similarity(a[None], b[None]).item()
        assert max_abs < 0.05 and cos > 0.9999, (max_abs, cos)
    finally:
        model.close()


def test_missing_and_misshapen_tensors(gpu, converted, manifest, tmp_path):
    from safetensors.torch import save_file
    _, out = converted
    cfg = ckpt.config_from_json(os.path.join(converted[0], "config.json"))
    partial = {k: v for k, v in out.items() if k != "blocks.1.cross_attn.kv.weight"}
    save_file(partial, str(tmp_path / "model.safetensors"))
    model = RDT1B(cfg)
    try:
        with pytest.raises(_capi.SfbError) as e:
            model.load_checkpoint(str(tmp_path))
        assert e.value.status == _capi.SFB_ERR_INVALID and "blocks.1.cross_attn.kv" in str(e.value)
        n, first = model.params_missing()
        assert n == 2 and first.startswith("blocks.1.cross_attn.kv.weight_")
        bad = tmp_path / "bad.safetensors"
        save_file({"blocks.0.attn.proj.weight": torch.zeros(cfg.hidden, cfg.hidden + 64)}, str(bad))
        with pytest.raises(_capi.SfbError) as e:
            model.load_safetensors(str(bad))
        assert e.value.status == _capi.SFB_ERR_SHAPE
        save_file({"blocks.0.norm1.weight": torch.zeros(cfg.hidden, dtype=torch.int32)}, str(bad))
        with pytest.raises(_capi.SfbError) as e:
            model.load_safetensors(str(bad))
        assert e.value.status == _capi.SFB_ERR_DTYPE
        # a float weight holding a NaN or an infinity has no int8 value: the load fails
        for bad_value in (float("nan"), float("inf")):
            w = torch.randn(cfg.hidden, cfg.hidden) * 0.02
            w[5, 17] = bad_value
            save_file({"blocks.0.attn.proj.weight": w}, str(bad))
            with pytest.raises(_capi.SfbError) as e:
                model.load_safetensors(str(bad))
            assert e.value.status == _capi.SFB_ERR_RANGE and "blocks.0.attn.proj.weight" in str(e.value)
    finally:
        model.close()


def test_prequantised_pairs_round_trip(gpu, converted, tmp_path):
    """An int8 checkpoint (weight_q int8 + weight_scale fp32 per projection, as
    the model stores them) loads bit for bit into a second model."""
    from safetensors.torch import save_file
    cfg = ckpt.config_from_json(os.path.join(converted[0], "config.json"))
    a = ckpt.load_rdt1b(converted[0])
    b = RDT1B(cfg, seed=99)
    try:
        names = ["blocks.1.attn.qkv", "blocks.0.ffn.fc2", "final_layer.ffn_final.fc2"]
        t = {}
        for n in names:
            t[n + ".weight_q"] = a.param(n + ".weight_q").cpu()
            t[n + ".weight_scale"] = a.param(n + ".weight_scale").cpu()
            t[n + ".bias"] = a.param(n + ".bias").cpu()
        save_file(t, str(tmp_path / "int8.safetensors"))
        loaded, ignored = b.load_safetensors(str(tmp_path / "int8.safetensors"))
        assert (loaded, ignored) == (3 * len(names), 0)
        for k, v in t.items():
            assert torch.equal(b.param(k).cpu(), v), k
    finally:
        a.close()
        b.close()
