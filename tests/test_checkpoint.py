"""CPU checks of the checkpoint path (no kernel runs): the native safetensors
reader against files written by the safetensors library, the key mapping and
config.json reading against the reference converter's own output
(tests/golden/rdt1b_checkpoint_manifest.json, made by
tests/golden/make_checkpoint_golden.py), and the error behaviour of the
reference's SafeTensorsLoader (src/loader/safetensors.cpp:65-100)."""
import importlib.util
import json
import os
import struct

import numpy as np
import pytest
import torch

from oracle.rdt1b_ref import quantize_rows_int8
from servoflow_b200 import _capi
from servoflow_b200 import checkpoint as ckpt

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _gen():
    spec = importlib.util.spec_from_file_location("make_checkpoint_golden",
                                                  os.path.join(GOLDEN, "make_checkpoint_golden.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


@pytest.fixture(scope="module")
def manifest():
    with open(os.path.join(GOLDEN, "rdt1b_checkpoint_manifest.json")) as f:
        return json.load(f)


def test_key_mapping_matches_the_converter(manifest):
    gen = _gen()
    assert sorted(gen.hf_checkpoint()) == sorted(manifest["mapping"])
    for hf, sf in manifest["mapping"].items():
        assert ckpt.checkpoint_key(hf) == sf, hf
    # names the converter's rules cover beyond the fixture
    assert ckpt.checkpoint_key("model.blocks.27.ffn.fc2.bias") == "blocks.27.ffn.fc2.bias"
    assert ckpt.checkpoint_key("lr_scheduler.last_epoch") is None
    assert ckpt.checkpoint_key("x_pos_embed") is None        # converted names carry no "model."


def test_inspect_matches_the_safetensors_library(tmp_path):
    from safetensors import safe_open
    gen = _gen()
    t = gen.write_hf(str(tmp_path))
    path = str(tmp_path / "model.safetensors")
    ours = ckpt.inspect(path)
    with open(path, "rb") as f:
        hlen = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(hlen))
    header.pop("__metadata__", None)
    assert [e["name"] for e in ours] == sorted(header) == sorted(t)
    with safe_open(path, framework="pt") as f:
        for e in ours:
            h = header[e["name"]]
            assert e["dtype"] == h["dtype"]
            assert list(e["shape"]) == h["shape"] == list(f.get_slice(e["name"]).get_shape())
            assert list(e["data_offsets"]) == h["data_offsets"]


def _write_raw(path, header_bytes, data=b"", hlen=None):
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(header_bytes) if hlen is None else hlen))
        f.write(header_bytes)
        f.write(data)


def test_inspect_errors(tmp_path):
    def status(path):
        try:
            ckpt.inspect(str(path))
            return 0
        except _capi.SfbError as e:
            return e.status

    assert status(tmp_path / "absent.safetensors") == _capi.SFB_ERR_IO
    (tmp_path / "short").write_bytes(b"\x01\x00")
    assert status(tmp_path / "short") == _capi.SFB_ERR_IO
    _write_raw(tmp_path / "long", b"{}", hlen=1 << 40)
    assert status(tmp_path / "long") == _capi.SFB_ERR_IO
    _write_raw(tmp_path / "bad", b'{"a": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]')
    assert status(tmp_path / "bad") == _capi.SFB_ERR_IO
    _write_raw(tmp_path / "f64", b'{"a": {"dtype": "F64", "shape": [1], "data_offsets": [0, 8]}}', b"\0" * 8)
    assert status(tmp_path / "f64") == _capi.SFB_ERR_DTYPE
    # metadata, escapes, unicode and an empty tensor parse
    hdr = json.dumps({"__metadata__": {"format": "pt", "note": "a\"b\\u00e9"},
                      "café.w": {"dtype": "BF16", "shape": [2, 0], "data_offsets": [0, 0]},
                      "b": {"dtype": "I8", "shape": [3], "data_offsets": [0, 3]}}).encode()
    _write_raw(tmp_path / "ok", hdr, b"\1\2\3")
    e = ckpt.inspect(str(tmp_path / "ok"))
    assert [x["name"] for x in e] == ["b", "café.w"]
    assert e[1]["shape"] == (2, 0) and e[0]["dtype"] == "I8"


def test_config_from_converter_and_hf_json(manifest, tmp_path):
    c = manifest["cfg"]
    for name, content in (("sf.json", manifest["config"]), ("hf.json", manifest["hf_config"])):
        p = tmp_path / name
        p.write_text(json.dumps(content))
        cfg = ckpt.config_from_json(str(p))
        for k, v in c.items():
            assert getattr(cfg, k) == v, (name, k)
        assert cfg.num_steps == 5 and cfg.max_sessions == 1 and cfg.ctrl_freq == 25
    # fields the runtime fixes, and RDT1BConfig::validate()
    bad = dict(manifest["config"], freq_dim=128)
    (tmp_path / "bad.json").write_text(json.dumps(bad))
    with pytest.raises(_capi.SfbError) as e:
        ckpt.config_from_json(str(tmp_path / "bad.json"))
    assert e.value.status == _capi.SFB_ERR_UNSUPPORTED
    (tmp_path / "heads.json").write_text(json.dumps({"hidden_size": 250, "num_attention_heads": 4}))
    with pytest.raises(_capi.SfbError) as e:
        ckpt.config_from_json(str(tmp_path / "heads.json"))
    assert e.value.status == _capi.SFB_ERR_INVALID


def test_converter_cast_is_round_to_nearest_even(manifest):
    # the converted tensors are torch's .to(bfloat16) of the HF tensors; the
    # device conversion of the loader is checked against these hashes on the GPU
    gen = _gen()
    t = gen.hf_checkpoint()
    for hf, sf in manifest["mapping"].items():
        if sf is None:
            continue
        target = torch.float32 if sf.startswith("action_norm.") else torch.bfloat16
        assert gen.sha256(t[hf].to(target)) == manifest["tensors"][sf]["sha256"], sf


def test_quantizer_restatement():
    rng = np.random.default_rng(0)
    w = rng.normal(0, 0.02, (6, 64)).astype(np.float32)
    w[2] = 0
    w[3, 5] = 1.5
    q, s = quantize_rows_int8(w)
    assert q.dtype == np.int8 and s.dtype == np.float32
    assert s[2] == 1 and not q[2].any()
    assert np.abs(q).max() == 127 and q[3, 5] == 127
    assert np.all(np.abs(q.astype(np.float32) * s[:, None] - w) <= s[:, None] / 2 + 1e-9)


def test_inspect_survives_corrupted_headers(tmp_path):
    """Truncated and byte-flipped copies of a valid file: the reader returns
    OK or an error status, never crashes (it parses untrusted files)."""
    import random
    from safetensors.torch import save_file
    save_file({"a.weight": torch.zeros(3, 4), "b": torch.ones(2, dtype=torch.int8)}, str(tmp_path / "ok.st"))
    good = (tmp_path / "ok.st").read_bytes()
    hlen = struct.unpack("<Q", good[:8])[0]
    rng = random.Random(7)
    bad = tmp_path / "bad.st"
    for i in range(300):
        b = bytearray(good)
        kind = i % 3
        if kind == 0:
            b = b[: rng.randrange(0, 8 + hlen + 1)]
        elif kind == 1:
            for _ in range(rng.randrange(1, 4)):
                b[rng.randrange(8, 8 + hlen)] = rng.randrange(256)
        else:
            b[:8] = struct.pack("<Q", rng.choice([0, 1, hlen - 1, hlen + 1, 2 ** 63, 2 ** 64 - 1]))
        bad.write_bytes(bytes(b))
        try:
            ckpt.inspect(str(bad))
        except _capi.SfbError as e:
            assert e.status in (_capi.SFB_ERR_IO, _capi.SFB_ERR_DTYPE, _capi.SFB_ERR_SHAPE), e.status


def test_config_reader_survives_corrupted_json(manifest, tmp_path):
    import random
    good = json.dumps(manifest["hf_config"]).encode()
    rng = random.Random(11)
    p = tmp_path / "cfg.json"
    for i in range(300):
        b = bytearray(good)
        if i % 2:
            b = b[: rng.randrange(0, len(b))]
        else:
            for _ in range(rng.randrange(1, 4)):
                b[rng.randrange(len(b))] = rng.randrange(256)
        p.write_bytes(bytes(b))
        try:
            ckpt.config_from_json(str(p))
        except _capi.SfbError as e:
            assert e.status in (_capi.SFB_ERR_IO, _capi.SFB_ERR_INVALID, _capi.SFB_ERR_UNSUPPORTED), e.status
    # deep nesting is refused, not recursed into without bound
    p.write_text("[" * 100000 + "]" * 100000)
    with pytest.raises(_capi.SfbError) as e:
        ckpt.config_from_json(str(p))
    assert e.value.status == _capi.SFB_ERR_IO
