"""CPU checks of the oracle against the reference's golden vectors and its
Python oracle (torch SDPA math), so the oracle can be trusted as the GPU
parity checker."""
import json
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def sdpa(q, k, v, mask=None, scale=None, causal=False):
    with torch.nn.attention.sdpa_kernel(torch.nn.attention.SDPBackend.MATH):
        return F.scaled_dot_product_attention(
            torch.from_numpy(q).double(), torch.from_numpy(k).double(), torch.from_numpy(v).double(),
            attn_mask=mask, scale=scale, is_causal=causal).numpy()


def test_golden_self_attention_fp32():
    g = np.load(os.path.join(GOLDEN, "attn_self_f32.npz"))
    out = oracle.attention(g["q"], g["k"], g["v"], scale=float(g["scale"]))
    assert np.abs(out - g["out"]).max() <= 1e-6


def test_golden_masked():
    g = np.load(os.path.join(GOLDEN, "attn_masked_f32.npz"))
    out = oracle.attention(g["q"], g["k"], g["v"], key_mask=g["key_mask"])
    assert np.abs(out - g["out"]).max() <= 1e-6


def test_golden_constant_kat():
    g = np.load(os.path.join(GOLDEN, "attn_const.npz"))
    q = np.full(g["out"].shape, float(g["value"]), np.float32)
    out = oracle.attention(q, q, q)
    assert np.abs(out - g["out"]).max() <= 1e-7
    assert np.abs(out - 0.01).max() <= 1e-7


def test_scale_zero_means_inv_sqrt_d():
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((1, 2, 9, 32), dtype=np.float32) for _ in range(3))
    a = oracle.attention(q, k, v, scale=0.0)
    b = oracle.attention(q, k, v, scale=1.0 / np.sqrt(32))
    assert np.array_equal(a, b)


@pytest.mark.parametrize("Lq,Lk", [(1, 1), (5, 67), (67, 67), (130, 31)])
def test_causal_matches_sdpa(Lq, Lk):
    rng = np.random.default_rng(Lq * 1000 + Lk)
    q = rng.standard_normal((1, 2, Lq, 64), dtype=np.float32)
    k = rng.standard_normal((1, 2, Lk, 64), dtype=np.float32)
    v = rng.standard_normal((1, 2, Lk, 64), dtype=np.float32)
    # top-left causal, like the reference kernel (attention.cu:117) and SDPA
    keep = np.tril(np.ones((Lq, Lk), dtype=bool))
    ref = sdpa(q, k, v, mask=torch.from_numpy(keep))
    out = oracle.attention(q, k, v, causal=True)
    assert np.abs(out - ref).max() <= 1e-6


def test_kv_len_and_gqa_match_sdpa():
    rng = np.random.default_rng(3)
    B, H, Hkv, Lq, Lk = 3, 4, 2, 11, 40
    q = rng.standard_normal((B, H, Lq, 64), dtype=np.float32)
    k = rng.standard_normal((B, Hkv, Lk, 64), dtype=np.float32)
    v = rng.standard_normal((B, Hkv, Lk, 64), dtype=np.float32)
    lens = np.array([40, 1, 17], np.int32)
    keep = np.arange(Lk)[None, :] < lens[:, None]
    ref = sdpa(q, np.repeat(k, 2, axis=1), np.repeat(v, 2, axis=1),
               mask=torch.from_numpy(keep[:, None, None, :]))
    out = oracle.attention(q, k, v, kv_len=lens)
    assert np.abs(out - ref).max() <= 1e-6


@pytest.mark.parametrize("shape", [(2, 1, 9, 40), (1, 1, 9, 40), (2, 1, 1, 40)])
def test_additive_mask_matches_sdpa(shape):
    """The float [B, 1, Sq, Sk] mask of IBackend::attention (ops/attention.h:16),
    added to the scaled logits as torch SDPA adds a float attn_mask; -inf drops
    a key. Broadcast forms [1, 1, Sq, Sk] and [B, 1, 1, Sk] included."""
    rng = np.random.default_rng(sum(shape))
    B, H, Lq, Lk = 2, 3, 9, 40
    q = rng.standard_normal((B, H, Lq, 64), dtype=np.float32)
    k = rng.standard_normal((B, H, Lk, 64), dtype=np.float32)
    v = rng.standard_normal((B, H, Lk, 64), dtype=np.float32)
    m = rng.standard_normal(shape).astype(np.float32) * 2
    m[rng.random(shape) < 0.25] = -np.inf
    m[..., 0] = 0.0                        # every row keeps a key
    ref = sdpa(q, k, v, mask=torch.from_numpy(m).double())
    out = oracle.attention(q, k, v, attn_mask=m)
    assert np.abs(out - ref).max() <= 1e-6


def test_fully_masked_row_is_zero():
    q = np.ones((2, 1, 3, 64), np.float32)
    out = oracle.attention(q, q, q, kv_len=np.array([0, 3], np.int32))
    assert np.all(out[0] == 0) and np.allclose(out[1], 1.0)


def test_dequant_kats():
    with open(os.path.join(GOLDEN, "dequant_kat.json")) as f:
        kat = json.load(f)
    for case in ("per_tensor", "per_channel"):
        c = kat[case]
        out = oracle.dequant_int8(np.array(c["q"], np.int8), np.array(c["scale"], np.float32),
                                  round_mode=1)
        assert np.abs(out - np.array(c["out"], np.float32)).max() <= c["tol"]


def test_f16_rounding_matches_numpy():
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.standard_normal(2000).astype(np.float32) * 10 ** rng.uniform(-6, 4, 2000)
                        .astype(np.float32), np.array([65504, 65519, 1e-8, -3e-5], np.float32)])
    ours = np.array([oracle.lib().sfo_round_f16(float(v)) for v in x], np.float32)
    assert np.array_equal(ours, x.astype(np.float16).astype(np.float32))


def test_bf16_rounding_matches_torch():
    x = torch.randn(4000) * 37
    ours = np.array([oracle.lib().sfo_round_bf16(float(v)) for v in x], np.float32)
    assert np.array_equal(ours, x.bfloat16().float().numpy())


def test_dequant_fp16_rounding_is_reference_hmul():
    # int8 · fp16 is exact in fp32, so __hmul rounds the exact product once
    rng = np.random.default_rng(9)
    q = rng.integers(-128, 128, (8, 32), dtype=np.int8)
    s = rng.uniform(1e-3, 1e-1, 8).astype(np.float16).astype(np.float32)
    out = oracle.dequant_int8(q, s, round_mode=1)
    exact = q.astype(np.float64) * s[:, None].astype(np.float64)
    assert np.array_equal(out, exact.astype(np.float16).astype(np.float32))


def test_rdt1b_oracle_matches_reference_model():
    """oracle/rdt1b_ref.RefRDT against the reference's own PyTorch RDT-1B
    (tests/alignment/test_rdt1b_alignment.py:73-210 in the reference), run by
    tests/golden/make_rdt1b_golden.py on seeded weights and inputs: full
    language length (no masking), fp32."""
    import importlib.util
    from types import SimpleNamespace
    from oracle.rdt1b_ref import RefRDT

    spec = importlib.util.spec_from_file_location(
        "make_rdt1b_golden", os.path.join(GOLDEN, "make_rdt1b_golden.py"))
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    g = np.load(os.path.join(GOLDEN, "rdt1b_small.npz"))
    x = gen.inputs()
    for k in ("lang", "img", "state", "noisy"):
        assert np.array_equal(x[k].numpy(), g[k])      # the seeded inputs regenerate exactly
    c = gen.CFG
    cfg = SimpleNamespace(hidden=c["hidden_size"], heads=c["num_heads"], num_layers=c["depth"],
                          ctrl_freq=int(g["freq"]))
    w = gen.weights()
    w["x_pos_embed"] = w["x_pos_embed"][0]
    w["lang_cond_pos_embed"] = w["lang_cond_pos_embed"][0]
    w["img_cond_pos_embed"] = w["img_cond_pos_embed"][0]
    m = RefRDT(w, cfg)
    with torch.no_grad():
        lang_c, img_c = m.encode(x["lang"], x["img"])
        lang_len = torch.tensor([x["lang"].shape[1]])
        out = m.forward(lang_c, img_c, lang_len, x["state"][:, 0], x["noisy"], int(g["t"]))
    assert out.shape == g["out"].shape
    np.testing.assert_allclose(out.numpy(), g["out"], rtol=0, atol=1e-5)
