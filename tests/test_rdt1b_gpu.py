"""GPU tests of the RDT-1B denoising runtime against the CPU oracle
(oracle/rdt1b_ref.py), at full width (hidden 2048, 32 heads) with 2 blocks and
shortened condition lengths so the fp32 CPU oracle stays fast.

Criteria: the reference's own alignment bar for a bf16 model
(tests/alignment/test_rdt1b_alignment.py:426): max |ours − oracle| < 0.05 and
cosine similarity > 0.9999.
"""
import numpy as np
import pytest
import torch

from oracle import rdt1b_ref
from servoflow_b200.rdt1b import RDT1B, default_config

pytestmark = pytest.mark.gpu


def close(ours, ref):
    a = ours.float().cpu().reshape(-1).double()
    b = ref.float().reshape(-1).double()
    max_abs = (a - b).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(a[None], b[None]).item()
    return max_abs, cos


@pytest.fixture(scope="module")
def setup(gpu):
    cfg = default_config(num_layers=2, max_lang_len=64, img_len=256, max_sessions=2)
    model = RDT1B(cfg, seed=1234)
    g = torch.Generator().manual_seed(42)
    B = 2
    lang = torch.randn(B, cfg.max_lang_len, cfg.lang_dim, generator=g).bfloat16()
    img = torch.randn(B, cfg.img_len, cfg.img_dim, generator=g).bfloat16()
    state = torch.randn(B, cfg.state_dim, generator=g).bfloat16()
    lens = torch.tensor([40, 64], dtype=torch.int32)
    noise = torch.randn(B, cfg.horizon, cfg.action_dim, generator=g)
    dev = gpu
    model.encode(lang.to(dev), lens.to(dev), img.to(dev), state.to(dev))
    torch.cuda.synchronize()
    ref = rdt1b_ref.RefRDT(rdt1b_ref.load_weights(model, cfg), cfg)
    lang_c, img_c = ref.encode(lang.float(), img.float())
    yield dict(cfg=cfg, model=model, ref=ref, lang=lang, img=img, state=state, lens=lens, noise=noise,
               lang_c=lang_c, img_c=img_c, dev=dev)
    model.close()


def test_single_network_evaluation(setup):
    s = setup
    out = torch.empty(2, s["cfg"].horizon, s["cfg"].action_dim, device=s["dev"])
    s["model"].forward(s["noise"].to(s["dev"]), 999.0, out)
    torch.cuda.synchronize()
    ref = s["ref"].forward(s["lang_c"], s["img_c"], s["lens"], s["state"].float(), s["noise"], 999)
    max_abs, cos = close(out, ref)
    assert max_abs < 0.05 and cos > 0.9999, (max_abs, cos)


def test_schedule_matches_oracle(setup):
    ts, a, b, c = setup["model"].schedule()
    rts, ra, rb, rc = rdt1b_ref.dpm_schedule(setup["cfg"].num_steps)
    assert ts == [float(t) for t in rts]
    for x, y in ((a, ra), (b, rb), (c, rc)):
        assert np.allclose(x, y, rtol=1e-6, atol=1e-7)


def test_sampling_graph_matches_oracle_and_replays(setup):
    s = setup
    noise = s["noise"].to(s["dev"])
    out1 = torch.empty_like(noise)
    out2 = torch.empty_like(noise)
    out3 = torch.empty_like(noise)
    s["model"].sample(noise, out1, use_graph=False)      # eager
    s["model"].sample(noise, out2, use_graph=True)       # eager first call, then capture
    s["model"].sample(noise, out3, use_graph=True)       # graph replay
    torch.cuda.synchronize()
    assert torch.equal(out1, out2) and torch.equal(out2, out3)
    ref = s["ref"].sample(s["lang_c"], s["img_c"], s["lens"], s["state"].float(), s["noise"])
    max_abs, cos = close(out3, ref)
    assert max_abs < 0.05 and cos > 0.9999, (max_abs, cos)


def test_masked_language_tokens_do_not_matter(setup):
    s = setup
    lang2 = s["lang"].clone()
    lang2[0, 40:] = torch.randn(24, s["cfg"].lang_dim).bfloat16() * 5    # beyond lang_len[0]
    m = s["model"]
    noise = s["noise"].to(s["dev"])
    a = torch.empty_like(noise)
    b = torch.empty_like(noise)
    m.forward(noise, 599.0, a)
    m.encode(lang2.to(s["dev"]), s["lens"].to(s["dev"]), s["img"].to(s["dev"]), s["state"].to(s["dev"]))
    m.forward(noise, 599.0, b)
    torch.cuda.synchronize()
    assert torch.equal(a[0], b[0])
    m.encode(s["lang"].to(s["dev"]), s["lens"].to(s["dev"]), s["img"].to(s["dev"]), s["state"].to(s["dev"]))
    torch.cuda.synchronize()


def test_sessions_are_independent(setup):
    # session 1's actions do not depend on session 0's inputs (same batch, same bits)
    s = setup
    m = s["model"]
    dev = s["dev"]
    noise = s["noise"].to(dev)
    a = torch.empty_like(noise)
    b = torch.empty_like(noise)
    m.sample(noise, a)
    lang2, img2, state2 = s["lang"].clone(), s["img"].clone(), s["state"].clone()
    g = torch.Generator().manual_seed(7)
    lang2[0] = torch.randn(lang2.shape[1:], generator=g).bfloat16()
    img2[0] = torch.randn(img2.shape[1:], generator=g).bfloat16()
    state2[0] = torch.randn(state2.shape[1:], generator=g).bfloat16()
    noise2 = noise.clone()
    noise2[0] = torch.randn(noise.shape[1:], generator=g).to(dev)
    m.encode(lang2.to(dev), s["lens"].to(dev), img2.to(dev), state2.to(dev))
    m.sample(noise2, b)
    torch.cuda.synchronize()
    assert torch.equal(a[1], b[1]) and not torch.equal(a[0], b[0])
    m.encode(s["lang"].to(dev), s["lens"].to(dev), s["img"].to(dev), s["state"].to(dev))
    torch.cuda.synchronize()


def test_api_errors(setup):
    """Bad arguments on a live model return statuses and leave it usable."""
    import ctypes
    from servoflow_b200 import _capi
    s = setup
    m, lib, dev = s["model"], s["model"].lib, s["dev"]
    cfg = s["cfg"]
    too_many = cfg.max_sessions + 1
    big = torch.zeros(too_many, cfg.horizon, cfg.action_dim, device=dev)
    out = torch.empty_like(big)
    sh = torch.cuda.current_stream().cuda_stream
    assert lib.sfb_rdt1b_forward(m.h, too_many, big.data_ptr(), 1.0, out.data_ptr(), sh) == _capi.SFB_ERR_SHAPE
    assert lib.sfb_rdt1b_sample(m.h, too_many, big.data_ptr(), out.data_ptr(), 1, sh) == _capi.SFB_ERR_SHAPE
    assert lib.sfb_rdt1b_sample(m.h, 0, big.data_ptr(), out.data_ptr(), 1, sh) == _capi.SFB_ERR_SHAPE
    assert lib.sfb_rdt1b_encode(m.h, too_many, big.data_ptr(), big.data_ptr(), big.data_ptr(),
                                big.data_ptr(), sh) == _capi.SFB_ERR_SHAPE
    p, n, dt = ctypes.c_void_p(), ctypes.c_int64(), ctypes.c_int32()
    assert lib.sfb_rdt1b_param(m.h, b"blocks.0.no_such.weight", ctypes.byref(p), ctypes.byref(n),
                               ctypes.byref(dt)) == _capi.SFB_ERR_INVALID
    assert lib.sfb_rdt1b_schedule(m.h, None, None, None, None, cfg.num_steps + 1) == _capi.SFB_ERR_INVALID
    # still usable
    noise = s["noise"].to(dev)
    y = torch.empty_like(noise)
    m.forward(noise, 999.0, y)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()


@pytest.fixture(scope="module")
def one(gpu):
    """One session (the persistent projection kernel's path) at full width,
    3 blocks (language, image, language), short conditions."""
    cfg = default_config(num_layers=3, max_lang_len=96, img_len=300, max_sessions=1)
    model = RDT1B(cfg, seed=4321)
    g = torch.Generator().manual_seed(44)
    lang = torch.randn(1, cfg.max_lang_len, cfg.lang_dim, generator=g).bfloat16()
    img = torch.randn(1, cfg.img_len, cfg.img_dim, generator=g).bfloat16()
    state = torch.randn(1, cfg.state_dim, generator=g).bfloat16()
    lens = torch.tensor([51], dtype=torch.int32)
    noise = torch.randn(1, cfg.horizon, cfg.action_dim, generator=g)
    model.encode(lang.to(gpu), lens.to(gpu), img.to(gpu), state.to(gpu))
    torch.cuda.synchronize()
    ref = rdt1b_ref.RefRDT(rdt1b_ref.load_weights(model, cfg), cfg)
    lang_c, img_c = ref.encode(lang.float(), img.float())
    yield dict(cfg=cfg, model=model, ref=ref, state=state, lens=lens, noise=noise, lang_c=lang_c,
               img_c=img_c, dev=gpu)
    model.close()


def test_one_session_paths_match_oracle(one):
    """Path 0 (persistent kernel: projections, self- and cross-attention as
    stages, norms folded in), path 1 (one kernel per projection) and path 2
    (persistent kernel between cross-attention kernels) all meet the bar
    against the oracle, and agree with each other."""
    s = one
    noise = s["noise"].to(s["dev"])
    outs = []
    for path in (0, 1, 2):
        s["model"].set_path(path)
        y = torch.empty_like(noise)
        s["model"].forward(noise, 999.0, y)
        torch.cuda.synchronize()
        outs.append(y)
    s["model"].set_path(0)
    ref = s["ref"].forward(s["lang_c"], s["img_c"], s["lens"], s["state"].float(), s["noise"], 999)
    for path, y in enumerate(outs):
        max_abs, cos = close(y, ref)
        print(f"[parity] one session, path {path}: max |d| {max_abs:.3e}, cos {cos:.7f}")
        assert max_abs < 0.05 and cos > 0.9999, (path, max_abs, cos)
    for y in outs[1:]:
        max_abs, cos = close(outs[0], y.cpu())
        assert max_abs < 0.05 and cos > 0.9999, (max_abs, cos)


def test_one_session_graph_replays_are_identical(one):
    s = one
    noise = s["noise"].to(s["dev"])
    eager, first, replay = (torch.empty_like(noise) for _ in range(3))
    s["model"].sample(noise, eager, use_graph=False)
    s["model"].sample(noise, first, use_graph=True)
    s["model"].sample(noise, replay, use_graph=True)
    torch.cuda.synchronize()
    assert torch.equal(eager, first) and torch.equal(first, replay)
    ref = s["ref"].sample(s["lang_c"], s["img_c"], s["lens"], s["state"].float(), s["noise"])
    max_abs, cos = close(replay, ref)
    assert max_abs < 0.05 and cos > 0.9999, (max_abs, cos)
    from servoflow_b200.backend import B200Backend
    assert B200Backend(0).device_error(reset=True) == 0


def test_profile_dense_reports_every_launch(one):
    """sfb_rdt1b_profile_dense: one entry per persistent-kernel launch of an
    evaluation, with positive bytes and durations, and the handle's path
    unchanged afterwards."""
    s = one
    s["model"].set_path(1)
    prof = s["model"].profile_dense(999.0)
    cfg = s["cfg"]
    stages = cfg.num_layers * 8 + 2                       # per block 8 stages, then the final layer's 2
    assert len(prof) == (stages + 47) // 48
    assert all(b > 0 and us > 0 for b, us in prof)
    # the weights alone: every block's int8 projections are read once
    D = cfg.hidden
    assert sum(b for b, _ in prof) > cfg.num_layers * 8 * D * D
    noise = s["noise"].to(s["dev"])
    y = torch.empty_like(noise)
    s["model"].forward(noise, 999.0, y)                   # still path 1: the per-projection kernels
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
    s["model"].set_path(0)


@pytest.mark.parametrize("lang_len", [1, 64, 96])
def test_one_session_persistent_kernel_language_lengths(gpu, lang_len):
    """The persistent kernel's cross-attention stage splits a head's valid
    keys over its cluster's four CTAs: one key (three CTAs with no tile), a
    length inside the first tile, and every key of the cache, each against
    the oracle (the image stage covers several tiles per CTA elsewhere)."""
    cfg = default_config(num_layers=2, max_lang_len=96, img_len=600, max_sessions=1)
    model = RDT1B(cfg, seed=99)
    try:
        g = torch.Generator().manual_seed(7 + lang_len)
        lang = torch.randn(1, cfg.max_lang_len, cfg.lang_dim, generator=g).bfloat16()
        img = torch.randn(1, cfg.img_len, cfg.img_dim, generator=g).bfloat16()
        state = torch.randn(1, cfg.state_dim, generator=g).bfloat16()
        lens = torch.tensor([lang_len], dtype=torch.int32)
        noise = torch.randn(1, cfg.horizon, cfg.action_dim, generator=g)
        model.encode(lang.to(gpu), lens.to(gpu), img.to(gpu), state.to(gpu))
        model.set_path(0)
        y = torch.empty(1, cfg.horizon, cfg.action_dim, device=gpu)
        model.forward(noise.to(gpu), 999.0, y)
        torch.cuda.synchronize()
        ref = rdt1b_ref.RefRDT(rdt1b_ref.load_weights(model, cfg), cfg)
        lang_c, img_c = ref.encode(lang.float(), img.float())
        r = ref.forward(lang_c, img_c, lens, state.float(), noise, 999)
        max_abs, cos = close(y, r)
        print(f"[parity] path 0, lang_len {lang_len}: max |d| {max_abs:.3e}, cos {cos:.7f}")
        assert max_abs < 0.05 and cos > 0.9999, (lang_len, max_abs, cos)
    finally:
        model.close()
