"""GPU tests of the control-tick engine (sfb_rdt1b_tick), the counterpart of
InferenceEngine::infer with its frame-id condition cache
(src/engine/inference_engine.cpp:90-174): conditions are re-encoded only when
the frame id changes, a cache hit reuses the K/V cache bit for bit, and the
per-tick path from pinned host buffers equals encode + sample on the device."""
import pytest
import torch

from servoflow_b200.rdt1b import RDT1B, default_config

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rig(gpu):
    cfg = default_config(num_layers=2, max_lang_len=64, img_len=256, max_sessions=1)
    model = RDT1B(cfg, seed=99)
    g = torch.Generator().manual_seed(7)
    host = dict(lang=torch.randn(1, cfg.max_lang_len, cfg.lang_dim, generator=g).bfloat16().pin_memory(),
                img=torch.randn(1, cfg.img_len, cfg.img_dim, generator=g).bfloat16().pin_memory(),
                lens=torch.tensor([40], dtype=torch.int32).pin_memory(),
                state=torch.randn(1, cfg.state_dim, generator=g).bfloat16().pin_memory(),
                noise=torch.randn(1, cfg.horizon, cfg.action_dim, generator=g).pin_memory())
    yield cfg, model, host, g
    model.close()


def reference_run(model, h, dev):
    """encode + sample on device copies: the path the tick must equal."""
    out = torch.empty(h["noise"].shape, device=dev)
    model.encode(h["lang"].to(dev), h["lens"].to(dev), h["img"].to(dev), h["state"].to(dev))
    model.sample(h["noise"].to(dev), out)
    torch.cuda.synchronize()
    return out.cpu()


def test_tick_cache_by_frame_id(rig, gpu):
    cfg, model, h, g = rig
    act = torch.empty(h["noise"].shape).pin_memory()
    model.invalidate_condition()
    t0, e0 = model.tick_stats()
    model.tick(1, h["state"], h["noise"], act, h["lang"], h["lens"], h["img"])
    torch.cuda.synchronize()
    a1 = act.clone()
    assert torch.isfinite(a1).all()
    # same frame: no re-encode, the cached K/V give the same actions bit for bit,
    # even though the caller's buffers now hold other data (the reference keys the
    # cache by frame id, not by pointer or content)
    old_lang = h["lang"].clone()
    h["lang"].copy_(torch.randn(h["lang"].shape, generator=g).bfloat16())
    model.tick(1, h["state"], h["noise"], act)
    torch.cuda.synchronize()
    assert torch.equal(act, a1)
    assert model.tick_stats() == (t0 + 2, e0 + 1)
    # a new frame re-encodes from the new buffers
    model.tick(2, h["state"], h["noise"], act, h["lang"], h["lens"], h["img"])
    torch.cuda.synchronize()
    a2 = act.clone()
    assert not torch.equal(a2, a1)
    assert model.tick_stats()[1] == e0 + 2
    assert torch.equal(a2, reference_run(model, h, gpu))
    # a new robot state counts on a cache hit too
    h2 = dict(h)
    h2["state"] = (h["state"].float() + 0.5).bfloat16().pin_memory()
    model.tick(2, h2["state"], h["noise"], act)
    torch.cuda.synchronize()
    assert not torch.equal(act, a2)
    assert torch.equal(act, reference_run(model, h2, gpu))
    # invalidation forces an encode on the same frame id
    model.invalidate_condition()
    h["lang"].copy_(old_lang)
    model.tick(2, h["state"], h["noise"], act, h["lang"], h["lens"], h["img"])
    torch.cuda.synchronize()
    assert torch.equal(act, a1)


def test_tick_errors(rig, gpu):
    from servoflow_b200 import _capi
    cfg, model, h, _ = rig
    act = torch.empty(h["noise"].shape).pin_memory()
    model.invalidate_condition()
    with pytest.raises(_capi.SfbError) as e:
        model.tick(3, h["state"], h["noise"], act)           # must encode, no conditions given
    assert e.value.status == _capi.SFB_ERR_INVALID
