"""GPU parity of the RDT-1B runtime at the headline configuration (config 4):
28 blocks, hidden 2048, 32 heads, language condition 1024 tokens with a short
valid length (masked keys), image condition 4374 tokens, batch 1, the 5-step
DPM-Solver++ sampler in one CUDA graph. The same check at the serving
configuration (config 5's batch of 32 sessions in one model), comparing the
first and the last session.

Oracle: oracle/rdt1b_ref.RefRDT in fp32 on the model's exact int8 weights
(q·s), the reference's own alignment model restated. Criteria: the
reference's bar for a bf16 model (tests/alignment/test_rdt1b_alignment.py:426):
max |ours − oracle| < 0.05 and cosine similarity > 0.9999.
"""
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


def inputs(cfg, B, seed, lens):
    g = torch.Generator().manual_seed(seed)
    lang = torch.randn(B, cfg.max_lang_len, cfg.lang_dim, generator=g).bfloat16()
    img = torch.randn(B, cfg.img_len, cfg.img_dim, generator=g).bfloat16()
    state = torch.randn(B, cfg.state_dim, generator=g).bfloat16()
    noise = torch.randn(B, cfg.horizon, cfg.action_dim, generator=g)
    return lang, img, state, torch.tensor(lens, dtype=torch.int32), noise


@pytest.fixture(scope="module")
def full(gpu):
    cfg = default_config(max_sessions=1)                 # 28 blocks, lang 1024, image 4374
    assert (cfg.num_layers, cfg.max_lang_len, cfg.img_len) == (28, 1024, 4374)
    model = RDT1B(cfg, seed=2024)
    lang, img, state, lens, noise = inputs(cfg, 1, 42, [37])
    model.encode(lang.to(gpu), lens.to(gpu), img.to(gpu), state.to(gpu))
    torch.cuda.synchronize()
    ref = rdt1b_ref.RefRDT(rdt1b_ref.load_weights(model, cfg), cfg)
    with torch.inference_mode():
        lang_c, img_c = ref.encode(lang.float(), img.float())
        kv = ref.cross_kv_all(lang_c, img_c)
    yield dict(cfg=cfg, model=model, ref=ref, kv=kv, lang_c=lang_c, img_c=img_c, lens=lens,
               state=state, noise=noise, dev=gpu)
    model.close()


@pytest.mark.parametrize("path", [1, 0])
def test_full_config_single_evaluation(full, path):
    """One evaluation on the per-projection path (1, the default) and on the
    persistent kernel with every attention as a stage (0)."""
    f = full
    out = torch.empty(1, f["cfg"].horizon, f["cfg"].action_dim, device=f["dev"])
    f["model"].set_path(path)
    try:
        f["model"].forward(f["noise"].to(f["dev"]), 999.0, out)
        torch.cuda.synchronize()
    finally:
        f["model"].set_path(1)
    with torch.inference_mode():
        ref = f["ref"].forward(f["lang_c"], f["img_c"], f["lens"], f["state"].float(), f["noise"], 999,
                               f["kv"])
    max_abs, cos = close(out, ref)
    print(f"[parity] config 4 forward t=999, path {path}: max |d| {max_abs:.3e}, cos {cos:.7f}")
    assert max_abs < 0.05 and cos > 0.9999, (max_abs, cos)


def test_full_config_sampling_graph(full):
    f = full
    noise = f["noise"].to(f["dev"])
    eager, first, replay = (torch.empty_like(noise) for _ in range(3))
    f["model"].sample(noise, eager, use_graph=False)
    f["model"].sample(noise, first, use_graph=True)      # eager first call, then capture
    f["model"].sample(noise, replay, use_graph=True)     # graph replay
    torch.cuda.synchronize()
    assert torch.equal(eager, first) and torch.equal(first, replay)
    with torch.inference_mode():
        ref = f["ref"].sample(f["lang_c"], f["img_c"], f["lens"], f["state"].float(), f["noise"], f["kv"])
    max_abs, cos = close(replay, ref)
    print(f"[parity] config 4 5-step graph: max |d| {max_abs:.3e}, cos {cos:.7f}")
    assert max_abs < 0.05 and cos > 0.9999, (max_abs, cos)


def test_serving_batch_first_and_last_session(gpu):
    """32 sessions in one model (config 5 per GPU), each with its own
    language length; sessions 0 and 31 against the oracle run on those two
    sessions alone."""
    cfg = default_config(max_sessions=32)
    model = RDT1B(cfg, seed=77)
    try:
        g = torch.Generator().manual_seed(5)
        lens = torch.randint(8, cfg.max_lang_len + 1, (32,), generator=g, dtype=torch.int32)
        lang, img, state, lens, noise = inputs(cfg, 32, 43, lens.tolist())
        model.encode(lang.to(gpu), lens.to(gpu), img.to(gpu), state.to(gpu))
        out = torch.empty(32, cfg.horizon, cfg.action_dim, device=gpu)
        model.sample(noise.to(gpu), out)
        torch.cuda.synchronize()
        ref = rdt1b_ref.RefRDT(rdt1b_ref.load_weights(model, cfg), cfg)
        pick = [0, 31]
        with torch.inference_mode():
            lang_c, img_c = ref.encode(lang[pick].float(), img[pick].float())
            r = ref.sample(lang_c, img_c, lens[pick], state[pick].float(), noise[pick])
        for i, s in enumerate(pick):
            max_abs, cos = close(out[s], r[i])
            print(f"[parity] config 5 session {s} (lang_len {int(lens[s])}): max |d| {max_abs:.3e}, cos {cos:.7f}")
            assert max_abs < 0.05 and cos > 0.9999, (s, max_abs, cos)
    finally:
        model.close()
