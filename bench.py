#!/usr/bin/env python3
"""Benchmark of the B200 RDT-1B denoising path (one JSON line on rank 0).

Headline workload (config 4): the full RDT-1B DiT denoise at batch 1 — 28
blocks, hidden 2048, 32 heads, int8 per-channel weights, self-attention over
the 67 action-chunk tokens, cross-attention alternating between the masked
language condition (1024 keys) and the image condition (4374 keys), 5
DPM-Solver++ steps replayed as one CUDA graph. One step = one full 5-step
denoise of one session's action chunk (64 x 128 fp32 noise) with the control
tick's condition K/V cache resident. The working set streamed per denoise
(7.9 GB of int8 weights and cached K/V) is ~60x the 126 MB L2, so no flush
is needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Reported beside the headline:
  e2e       the same denoise through the public call with host buffers:
            pinned host noise in, pinned host actions out, copies inside the
            timed region (RDT1B.sample_host -> sfb_rdt1b_sample).
  roofline  the dominant kernel, the int8-weight linear layer
            (w8a16_gemm_kernel): all 168 block projections of one network
            evaluation launched back to back through sfb_w8a16_linear with
            the model's weights (M = 67 tokens), algorithmic bytes
            (int8 W + scale + bias + X + Y [+ residual]) / event-timed
            duration per launch, against the measured HBM copy bandwidth.
  attention the image cross-attention kernel alone (config 2: Lq 67, Lk 4374),
            launched back to back over 8 distinct K/V caches (more than twice
            the L2, so every launch reads HBM), GB/s and TFLOP/s vs the peaks.
  cpu_baseline / --impl reference
            the CPU oracle of the same network (oracle/rdt1b_ref.py, torch
            fp32 on all host threads), each step one whole 5-step denoise.
            The reference has no CPU path (only its CUDA backend registers),
            so this restatement stands in.
  attention.configs.*.ref_naive_us / ref_fa2_us
            the reference's own CUDA attention on the same inputs: its naive
            kernel (ops/attention.cu:90-139, oracle/_ref/libsfref.so) and its
            FlashAttention-2 forward (oracle/_ref/libsfref_fa2.so), both
            built from the reference's sources for sm_100a.

Multi-GPU (torchrun, one process per GPU): each rank serves its own session
(own weights, K/V cache and graph) with no collective on the hot path (weak
scaling); the only collectives are barriers and the max over ranks of the
timings.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import sys
import time
from types import SimpleNamespace

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "RDT-1B denoise p50 latency (ms, B=1); attention TFLOP/s & GB/s vs B200 peak"
# RDT-1B shapes (reference config.h)
HIDDEN, HEADS, LAYERS, HORIZON, ACTION, LANG_LEN, IMG_LEN, STEPS = 2048, 32, 28, 64, 128, 1024, 4374, 5
TOKENS = HORIZON + 3


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def profiled_traffic(name):
    """DRAM bytes per launch from a committed ncu summary, if present."""
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", open(p).read())
    return float(m.group(1)) if m else None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML (read-only) every
    5 ms while the timed region runs."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.samples = []
        self.smax = None
        self._stop = None

    def _run(self):
        import pynvml
        h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
        self.smax = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        while not self._stop.is_set():
            try:
                sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                util = pynvml.nvmlDeviceGetUtilizationRates(h).gpu
                self.samples.append((float(sm), int(r), int(util)))
            except Exception:
                pass
            self._stop.wait(0.005)

    def __enter__(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            # NVML enumerates physical GPUs; map through CUDA_VISIBLE_DEVICES when set
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            if vis:
                ids = [x for x in vis.split(",") if x.strip()]
                if self.gpu < len(ids) and ids[self.gpu].strip().isdigit():
                    self.gpu = int(ids[self.gpu])
            self._stop = threading.Event()
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception:
            self._stop = None
        return self

    def __exit__(self, *exc):
        if self._stop is not None:
            self._stop.set()
            self._t.join(timeout=2)

    def summary(self):
        sm = [s for s, _, _ in self.samples]
        busy = [s for s, _, u in self.samples if u > 0] or sm
        reasons = sorted({n for _, r, _ in self.samples for n, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": float(np.median(busy)) if busy else None, "sm_max_mhz": self.smax,
                "reasons": reasons, "samples": len(sm), "source": "NVML, 5 ms polling"}


def dist_setup():
    from servoflow_b200.sessions import rank_env
    r = rank_env()
    return r.world, r.rank, r.local


# ── CPU oracle timing (cpu_baseline and --impl reference) ─────────────────────
class CpuDenoise:
    """The CPU oracle network (oracle/rdt1b_ref.py, fp32 torch) on the host
    cores, running the whole config-4 denoise each call: state adaptor,
    timestep/frequency embedders, all 28 blocks, final layer and the 5
    DPM-Solver++ updates, with the per-tick cross-attention K/V cache held
    (as the GPU runtime holds it). The reference has no CPU path (only its
    CUDA backend registers), so this restatement stands in for it."""

    def __init__(self, threads, seed=0):
        import torch
        from oracle.rdt1b_ref import RefRDT, random_weights
        self.torch = torch
        torch.set_num_threads(threads)
        self.threads = torch.get_num_threads()
        cfg = SimpleNamespace(hidden=HIDDEN, heads=HEADS, num_layers=LAYERS, action_dim=ACTION,
                              horizon=HORIZON, state_dim=ACTION, lang_dim=4096, img_dim=1152,
                              max_lang_len=LANG_LEN, img_len=IMG_LEN, num_steps=STEPS, ctrl_freq=25)
        self.ref = RefRDT(random_weights(cfg, seed=seed), cfg)
        g = torch.Generator().manual_seed(seed + 1)
        # the per-tick cache at the conditions' shapes (values do not matter for timing)
        self.kv = [(torch.randn(1, LANG_LEN if l % 2 == 0 else IMG_LEN, HIDDEN, generator=g),
                    torch.randn(1, LANG_LEN if l % 2 == 0 else IMG_LEN, HIDDEN, generator=g))
                   for l in range(LAYERS)]
        self.lang_len = torch.randint(8, LANG_LEN + 1, (1,), generator=g)
        self.state = torch.randn(1, ACTION, generator=g)
        self.noise = torch.randn(1, HORIZON, ACTION, generator=g)

    def denoise_ms(self):
        """One full 5-step denoise; milliseconds."""
        with self.torch.inference_mode():
            t0 = time.perf_counter()
            out = self.ref.sample(None, None, self.lang_len, self.state, self.noise, self.kv)
            ms = (time.perf_counter() - t0) * 1e3
        assert bool(self.torch.isfinite(out).all())
        return ms

    def sample_text(self, n):
        return (f"{n} full config-4 denoise(s) (28 blocks x 5 DPM-Solver++ steps, adaptors, embedders, "
                f"final layer; cross K/V cached), fp32 torch on {self.threads} threads, oracle/rdt1b_ref.py")

    def baseline(self, budget_s):
        """cpu_baseline object: full denoises until the time budget is spent (at least one)."""
        ts = []
        t_end = time.perf_counter() + budget_s
        while time.perf_counter() < t_end or not ts:
            ts.append(self.denoise_ms())
        return {"value": float(np.median(ts)), "unit": "ms", "cores": self.threads, "kind": "port",
                "sample": self.sample_text(len(ts))}


def run_reference(args, world, rank):
    """The CPU oracle of the whole denoise on the host CPU, rank 0 only: each
    step is one full config-4 denoise. Steps stop early once the time budget
    is spent; steps_measured says how many ran."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    s = CpuDenoise(threads)
    budget = 240.0                                  # seconds for warm-up + timed steps
    t_start = time.perf_counter()
    for _ in range(min(args.warmup, 1)):            # one warm-up denoise (each is a full pass)
        s.denoise_ms()
    ts = []
    for _ in range(args.steps):
        if ts and time.perf_counter() - t_start > budget:
            break
        ts.append(s.denoise_ms())
    p50 = float(np.median(ts))
    line = {
        "impl": "reference", "metric": METRIC, "value": p50, "unit": "ms", "n_gpus": world,
        "steps": args.steps, "steps_measured": len(ts), "warmup": min(args.warmup, 1),
        "ms_per_step": float(np.mean(ts)), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic, seeded",
        "config": {"workload": "config 4: full RDT-1B denoise, B=1 session per GPU, 28 blocks, hidden "
                               "2048, 32 heads, lang 1024 (masked) / image 4374 cross-attention, "
                               "5 DPM-Solver++ steps, condition K/V cache resident",
                   "global_batch": 1, "seq_len": TOKENS,
                   "parallelism": f"host CPU, torch fp32, {s.threads} threads"},
        "cpu_baseline": {"value": p50, "unit": "ms", "cores": s.threads, "kind": "port",
                         "sample": s.sample_text(len(ts)) + " per step"},
        "e2e": {"value": p50, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ── GPU arm ───────────────────────────────────────────────────────────────────
def block_gemms(model):
    """(name, N, K, act, has_residual) of the 168 block projections of one
    network evaluation, in launch order."""
    out = []
    for l in range(LAYERS):
        p = f"blocks.{l}."
        out += [(p + "attn.qkv", 3 * HIDDEN, HIDDEN, 0, False), (p + "attn.proj", HIDDEN, HIDDEN, 0, True),
                (p + "cross_attn.q", HIDDEN, HIDDEN, 0, False),
                (p + "cross_attn.proj", HIDDEN, HIDDEN, 0, True),
                (p + "ffn.fc1", HIDDEN, HIDDEN, 1, False), (p + "ffn.fc2", HIDDEN, HIDDEN, 0, True)]
    return out


def gemm_roofline(model, dev, reps):
    """Event-timed duration per launch of the block projections, launched back
    to back through the C ABI with the model's weights (HBM-resident, 0.96 GB
    per pass, so every launch streams its weights from HBM)."""
    import torch
    from servoflow_b200 import _capi
    capi = _capi.lib()
    M = TOKENS
    g = torch.Generator().manual_seed(7)
    x = (torch.randn(M, HIDDEN, generator=g) * 0.5).bfloat16().to(dev)
    res = (torch.randn(M, HIDDEN, generator=g) * 0.5).bfloat16().to(dev)
    y = torch.empty(M, 3 * HIDDEN, dtype=torch.bfloat16, device=dev)
    sh = torch.cuda.current_stream().cuda_stream
    calls, nbytes = [], 0
    for name, N, K, act, has_res in block_gemms(model):
        wq = model.param_ptr(name + ".weight_q")[0]
        ws = model.param_ptr(name + ".weight_scale")[0]
        wb = model.param_ptr(name + ".bias")[0]
        calls.append((wq, ws, wb, res.data_ptr() if has_res else None, N, K, act))
        nbytes += N * K + N * 4 + N * 2 + M * K * 2 + M * N * 2 + (M * N * 2 if has_res else 0)

    def run():
        for wq, ws, wb, rp, N, K, act in calls:
            rc = capi.sfb_w8a16_linear(x.data_ptr(), K, wq, ws, wb, rp, HIDDEN if rp else 0,
                                       y.data_ptr(), N, 2, M, N, K, act, 0, sh)
            if rc:
                raise _capi.SfbError(rc, "w8a16_linear")

    run()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(); run(); e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e-3)
    per_launch = float(np.median(ts)) / len(calls)
    return nbytes / len(calls), per_launch, len(calls) * (reps + 1)


def attention_roofline(be, dev, reps, sets=8):
    """Image cross-attention (config 2) alone: `reps` launches back to back,
    rotating over `sets` distinct K/V caches (8 x 35.8 MB, > 2x the L2), so
    every launch streams its K/V from HBM; event-timed per batch."""
    import ctypes
    import torch
    from servoflow_b200 import _capi
    from servoflow_b200.backend import attention_args
    capi = _capi.lib()
    g = torch.Generator().manual_seed(11)
    q = torch.randn(1, HEADS, TOKENS, 64, generator=g).bfloat16().to(dev)
    # the K/V cache as the model stores it: K bf16, V fp16 (sfb_attn_args.v_dtype)
    kv = [(torch.randn(1, HEADS, IMG_LEN, 64, generator=g).bfloat16().to(dev),
           torch.randn(1, HEADS, IMG_LEN, 64, generator=g).half().to(dev)) for _ in range(sets)]
    out = torch.empty_like(q)
    cargs = [attention_args(q, k, v, out) for k, v in kv]
    pargs = [ctypes.byref(a) for a in cargs]
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream

    def run(n):
        for i in range(n):
            _capi.check(capi.sfb_attention_fwd(pargs[i % sets], sh), "attention")

    run(2 * sets)
    torch.cuda.synchronize()
    per = []
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream); run(reps); e1.record(stream)
        torch.cuda.synchronize()
        per.append(e0.elapsed_time(e1) / reps)
    nbytes = 2 * (2 * HEADS * TOKENS * 64 + 2 * HEADS * IMG_LEN * 64)
    flops = 4.0 * HEADS * TOKENS * IMG_LEN * 64
    return nbytes, flops, float(np.median(per)), float(np.min(per)), 5 * reps + 2 * sets


def attention_batched(dev, sessions=32, reps=10):
    """The image cross-attention of the serving configuration: `sessions`
    sessions' K/V caches (32 x 35.8 MB = 1.15 GB, ~9x the L2) in one launch,
    so every launch streams its K/V from HBM. Returns (algorithmic bytes,
    median ms per launch)."""
    import ctypes
    import torch
    from servoflow_b200 import _capi
    from servoflow_b200.backend import attention_args
    capi = _capi.lib()
    g = torch.Generator().manual_seed(12)
    q = torch.randn(sessions, HEADS, TOKENS, 64, generator=g).bfloat16().to(dev)
    k = torch.randn(sessions, HEADS, IMG_LEN, 64, generator=g).bfloat16().to(dev)
    v = torch.randn(sessions, HEADS, IMG_LEN, 64, generator=g).half().to(dev)
    out = torch.empty_like(q)
    a = attention_args(q, k, v, out)
    stream = torch.cuda.current_stream()
    for _ in range(3):
        _capi.check(capi.sfb_attention_fwd(ctypes.byref(a), stream.cuda_stream), "attention")
    torch.cuda.synchronize()
    per = []
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            capi.sfb_attention_fwd(ctypes.byref(a), stream.cuda_stream)
        e1.record(stream)
        torch.cuda.synchronize()
        per.append(e0.elapsed_time(e1) / reps)
    nbytes = 2 * sessions * (2 * HEADS * TOKENS * 64 + 2 * HEADS * IMG_LEN * 64)
    del q, k, v, out
    return nbytes, float(np.median(per))


def serving(dev, rank, batches, sessions=32):
    """Config 5 on this GPU: `sessions` independent robot sessions batched in one
    model (M = 32 · 67 tokens per projection), full 5-step denoise per batch;
    returns per-batch device latencies (ms)."""
    import torch
    from servoflow_b200.rdt1b import RDT1B, default_config
    from servoflow_b200.sessions import rank_env, session_ids, session_seed
    first = session_ids(rank_env().world, rank, sessions).start     # this rank's global sessions
    model = RDT1B(default_config(max_sessions=sessions), seed=session_seed(first, "serving"))
    g = torch.Generator().manual_seed(session_seed(first, "serving") + 100000)
    lang = torch.randn(sessions, LANG_LEN, 4096, generator=g).bfloat16().to(dev)
    lens = torch.randint(8, LANG_LEN + 1, (sessions,), generator=g, dtype=torch.int32).to(dev)
    img = torch.randn(sessions, IMG_LEN, 1152, generator=g).bfloat16().to(dev)
    state = torch.randn(sessions, 128, generator=g).bfloat16().to(dev)
    noise = torch.randn(sessions, HORIZON, ACTION, generator=g).to(dev)
    actions = torch.empty_like(noise)
    model.encode(lang, lens, img, state)
    del lang, img
    for _ in range(3):
        model.sample(noise, actions)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    st = [torch.cuda.Event(enable_timing=True) for _ in range(batches)]
    en = [torch.cuda.Event(enable_timing=True) for _ in range(batches)]
    for i in range(batches):
        st[i].record(stream)
        model.sample(noise, actions)
        en[i].record(stream)
    torch.cuda.synchronize()
    assert torch.isfinite(actions).all()
    ms = [a.elapsed_time(b) for a, b in zip(st, en)]
    model.close()
    return ms


def attention_configs(dev, reps=50):
    """Configs 1-3 of the attention path through the C ABI, each warm (back to
    back, same inputs) and cold (a 256 MB buffer, twice the L2, written between
    launches; only the attention launch is timed). Config 1: self-attention,
    B=1, H=32, Lq=Lk=67, fp32 (and bf16). Config 2: image cross-attention, B=1,
    Lk=4374, bf16. Config 3: masked language cross-attention, B=16, Lk padded
    to 1024, valid lengths L_b ~ U[8, 1024] (seeded), bf16; its bytes count
    valid keys only. Beside ours, on the same inputs: the reference's own CUDA
    attention, its naive kernel (every dtype) and its FlashAttention-2 (bf16),
    which ignore the mask (attention.cu:30) and so run config 3 over all 1024
    keys. Returns {name: {alg_bytes, flops, warm_us, cold_us, ref_naive_*,
    ref_fa2_*}}."""
    import ctypes
    import torch
    from oracle import oracle
    from servoflow_b200 import _capi
    from servoflow_b200.backend import attention_args
    capi = _capi.lib()
    naive = oracle.ref_lib()
    fa2 = oracle.ref_fa2_lib()
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    g = torch.Generator().manual_seed(13)
    out = {}

    def measure(launch):
        for _ in range(5):
            launch()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            launch()
        e1.record(stream)
        torch.cuda.synchronize()
        warm = e0.elapsed_time(e1) / reps * 1e3
        st = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
        en = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
        for i in range(reps):
            flush.fill_(i & 0xff)
            st[i].record(stream)
            launch()
            en[i].record(stream)
        torch.cuda.synchronize()
        cold = float(np.median([x.elapsed_time(y) for x, y in zip(st, en)])) * 1e3
        return warm, cold

    def ours(a):
        pa = ctypes.byref(a)
        return lambda: _capi.check(capi.sfb_attention_fwd(pa, sh), "attention")

    def refs(q, k, v, o, entry):
        B, H, Lq, D = q.shape
        Lk = k.shape[2]
        code = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[q.dtype]
        if naive is not None:
            fn = lambda: naive.sfref_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                               code, B, H, Lq, Lk, D, 0.0, 0, sh)
            entry["ref_naive_warm_us"], entry["ref_naive_cold_us"] = measure(fn)
        if fa2 is not None and code != 0:
            ws = torch.empty(fa2.sfref_fa2_workspace_bytes(B, H, Lq), dtype=torch.uint8, device=dev)
            fn = lambda: fa2.sfref_fa2_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                                 code, B, H, Lq, Lk, D, 0.0, 0, ws.data_ptr(), ws.numel(), sh)
            entry["ref_fa2_warm_us"], entry["ref_fa2_cold_us"] = measure(fn)

    for name, dt, Lk in (("config1_self_fp32", torch.float32, TOKENS), ("config1_self_bf16", torch.bfloat16, TOKENS),
                         ("config2_image_bf16", torch.bfloat16, IMG_LEN)):
        q = torch.randn(1, HEADS, TOKENS, 64, generator=g).to(dt).to(dev)
        k, v = (torch.randn(1, HEADS, Lk, 64, generator=g).to(dt).to(dev) for _ in range(2))
        o = torch.empty_like(q)
        es = q.element_size()
        e = {"alg_bytes": 2 * HEADS * (TOKENS + Lk) * 64 * es, "flops": 4.0 * HEADS * TOKENS * Lk * 64}
        e["warm_us"], e["cold_us"] = measure(ours(attention_args(q, k, v, o)))
        refs(q, k, v, torch.empty_like(q), e)
        out[name] = e
    B3 = 16
    lens = torch.randint(8, LANG_LEN + 1, (B3,), generator=g, dtype=torch.int32)
    q = torch.randn(B3, HEADS, TOKENS, 64, generator=g).bfloat16().to(dev)
    k = torch.randn(B3, HEADS, LANG_LEN, 64, generator=g).bfloat16().to(dev)
    v = torch.randn(B3, HEADS, LANG_LEN, 64, generator=g).bfloat16().to(dev)
    o = torch.empty_like(q)
    sl = int(lens.sum())
    e = {"alg_bytes": 2 * B3 * HEADS * TOKENS * 64 * 2 + 2 * HEADS * 64 * 2 * sl,
         "flops": 4.0 * HEADS * TOKENS * 64 * sl}
    e["warm_us"], e["cold_us"] = measure(ours(attention_args(q, k, v, o, mask=lens.to(dev))))
    refs(q, k, v, torch.empty_like(q), e)
    out["config3_lang_masked_b16"] = e
    del flush
    return out


def octo_leg(dev, reps=50):
    """The Octo row: Octo-Small at the reference's defaults (12 blocks, hidden
    384, 64 tokens; diffusion head; 10 flow-matching steps), one session.
    Returns device-timed medians (ms): encode (backbone + readout), sample
    (one graph), sample from pinned host noise to host actions, and the
    sampling graph's kernel count."""
    import torch
    from servoflow_b200.octo import Octo, default_config
    from servoflow_b200.sessions import session_seed
    model = Octo(default_config(), seed=session_seed(0, "weights"))
    g = torch.Generator().manual_seed(4242)
    tokens = torch.randn(1, 64, 384, generator=g).bfloat16().to(dev)
    noise_h = torch.randn(1, 4, 7, generator=g).pin_memory()
    act_h = torch.empty_like(noise_h).pin_memory()
    noise = noise_h.to(dev)
    act = torch.empty_like(noise)
    stream = torch.cuda.current_stream()

    def timed(fn):
        for _ in range(3):
            fn()
        st = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
        en = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
        for i in range(reps):
            st[i].record(stream)
            fn()
            en[i].record(stream)
        torch.cuda.synchronize()
        return float(np.median([a.elapsed_time(b) for a, b in zip(st, en)]))

    enc = timed(lambda: model.encode(tokens))
    smp = timed(lambda: model.sample(noise, act))
    smp_h = timed(lambda: model.sample(noise_h, act_h))
    assert torch.isfinite(act).all() and torch.equal(act.cpu(), act_h)
    kernels = model.graph_kernels(1)
    model.close()
    return enc, smp, smp_h, kernels


def octo_cpu(threads: int, reps: int = 3):
    """The same two calls on the CPU oracle (fp32 torch, `threads` threads):
    median ms of encode and of a 10-step sample."""
    import time
    import torch
    from oracle import octo_ref
    from servoflow_b200.octo import default_config
    torch.set_num_threads(threads)
    cfg = default_config()
    ref = octo_ref.RefOcto(octo_ref.random_weights(cfg, seed=1), cfg)
    tokens, noise = torch.randn(1, 64, 384), torch.randn(1, 4, 7)
    enc, smp = [], []
    with torch.no_grad():
        for _ in range(reps):
            t0 = time.perf_counter(); _, cond = ref.encode(tokens); enc.append(time.perf_counter() - t0)
            t0 = time.perf_counter(); ref.sample(noise, cond); smp.append(time.perf_counter() - t0)
    return float(np.median(enc)) * 1e3, float(np.median(smp)) * 1e3


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-serving", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup()

    if args.impl == "reference":
        run_reference(args, world, rank)
        return

    import torch
    import torch.distributed as dist
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())

    from servoflow_b200 import build
    build.build_library()
    from servoflow_b200.backend import B200Backend
    from servoflow_b200.rdt1b import RDT1B, default_config
    be = B200Backend(dev.index)

    # one robot session per GPU: its own weights, condition and noise (seeded by session)
    from servoflow_b200.sessions import barrier, max_over_ranks, session_ids, session_seed
    sid = session_ids(world, rank, 1)[0]
    model = RDT1B(default_config(max_sessions=1), seed=session_seed(sid, "weights"))
    g = torch.Generator().manual_seed(session_seed(sid, "inputs"))
    lang = torch.randn(1, LANG_LEN, 4096, generator=g).bfloat16().to(dev)
    lang_len = torch.randint(8, LANG_LEN + 1, (1,), generator=g, dtype=torch.int32).to(dev)
    img = torch.randn(1, IMG_LEN, 1152, generator=g).bfloat16().to(dev)
    state = torch.randn(1, 128, generator=g).bfloat16().to(dev)
    noise_h = torch.randn(1, HORIZON, ACTION, generator=g).pin_memory()
    act_h = torch.empty_like(noise_h).pin_memory()
    noise = noise_h.to(dev)
    actions = torch.empty_like(noise)
    stream = torch.cuda.current_stream()

    model.encode(lang, lang_len, img, state)
    for _ in range(args.warmup):                       # the first call captures the graph
        model.sample(noise, actions)
    torch.cuda.synchronize()
    assert be.device_error() == 0
    kernels_per_step = model.graph_kernels(1)

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    sampler = ClockSampler(dev.index)
    with sampler:
        barrier()
        torch.cuda.synchronize()
        t_wall = time.perf_counter()
        for i in range(args.steps):
            starts[i].record(stream)
            model.sample(noise, actions)
            ends[i].record(stream)
        torch.cuda.synchronize()
        barrier()
        t_wall = time.perf_counter() - t_wall

        # end to end through the public call: pinned host noise in, host actions out
        for _ in range(3):
            model.sample_host(noise_h, act_h)
        torch.cuda.synchronize()
        e_st = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        e_en = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        for i in range(args.steps):
            e_st[i].record(stream)
            model.sample_host(noise_h, act_h)
            e_en[i].record(stream)
        torch.cuda.synchronize()

        # control ticks through sfb_rdt1b_tick from pinned host buffers: a new
        # camera frame every tick (conditions copied in, adaptors + 28 cross K/V
        # projections, denoise, actions out) and the same frame (state + noise in,
        # cached K/V, denoise, actions out)
        lang_h, img_h = lang.cpu().pin_memory(), img.cpu().pin_memory()
        lens_h, state_h = lang_len.cpu().pin_memory(), state.cpu().pin_memory()
        n_tick = min(args.steps, 20)
        frame = 1 << 40

        def ticks(new_frame):
            nonlocal frame
            st = [torch.cuda.Event(enable_timing=True) for _ in range(n_tick)]
            en = [torch.cuda.Event(enable_timing=True) for _ in range(n_tick)]
            for i in range(3 + n_tick):
                if new_frame or i == 0:
                    frame += 1
                if i >= 3:
                    st[i - 3].record(stream)
                model.tick(frame, state_h, noise_h, act_h, lang_h, lens_h, img_h)
                if i >= 3:
                    en[i - 3].record(stream)
            torch.cuda.synchronize()
            return np.array([a.elapsed_time(b) for a, b in zip(st, en)])

        tick_new_ms = ticks(True)
        tick_same_ms = ticks(False)
        tick_h2d_new = sum(t.numel() * t.element_size() for t in (lang_h, img_h, lens_h, state_h, noise_h))
        tick_h2d_same = state_h.numel() * state_h.element_size() + noise_h.numel() * 4
    assert be.device_error() == 0
    assert torch.isfinite(act_h).all()

    gemm_bytes, gemm_s, gemm_launches = gemm_roofline(model, dev, reps=5)
    serve_ms = [0.0] if args.no_serving else serving(dev, rank, batches=max(3, min(args.steps, 10)))
    at_bytes, at_flops, at_med, at_min, at_launches = attention_roofline(be, dev, reps=64)
    atb_bytes, atb_ms = attention_batched(dev)
    oc_enc, oc_smp, oc_smp_h, oc_kernels = octo_leg(dev)
    acfg = attention_configs(dev)
    assert be.device_error() == 0

    ms = np.array([s.elapsed_time(e) for s, e in zip(starts, ends)])
    e2e_ms = np.array([s.elapsed_time(e) for s, e in zip(e_st, e_en)])
    stats = max_over_ranks([np.median(ms), np.mean(ms), np.percentile(ms, 99), np.median(e2e_ms),
                            np.median(tick_new_ms), np.median(tick_same_ms), gemm_s, at_med, at_min,
                            np.median(serve_ms), np.percentile(serve_ms, 99), atb_ms, oc_enc, oc_smp,
                            oc_smp_h], device=dev)
    (p50, mean, p99, e2e_p50, tick_new_p50, tick_same_p50, gemm_s, at_med, at_min, sv_p50, sv_p99, atb_ms,
     oc_enc, oc_smp, oc_smp_h) = stats

    if rank == 0:
        hbm, tflops, kind = peaks()
        gemm_gbs = gemm_bytes / gemm_s / 1e9
        at_gbs = at_bytes / (at_med * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": p50, "unit": "ms", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": mean, "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: random-init int8 weights, N(0,1) conditions and noise, seeded per session",
            "config": {"workload": "config 4: full RDT-1B denoise, B=1 session per GPU, 28 blocks, hidden "
                                   "2048, 32 heads, lang 1024 (masked) / image 4374 cross-attention, "
                                   "5 DPM-Solver++ steps in one CUDA graph, condition K/V cache resident",
                       "global_batch": world, "seq_len": TOKENS,
                       "l2": "not flushed: each denoise streams 7.9 GB (int8 weights + cached K/V), "
                             "~60x the 126 MB L2",
                       "parallelism": f"{world} independent session(s), one per GPU, no collective"},
            "p99_ms": p99,
            "throughput": {"value": world * 1e3 / mean, "unit": "denoises/s (all GPUs)",
                           "actions_per_s": world * 1e3 / mean * HORIZON},
            "tick_e2e": {"new_frame_ms": tick_new_p50, "same_frame_ms": tick_same_p50,
                         "h2d_bytes_new_frame": tick_h2d_new, "h2d_bytes_same_frame": tick_h2d_same,
                         "d2h_bytes": act_h.numel() * 4,
                         "what": "RDT1B.tick -> sfb_rdt1b_tick from pinned host buffers, copies inside the "
                                 "timed region; new frame: conditions copied in, adaptors + 28 cross K/V "
                                 "projections on the encode stream, denoise graph, actions out; same "
                                 "frame: state + noise in, cached K/V, denoise, actions out"},
            "roofline": {"bound": "hbm", "achieved": gemm_gbs, "peak": hbm, "unit": "GB/s",
                         "frac": gemm_gbs / hbm,
                         "traffic": profiled_traffic("w8a16_gemm_rdt1b_block.md"),
                         "peak_kind": f"{kind} (MEASURED_PEAKS.json hbm_gbs, burst copy)",
                         "kernel": "w8a16_gemm_kernel (int8-weight linear), dominant by time",
                         "alg_bytes_per_launch": gemm_bytes, "us_per_launch": gemm_s * 1e6,
                         "how": "168 block projections (M=67) back to back via sfb_w8a16_linear, "
                                "model weights, CUDA events, max over ranks"},
            "attention": {"kernel": "attn_fwd_tc_kernel<bf16>, image cross-attention (config 2), "
                                    "bf16 Q/K, fp16 V cache",
                          "us_per_launch": at_med * 1e3, "best_batch_us_per_launch": at_min * 1e3,
                          "achieved_gbs": at_gbs, "frac_hbm": at_gbs / hbm,
                          "tflops": at_flops / (at_med * 1e-3) / 1e12,
                          "frac_tensor": at_flops / (at_med * 1e-3) / 1e12 / tflops,
                          "alg_bytes_per_launch": at_bytes,
                          "traffic": profiled_traffic("attn_fwd_tc_image_xattn.md"),
                          "l2": "64 launches back to back over 8 distinct K/V caches (286 MB > 2x L2): "
                                "every launch reads its K/V from HBM; median of 5 batches",
                          "launch": "sfb_attention_fwd, programmatic dependent launch: a launch's "
                                    "barrier/TMEM setup overlaps the previous launch's tail",
                          "serving_32_sessions": {
                              "what": "the serving configuration's image cross-attention: 32 sessions in one "
                                      "launch, K/V 1.15 GB (~9x L2), streamed from HBM every launch",
                              "us_per_launch": atb_ms * 1e3,
                              "achieved_gbs": atb_bytes / (atb_ms * 1e-3) / 1e9,
                              "frac_hbm": atb_bytes / (atb_ms * 1e-3) / 1e9 / hbm,
                              "alg_bytes_per_launch": atb_bytes},
                          "configs": {n: dict(e, cold_gbs=e["alg_bytes"] / (e["cold_us"] * 1e-6) / 1e9,
                                              cold_frac_hbm=e["alg_bytes"] / (e["cold_us"] * 1e-6) / 1e9 / hbm,
                                              cold_tflops=e["flops"] / (e["cold_us"] * 1e-6) / 1e12,
                                              **({"speedup_vs_ref_fa2_cold": e["ref_fa2_cold_us"] / e["cold_us"]}
                                                 if "ref_fa2_cold_us" in e else {}),
                                              **({"speedup_vs_ref_naive_cold": e["ref_naive_cold_us"] / e["cold_us"]}
                                                 if "ref_naive_cold_us" in e else {}))
                                      for n, e in acfg.items()},
                          "configs_note": "rank 0's device times (CUDA events); cold = a 256 MB "
                                          "buffer written before each launch, warm = back to back; "
                                          "config 3 bytes over valid keys only; ref_naive / ref_fa2 = "
                                          "the reference's own CUDA attention (naive kernel, "
                                          "FlashAttention-2) built from its sources for sm_100a, same "
                                          "inputs (config 3 unmasked: the reference drops masks)"},
            "e2e": {"value": e2e_p50, "unit": "ms", "h2d_bytes_per_step": noise_h.numel() * 4,
                    "d2h_bytes_per_step": act_h.numel() * 4,
                    "path": "RDT1B.sample_host -> sfb_rdt1b_sample: pinned host noise -> device, "
                            "graph replay, actions -> pinned host, all inside the timed region"},
            "serving": None if args.no_serving else {
                "what": "config 5: 32 independent sessions per GPU batched in one model, full 5-step "
                        "denoise per batch (graph), sharded by session, no collective",
                "sessions_per_gpu": 32, "sessions_total": 32 * world,
                "batch_p50_ms": sv_p50, "batch_p99_ms": sv_p99,
                "per_session_p99_ms": sv_p99,
                "actions_per_s": world * 32 * HORIZON * 1e3 / sv_p50,
                "chunks_per_s": world * 32 * 1e3 / sv_p50},
            "octo": {"what": "Octo-Small at the reference's defaults (12 pre-LN blocks, hidden 384, "
                             "6 heads, 64 tokens; MLP diffusion head; 10 flow-matching Euler steps in "
                             "one CUDA graph), one session per GPU",
                     "encode_ms": oc_enc, "sample_ms": oc_smp, "sample_host_ms": oc_smp_h,
                     "sample_graph_kernels": oc_kernels,
                     "path": "Octo.encode / Octo.sample -> sfb_octo_encode / sfb_octo_sample; "
                             "sample_host_ms copies pinned host noise in and actions out inside the "
                             "timed region"},
            "gpu_launches": kernels_per_step * args.steps * world,
            "gpu_launches_note": f"{kernels_per_step} kernels per denoise graph x {args.steps} timed steps "
                                 f"x {world} GPU(s) "
                                 f"(counted from the captured graph's kernel nodes); the e2e, tick and "
                                 f"roofline passes add more",
            "clocks": sampler.summary(),
            "wall_s_device_loop": t_wall,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = CpuDenoise(os.cpu_count() or 1).baseline(15.0)
            ce, cs = octo_cpu(os.cpu_count() or 1)
            line["octo"]["cpu_oracle"] = {"encode_ms": ce, "sample_ms": cs, "cores": os.cpu_count() or 1,
                                          "kind": "port", "what": "oracle/octo_ref.py, fp32 torch"}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
