"""GPU parity tests of the fused int8-weight linear layer (sfb_w8a16_linear)
against the oracle: dequantise-then-GEMM in double precision
(oracle/sfo_oracle.c: sfo_w8a16_linear).

Tolerance: the kernel accumulates exact fp32 products in fp32 and rounds the
result once to bf16, so |ours − oracle| <= 1 bf16 ulp of |oracle| + 1e-6·K·max|x||q|s
(the fp32 summation term is far below the ulp for these sizes); fp32 output:
relative 1e-4."""
import numpy as np
import pytest
import torch

from oracle import oracle
from servoflow_b200.backend import B200Backend

pytestmark = pytest.mark.gpu


def ulp_bf16(x):
    ax = np.maximum(np.abs(x), 2.0 ** -126)
    return np.exp2(np.floor(np.log2(ax)) - 7)


def make(M, N, K, seed, dev, bias=True, residual=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).bfloat16()
    wf = torch.randn(N, K, generator=g) * 0.02
    s = wf.abs().amax(dim=1) / 127.0                       # symmetric per output channel
    q = torch.round(wf / s[:, None]).clamp(-127, 127).to(torch.int8)
    b = (torch.randn(N, generator=g) * 0.1).bfloat16() if bias else None
    r = torch.randn(M, N, generator=g).bfloat16() if residual else None
    to = lambda t: None if t is None else t.to(dev)
    return x.to(dev), q.to(dev), s.float().to(dev), to(b), to(r)


def check(be, M, N, K, seed, dev, act="none", bias=True, residual=False, splits=0, f32=False):
    x, q, s, b, r = make(M, N, K, seed, dev, bias, residual)
    if f32 and r is not None:
        r = (r.float() + 1e-3).contiguous()             # the residual has the output's dtype
    y = torch.empty(M, N, dtype=torch.float32 if f32 else torch.bfloat16, device=dev)
    be.w8a16_linear(x, q, s, y, bias=b, residual=r, act=act, num_splits=splits)
    torch.cuda.synchronize()
    ref = oracle.w8a16_linear(x.float().cpu().numpy(), q.cpu().numpy(), s.cpu().numpy(),
                              None if b is None else b.float().cpu().numpy(),
                              None if r is None else r.float().cpu().numpy(),
                              act={"none": 0, "gelu": 1, "silu": 2}[act])
    out = y.float().cpu().numpy()
    if f32:
        tol = 1e-4 * np.maximum(np.abs(ref), 1.0)
    else:
        tol = ulp_bf16(ref) + 1e-4
    err = np.abs(out - ref)
    assert not np.isnan(out).any()
    assert (err <= tol).all(), f"max err {err.max():.3e} (ref {ref.flat[err.argmax()]:.4f})"


@pytest.fixture(scope="module")
def be(gpu):
    b = B200Backend(0)
    b.device_error(reset=True)
    yield b
    assert b.device_error(reset=True) == 0


# RDT-1B projection shapes at one denoising step (67 tokens)
@pytest.mark.parametrize("N", [2048, 4096, 6144])
def test_rdt_step_shapes(be, gpu, N):
    check(be, 67, N, 2048, N, gpu)


def test_gelu_and_residual(be, gpu):
    check(be, 67, 2048, 2048, 5, gpu, act="gelu", residual=True)


def test_silu_single_token(be, gpu):
    check(be, 1, 2048, 256, 6, gpu, act="silu")


@pytest.mark.parametrize("M", [1, 16, 32, 33, 100, 128, 255, 256, 300, 600])
def test_token_counts(be, gpu, M):
    check(be, M, 256, 512, M, gpu)


@pytest.mark.parametrize("splits", [1, 2, 4, 8])
def test_split_k(be, gpu, splits):
    check(be, 67, 512, 2048, 40 + splits, gpu, splits=splits)


@pytest.mark.parametrize("N,splits", [(32, 0), (96, 0), (96, 1)])
def test_partial_channel_tiles(be, gpu, N, splits):
    # N below one 128- or 64-channel weight tile: rows past N are zero-filled
    # by the tile load and never stored
    check(be, 67, N, 256, 50 + N + splits, gpu, splits=splits)


def test_fp32_output_no_bias(be, gpu):
    check(be, 67, 256, 1024, 9, gpu, bias=False, f32=True)


def test_kv_projection_shape(be, gpu):
    # per-tick cross-attention K/V projection of the image condition (4374 tokens)
    check(be, 4374, 512, 2048, 11, gpu)


def test_reference_dequant_then_matmul(be, gpu):
    # same numbers as the reference's two-step path: dequantise (bit-exact vs
    # the dequant op) then a plain fp32 matmul of the dequantised weight
    x, q, s, b, _ = make(67, 256, 512, 13, gpu)
    wd = torch.empty(256, 512, dtype=torch.float32, device=gpu)
    be.dequantize(q, s, wd)
    y = torch.empty(67, 256, dtype=torch.float32, device=gpu)
    be.w8a16_linear(x, q, s, y, bias=b)
    torch.cuda.synchronize()
    ref = x.float() @ wd.t() + b.float()
    assert torch.allclose(y, ref, rtol=1e-4, atol=1e-4)


# serving shapes (32 and 16 sessions × 67 tokens): 256-token tiles in one wave
# of 144 CTAs, and 128-token tiles chosen to fill the wave
@pytest.mark.parametrize("M,act,residual", [(2144, "none", False), (1072, "gelu", True)])
def test_serving_shapes(be, gpu, M, act, residual):
    check(be, M, 2048, 2048, 70 + M, gpu, act=act, residual=residual)


@pytest.mark.parametrize("M,splits", [(67, 0), (67, 1), (300, 0)])
def test_fp32_output_with_fp32_residual(be, gpu, M, splits):
    # the model's residual stream is fp32: y = x·Wᵀ + b + r with r and y fp32 (may alias)
    check(be, M, 2048, 2048, 13 + M, gpu, residual=True, f32=True, splits=splits)


@pytest.mark.parametrize("M,K,F,N,f32", [(67, 2048, 2048, 2048, False), (67, 2048, 2048, 2048, True),
                                         (80, 1024, 512, 128, False), (1, 256, 256, 64, True)])
def test_mlp_as_one_launch(be, gpu, M, K, F, N, f32):
    """sfb_w8a16_mlp (two stages of the persistent projection kernel) against
    the oracle, and against two sfb_w8a16_linear calls within one output ulp."""
    g = torch.Generator().manual_seed(M + K + F + N)
    x = torch.randn(M, K, generator=g).bfloat16().to(gpu)

    def layer(n, k):
        wf = torch.randn(n, k, generator=g) * 0.02
        s = wf.abs().amax(dim=1) / 127.0
        q = torch.round(wf / s[:, None]).clamp(-127, 127).to(torch.int8)
        b = (torch.randn(n, generator=g) * 0.1).bfloat16()
        return q.to(gpu), s.float().to(gpu), b.to(gpu)

    q1, s1, b1 = layer(F, K)
    q2, s2, b2 = layer(N, F)
    dt = torch.float32 if f32 else torch.bfloat16
    r = torch.randn(M, N, generator=g).to(dt).to(gpu)
    y = torch.empty(M, N, dtype=dt, device=gpu)
    be.w8a16_mlp(x, q1, s1, q2, s2, y, b1=b1, b2=b2, residual=r, act="gelu")
    h = torch.empty(M, F, dtype=torch.bfloat16, device=gpu)
    y2 = torch.empty_like(y)
    be.w8a16_linear(x, q1, s1, h, bias=b1, act="gelu")
    be.w8a16_linear(h, q2, s2, y2, bias=b2, residual=r)
    torch.cuda.synchronize()
    hr = oracle.w8a16_linear(x.float().cpu().numpy(), q1.cpu().numpy(), s1.cpu().numpy(),
                             b1.float().cpu().numpy(), None, act=1)
    hr = torch.from_numpy(hr).bfloat16().float().numpy()          # h is stored in bf16
    ref = oracle.w8a16_linear(hr, q2.cpu().numpy(), s2.cpu().numpy(), b2.float().cpu().numpy(),
                              r.float().cpu().numpy(), act=0)
    out = y.float().cpu().numpy()
    # h may round differently in one bf16 ulp where the two kernels' fp32 sums differ
    tol = 4 * ulp_bf16(ref) + 2e-3 * np.abs(ref).max()
    assert (np.abs(out - ref) <= tol).all(), np.abs(out - ref).max()
    assert (y.float() - y2.float()).abs().max().item() <= float(tol.max())
