"""The MLP entry point that allocates nothing (sfb_w8a16_mlp_noalloc), called
through the C ABI on the GPU.

It is for callers that cannot allocate device memory where they run the MLP
(a real-time loop that forbids cudaMalloc after start-up, a framework whose
allocator owns all device memory, a plugin that only receives its inputs and
outputs): its scratch lives in a fixed-size array inside the library. Two
calls in a row must each match the entry point that takes a caller-provided
workspace (sfb_w8a16_mlp), within the tolerance of the MLP parity test in
tests/test_w8a16_gpu.py; the second call also shows that whatever the first
left in the shared scratch does not leak into the next result. The file's
name makes pytest collect it last, so a run that stops at the first failure
has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def ulp_bf16(x):
    ax = np.maximum(np.abs(x), 2.0 ** -126)
    return np.exp2(np.floor(np.log2(ax)) - 7)


def _lib():
    from servoflow_b200 import _capi
    lib = _capi.lib()
    c = ctypes
    lib.sfb_w8a16_mlp_noalloc.restype = c.c_int
    lib.sfb_w8a16_mlp_noalloc.argtypes = [c.c_void_p, c.c_int64, c.c_void_p, c.c_void_p, c.c_void_p,
                                          c.c_void_p, c.c_void_p, c.c_void_p, c.c_void_p, c.c_int64,
                                          c.c_void_p, c.c_int64, c.c_int32, c.c_int32, c.c_int32, c.c_int32,
                                          c.c_int32, c.c_int32, c.c_void_p]
    lib.sfb_w8a16_mlp_noalloc_max_bytes.restype = c.c_size_t
    lib.sfb_w8a16_mlp_noalloc_max_bytes.argtypes = []
    return lib, _capi


def _layer(g, n, k, dev):
    wf = torch.randn(n, k, generator=g) * 0.02
    s = wf.abs().amax(dim=1) / 127.0
    q = torch.round(wf / s[:, None]).clamp(-127, 127).to(torch.int8)
    b = (torch.randn(n, generator=g) * 0.1).bfloat16()
    return q.to(dev), s.float().to(dev), b.to(dev)


def test_noalloc_mlp_matches_workspace_mlp_twice(gpu):
    lib, capi = _lib()
    M, K, F, N = 67, 2048, 2048, 2048
    sh = torch.cuda.current_stream().cuda_stream
    ws_bytes = lib.sfb_w8a16_mlp_workspace_bytes(M, F)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=gpu)
    for seed in (1, 2):                       # two calls in a row, different inputs
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(M, K, generator=g).bfloat16().to(gpu)
        q1, s1, b1 = _layer(g, F, K, gpu)
        q2, s2, b2 = _layer(g, N, F, gpu)
        r = torch.randn(M, N, generator=g).bfloat16().to(gpu)
        y_ws = torch.empty(M, N, dtype=torch.bfloat16, device=gpu)
        y_na = torch.empty_like(y_ws)
        args = lambda y: (x.data_ptr(), K, q1.data_ptr(), s1.data_ptr(), b1.data_ptr(), q2.data_ptr(),
                          s2.data_ptr(), b2.data_ptr(), r.data_ptr(), N, y.data_ptr(), N, capi.SFB_BF16,
                          M, K, F, N, 1)
        capi.check(lib.sfb_w8a16_mlp(*args(y_ws), ws.data_ptr(), ws_bytes, sh), "mlp")
        capi.check(lib.sfb_w8a16_mlp_noalloc(*args(y_na), sh), "mlp noalloc")
        torch.cuda.synchronize()
        a, b = y_na.float().cpu().numpy(), y_ws.float().cpu().numpy()
        tol = 4 * ulp_bf16(b) + 2e-3 * np.abs(b).max()
        assert np.isfinite(a).all()
        assert (np.abs(a - b) <= tol).all(), np.abs(a - b).max()


def test_noalloc_rejects_sizes_beyond_its_scratch(gpu):
    lib, capi = _lib()
    # M·F·2 bytes of hidden activations beyond the fixed scratch: refused, not run
    M, F = 80, 4096
    assert lib.sfb_w8a16_mlp_workspace_bytes(M, F) > lib.sfb_w8a16_mlp_noalloc_max_bytes()
    p = ctypes.c_void_p(256)
    rc = lib.sfb_w8a16_mlp_noalloc(p, 2048, p, p, None, p, p, None, None, 0, p, 2048, capi.SFB_BF16,
                                   M, 2048, F, 2048, 1, None)
    assert rc == capi.SFB_ERR_WORKSPACE
    assert b"static scratch" in lib.sfb_last_error()
