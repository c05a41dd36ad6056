"""GPU tests of the standalone int8 dequant op against the reference's known
answers (tests/unit/test_quantization.cpp:9-94) and the oracle (bit-exact:
integer × scale, rounded once)."""
import json
import os

import numpy as np
import pytest
import torch

from oracle import oracle
from servoflow_b200.backend import B200Backend

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def be(gpu):
    return B200Backend(0)


@pytest.mark.parametrize("case", ["per_tensor", "per_channel"])
def test_reference_kats(be, gpu, case):
    with open(os.path.join(GOLDEN, "dequant_kat.json")) as f:
        c = json.load(f)[case]
    q = torch.tensor(c["q"], dtype=torch.int8, device=gpu)
    s = torch.tensor(c["scale"], dtype=torch.float16, device=gpu)
    out = torch.empty(q.shape, dtype=torch.float16, device=gpu)
    be.dequantize(q, s, out)
    torch.cuda.synchronize()
    assert np.abs(out.float().cpu().numpy() - np.array(c["out"], np.float32)).max() <= c["tol"]


@pytest.mark.parametrize("out_dtype,mode", [(torch.float16, 1), (torch.bfloat16, 2),
                                            (torch.float32, 0)])
@pytest.mark.parametrize("scale_dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("rows,cols,per_channel", [(6144, 2048, True), (7, 33, True),
                                                   (3, 1000, False), (1, 5, False)])
def test_random_bit_exact(be, gpu, out_dtype, mode, scale_dtype, rows, cols, per_channel):
    g = torch.Generator().manual_seed(rows + cols)
    q = torch.randint(-128, 128, (rows, cols), dtype=torch.int8, generator=g)
    n = rows if per_channel else 1
    s = (torch.rand(n, generator=g) * 0.05 + 1e-4).to(scale_dtype)
    out = torch.empty(rows, cols, dtype=out_dtype, device=gpu)
    be.dequantize(q.to(gpu), s.to(gpu), out)
    torch.cuda.synchronize()
    ref = oracle.dequant_int8(q.numpy(), s.float().numpy(), round_mode=mode)
    assert np.array_equal(out.float().cpu().numpy(), ref)


def test_matches_reference_kernel(be, gpu):
    ref = oracle.ref_lib()
    if ref is None:
        pytest.skip("oracle/_ref/libsfref.so not built")
    g = torch.Generator().manual_seed(77)
    q = torch.randint(-128, 128, (256, 320), dtype=torch.int8, generator=g).to(gpu)
    s = (torch.rand(256, generator=g) * 0.02).half().to(gpu)
    a = torch.empty(256, 320, dtype=torch.float16, device=gpu)
    b = torch.empty_like(a)
    assert ref.sfref_dequantize(q.data_ptr(), s.data_ptr(), 256, a.data_ptr(), 256, 320, None) == 0
    be.dequantize(q, s, b)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
