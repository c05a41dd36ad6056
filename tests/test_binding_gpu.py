"""GPU run of the servoflow-side binding (integration/sfb_servoflow.hpp,
compiled against the reference's headers): the call patterns of the
reference's own callers of IBackend::attention and IBackend::dequantize,
through sf::Tensor views, against the oracle.

- Octo (src/models/octo/octo.cpp:79,209): fp16 Q/K/V [1, 6, 64, 64] with an
  all-zero fp16 additive mask [1, 1, 64, 64] — must equal unmasked attention.
- RDT-1B (include/servoflow/models/rdt1b/dit_block.h:141,153): a Bool
  [B, Sk] key-padding mask on the language cross-attention.
- Int32 [B] lengths and a general additive fp32 [B, 1, Sq, Sk] mask.
- dequantize with per-channel fp16 scales, bit-exact against the oracle.
Tolerances as tests/test_attention_gpu.py."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle
from servoflow_b200.backend import B200Backend

from test_attention_gpu import check_close, make, oracle_of, run

pytestmark = pytest.mark.gpu

F32, F16, BF16, I32, BOOL = 0, 1, 2, 5, 6
CODE = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16, torch.int32: I32, torch.bool: BOOL}


@pytest.fixture(scope="module")
def bind(gpu):
    b = oracle.binding_lib()
    if b is None:
        pytest.skip("binding not built (needs the reference tree at build time)")
    return b


def battn(b, q, k, v, mask=None, scale=0.0, causal=False):
    out = torch.empty_like(q)
    B, H, Lq, D = q.shape
    Lk = k.shape[2]
    sh = (ctypes.c_int64 * 4)(*(mask.shape if mask is not None else (0,)))
    rc = b.sfbind_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), CODE[q.dtype],
                            CODE[v.dtype], B, H, Lq, Lk, D,
                            mask.data_ptr() if mask is not None else None,
                            CODE[mask.dtype] if mask is not None else 0,
                            mask.dim() if mask is not None else 0, sh, scale, 1 if causal else 0,
                            torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0, b.sfbind_last_message()
    return out


def test_octo_zero_fp16_mask(bind, gpu):
    q, k, v = make(1, 6, 6, 64, 64, 64, torch.float16, 31, gpu)
    zero = torch.zeros(1, 1, 64, 64, dtype=torch.float16, device=gpu)
    out = battn(bind, q, k, v, zero)
    assert torch.equal(out, run(B200Backend(0), q, k, v))
    check_close(out, oracle_of(q, k, v), torch.float16)


def test_rdt1b_bool_key_mask(bind, gpu):
    B, Lk = 2, 1024
    q, k, v = make(B, 32, 32, 67, Lk, 64, torch.bfloat16, 32, gpu)
    lens = torch.tensor([37, 1024], dtype=torch.int32)
    keep = (torch.arange(Lk)[None, :] < lens[:, None]).to(gpu)
    out = battn(bind, q, k, v, keep)
    check_close(out, oracle_of(q, k, v, kv_len=lens.numpy()), torch.bfloat16)
    assert torch.equal(out, battn(bind, q, k, v, lens.to(gpu)))        # Int32 [B] lengths


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_additive_mask(bind, gpu, dtype):
    q, k, v = make(2, 4, 4, 67, 300, 64, dtype, 33, gpu)
    g = torch.Generator().manual_seed(34)
    m = torch.randn(2, 1, 67, 300, generator=g)
    m[torch.rand(2, 1, 67, 300, generator=g) < 0.2] = float("-inf")
    m[..., 0] = 0.0
    out = battn(bind, q, k, v, m.to(gpu))
    check_close(out, oracle_of(q, k, v, attn_mask=m.numpy()), dtype)


def test_dequantize_per_channel(bind, gpu):
    # per-output-channel fp16 scales, fp16 output: the reference's rule and
    # rounding (quantization.cu:18-50), restated by the oracle
    g = torch.Generator().manual_seed(35)
    q = torch.randint(-127, 128, (64, 96), generator=g, dtype=torch.int8)
    s = (torch.rand(64, generator=g) * 0.1).half()
    out = torch.empty(64, 96, dtype=torch.float16, device=gpu)
    qd, sd = q.to(gpu), s.to(gpu)
    rc = bind.sfbind_dequantize(qd.data_ptr(), sd.data_ptr(), F16, 64, out.data_ptr(), F16, 64, 96,
                                torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0, bind.sfbind_last_message()
    ref = oracle.dequant_int8(q.numpy(), s.float().numpy(), round_mode=1)
    assert np.array_equal(out.float().cpu().numpy(), ref)
