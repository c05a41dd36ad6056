"""The servoflow-side binding (integration/sfb_servoflow.hpp), compiled
against the reference's own headers (servoflow/core/tensor.h) into
oracle/_ref/libsfb_binding_test.so. These checks run without a GPU: the
binding rejects unusable masks with std::invalid_argument before any CUDA
call, as CUDABackend::check_device does (cuda_backend.cu:156-161)."""
import ctypes

import pytest

from oracle import oracle

F32, F16, BF16, I8, I32, BOOL = 0, 1, 2, 3, 5, 6


@pytest.fixture(scope="module")
def bind():
    b = oracle.binding_lib()
    if b is None:
        pytest.skip("binding not built (needs the reference tree at build time)")
    return b


def call(b, mask_dtype, shape, B=2, Lq=5, Lk=7):
    p = ctypes.c_void_p(16)                       # never dereferenced: rejected first
    sh = (ctypes.c_int64 * len(shape))(*shape)
    return b.sfbind_attention(p, p, p, p, BF16, BF16, B, 2, Lq, Lk, 64, p, mask_dtype, len(shape), sh,
                              0.0, 0, None)


@pytest.mark.parametrize("dtype,shape", [
    (BOOL, [2, 6]),          # key mask with the wrong Sk
    (BOOL, [2, 1, 5, 7]),    # key mask of rank 4
    (I32, [3]),              # lengths of the wrong batch
    (F16, [2, 2, 5, 7]),     # additive mask with a head dimension
    (F32, [3, 1, 5, 7]),     # additive mask of the wrong batch
    (F32, [2, 1, 4, 7]),     # additive mask of the wrong Sq
    (I8 + 1, [2, 7]),        # Int4 is no mask type
])
def test_bad_masks_raise_invalid_argument(bind, dtype, shape):
    assert call(bind, dtype, shape) == 1
    assert b"attention" in bind.sfbind_last_message()
