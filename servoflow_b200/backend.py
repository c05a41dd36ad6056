"""Python mirror of the reference's IBackend operator interface for the
attention path (include/servoflow/backend/backend.h:102-110, 201-206,
227-229), over the C ABI of libsfb200.so.

Used by the tests and by bench.py; the production host side is C++ and binds
the same C ABI (include/sfb200.h). torch supplies device memory and streams
only; every op runs a libsfb200 kernel, and raises if the library is missing
or the device is not an sm_100a part.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _capi

_DTYPE_CODE = {
    torch.float32: _capi.SFB_F32,
    torch.float16: _capi.SFB_F16,
    torch.bfloat16: _capi.SFB_BF16,
    torch.int8: _capi.SFB_I8,
    torch.int32: _capi.SFB_I32,
    torch.bool: _capi.SFB_BOOL,
}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise _capi.SfbError(_capi.SFB_ERR_DTYPE, f"dtype {dt}") from None


def _stream_handle(stream) -> int:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


def _check_device(t: torch.Tensor, name: str) -> None:
    # reference: CUDABackend::check_device raises std::invalid_argument
    # (src/backend/cuda/cuda_backend.cu:156-161)
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor on this backend's device")


def attention_args(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, out: torch.Tensor,
                   mask: Optional[torch.Tensor] = None, scale: float = 0.0,
                   is_causal: bool = False, num_splits: int = 0,
                   layout: str = "bhsd") -> _capi.AttnArgs:
    """Fills sfb_attn_args from 4-D tensors.

    layout "bhsd": [B, H, S, D] (the reference layout); "bshd": [B, S, H, D].
    mask: None, a bool/uint8 [B, Sk] key-padding mask (True = keep), an
    int32 [B] tensor of valid key lengths, or the reference interface's
    additive float mask (fp32/fp16/bf16, 4-D [B or 1, 1, Sq or 1, Sk], added
    to the scaled logits; -inf masks a key).
    """
    for t, n in ((Q, "Q"), (K, "K"), (V, "V"), (out, "out")):
        _check_device(t, n)
        if t.dim() != 4:
            raise _capi.SfbError(_capi.SFB_ERR_SHAPE, f"{n} must be 4-D")
        if t.stride(3) != 1:
            raise _capi.SfbError(_capi.SFB_ERR_SHAPE, f"{n}: head_dim must be contiguous")
    v_f16 = Q.dtype == torch.bfloat16 and V.dtype == torch.float16
    if not (Q.dtype == K.dtype == out.dtype and (V.dtype == Q.dtype or v_f16)):
        raise _capi.SfbError(_capi.SFB_ERR_DTYPE, "Q/K/V/out dtypes differ")
    if layout == "bhsd":
        bi, hi, si = 0, 1, 2
    elif layout == "bshd":
        bi, hi, si = 0, 2, 1
    else:
        raise ValueError(f"unknown layout {layout!r}")
    a = _capi.AttnArgs()
    a.q, a.k, a.v, a.out = Q.data_ptr(), K.data_ptr(), V.data_ptr(), out.data_ptr()
    for dst, t in ((a.q_stride, Q), (a.k_stride, K), (a.v_stride, V), (a.out_stride, out)):
        dst[0], dst[1], dst[2] = t.stride(bi), t.stride(hi), t.stride(si)
    a.batch, a.heads, a.seq_q, a.head_dim = Q.shape[bi], Q.shape[hi], Q.shape[si], Q.shape[3]
    a.heads_kv, a.seq_k = K.shape[hi], K.shape[si]
    if tuple(out.shape) != tuple(Q.shape) or tuple(V.shape) != tuple(K.shape) \
            or K.shape[bi] != Q.shape[bi] or K.shape[3] != Q.shape[3]:
        raise _capi.SfbError(_capi.SFB_ERR_SHAPE, "inconsistent Q/K/V/out shapes")
    a.dtype = dtype_code(Q.dtype)
    a.is_causal = 1 if is_causal else 0
    a.scale = float(scale)
    a.num_splits = int(num_splits)
    a.v_dtype = _capi.SFB_F16 if v_f16 else 0
    a.kv_len = None
    a.key_mask = None
    if mask is not None:
        _check_device(mask, "mask")
        if mask.dtype == torch.int32 and mask.dim() == 1:
            if mask.shape[0] != a.batch or not mask.is_contiguous():
                raise _capi.SfbError(_capi.SFB_ERR_SHAPE, "kv_len must be contiguous int32 [B]")
            a.kv_len = mask.data_ptr()
        elif mask.dtype in (torch.bool, torch.uint8) and mask.dim() == 2:
            if tuple(mask.shape) != (a.batch, a.seq_k) or mask.stride(1) != 1:
                raise _capi.SfbError(_capi.SFB_ERR_SHAPE, "key mask must be [B, Sk], row-contiguous")
            a.key_mask = mask.data_ptr()
            a.key_mask_stride_b = mask.stride(0)
        elif mask.dtype in (torch.float32, torch.float16, torch.bfloat16) and mask.dim() == 4:
            mb, mh, mq, mk = mask.shape
            if mb not in (1, a.batch) or mh != 1 or mq not in (1, a.seq_q) or mk != a.seq_k \
                    or (mk > 1 and mask.stride(3) != 1):
                raise _capi.SfbError(_capi.SFB_ERR_SHAPE, "additive mask must be [B|1, 1, Sq|1, Sk]")
            a.attn_mask = mask.data_ptr()
            a.attn_mask_dtype = dtype_code(mask.dtype)
            a.attn_mask_stride[0] = mask.stride(0) if mb > 1 else 0
            a.attn_mask_stride[1] = mask.stride(2) if mq > 1 else 0
        else:
            raise _capi.SfbError(_capi.SFB_ERR_SHAPE,
                                 "mask must be bool/uint8 [B, Sk], int32 [B] lengths or a float "
                                 "[B, 1, Sq, Sk] additive mask")
    return a


class B200Backend:
    """The attention-path subset of IBackend, backed by libsfb200 kernels."""

    def __init__(self, device: int = 0):
        self.device = device
        self._lib = _capi.lib()
        self._graphs = {}

    # IBackend::attention (backend.h:105-110)
    def attention(self, Q, K, V, out, mask=None, scale: float = 0.0, is_causal: bool = False,
                  stream=None, num_splits: int = 0, layout: str = "bhsd") -> None:
        a = attention_args(Q, K, V, out, mask, scale, is_causal, num_splits, layout)
        _capi.check(self._lib.sfb_attention_fwd(ctypes.byref(a), _stream_handle(stream)),
                    "attention")

    # IBackend::dequantize (backend.h:205-206)
    def dequantize(self, input, scale, output, stream=None) -> None:
        for t, n in ((input, "input"), (scale, "scale"), (output, "output")):
            _check_device(t, n)
        if input.dtype != torch.int8:
            raise ValueError("dequantize_int8: input must be Int8")   # quantization.cu:62-64
        if input.numel() == 0:
            return
        if not (input.is_contiguous() and output.is_contiguous() and scale.is_contiguous()):
            raise _capi.SfbError(_capi.SFB_ERR_SHAPE, "dequantize needs contiguous tensors")
        if output.shape != input.shape:
            raise _capi.SfbError(_capi.SFB_ERR_SHAPE, "output shape must equal input shape")
        rows = input.shape[0] if input.dim() > 0 else 1
        cols = input.numel() // max(rows, 1)
        _capi.check(self._lib.sfb_dequantize_int8(
            input.data_ptr(), scale.data_ptr(), dtype_code(scale.dtype), scale.numel(),
            output.data_ptr(), dtype_code(output.dtype), rows, cols, _stream_handle(stream)),
            "dequantize")

    # Two int8-weight linear layers as one persistent launch (a block's MLP at one session)
    def w8a16_mlp(self, x, w1, s1, w2, s2, out, b1=None, b2=None, residual=None, act: str = "gelu",
                  workspace=None, stream=None) -> None:
        """out[M, N] = act(x·(w1·s1)ᵀ + b1)·(w2·s2)ᵀ + b2 [+ residual] (sfb_w8a16_mlp)."""
        M, K = x.shape
        F, N = w1.shape[0], w2.shape[0]
        need = self._lib.sfb_w8a16_mlp_workspace_bytes(M, F)
        if workspace is None:
            workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
        acts = {"none": 0, "gelu": 1, "silu": 2}
        p = lambda t: None if t is None else t.data_ptr()
        _capi.check(self._lib.sfb_w8a16_mlp(
            x.data_ptr(), x.stride(0), w1.data_ptr(), s1.data_ptr(), p(b1), w2.data_ptr(), s2.data_ptr(),
            p(b2), p(residual), residual.stride(0) if residual is not None else 0, out.data_ptr(),
            out.stride(0), dtype_code(out.dtype), M, K, F, N, acts[act], workspace.data_ptr(),
            workspace.numel() * workspace.element_size(), _stream_handle(stream)), "w8a16_mlp")

    # Fused replacement of dequantize + gemm_bias_act (backend.h:160-185, 205-206)
    def w8a16_linear(self, x, w_q, w_scale, out, bias=None, residual=None, act: str = "none",
                     num_splits: int = 0, stream=None) -> None:
        """out[M, N] = act(x[M, K] · (w_q[N, K] · w_scale[N])ᵀ + bias) + residual."""
        for t, n in ((x, "x"), (w_q, "w_q"), (w_scale, "w_scale"), (out, "out")):
            _check_device(t, n)
        if x.dtype != torch.bfloat16 or w_q.dtype != torch.int8 or w_scale.dtype != torch.float32:
            raise _capi.SfbError(_capi.SFB_ERR_DTYPE, "x bf16, w_q int8, w_scale fp32 expected")
        if x.stride(1) != 1 or not w_q.is_contiguous() or out.stride(1) != 1:
            raise _capi.SfbError(_capi.SFB_ERR_SHAPE, "row-major tensors expected")
        M, K = x.shape
        N = w_q.shape[0]
        if w_q.shape[1] != K or tuple(out.shape) != (M, N) or w_scale.numel() != N:
            raise _capi.SfbError(_capi.SFB_ERR_SHAPE, "inconsistent shapes")
        if bias is not None and (bias.dtype != torch.bfloat16 or bias.numel() != N):
            raise _capi.SfbError(_capi.SFB_ERR_SHAPE, "bias must be bf16 [N]")
        if residual is not None and (residual.dtype != out.dtype or tuple(residual.shape) != (M, N)
                                     or residual.stride(1) != 1):
            raise _capi.SfbError(_capi.SFB_ERR_SHAPE, "residual must be [M, N] row-major in out's dtype")
        acts = {"none": 0, "gelu": 1, "silu": 2}
        _capi.check(self._lib.sfb_w8a16_linear(
            x.data_ptr(), x.stride(0), w_q.data_ptr(), w_scale.data_ptr(),
            None if bias is None else bias.data_ptr(),
            None if residual is None else residual.data_ptr(),
            0 if residual is None else residual.stride(0), out.data_ptr(), out.stride(0),
            dtype_code(out.dtype), M, N, K, acts[act], int(num_splits), _stream_handle(stream)),
            "w8a16_linear")

    # Graph hooks (backend.h:227-229; CUDABackend keeps one graph per stream,
    # cuda_backend.cu:592-608).
    def graph_begin_capture(self, stream) -> None:
        g = torch.cuda.CUDAGraph()
        self._graphs[_stream_handle(stream)] = g
        g.capture_begin()

    def graph_end_capture(self, stream) -> None:
        self._graphs[_stream_handle(stream)].capture_end()

    def graph_launch(self, stream) -> None:
        self._graphs[_stream_handle(stream)].replay()

    @staticmethod
    def device_error(reset: bool = True) -> int:
        code = ctypes.c_int(0)
        _capi.check(_capi.lib().sfb_device_error(ctypes.byref(code), 1 if reset else 0),
                    "device_error")
        return code.value
