// sfb_servoflow.hpp — the servoflow-side binding of libsfb200: what a
// servoflow maintainer includes in src/backend/cuda/cuda_backend.cu so that
// CUDABackend::attention and CUDABackend::dequantize forward to the C ABI of
// include/sfb200.h. It needs servoflow's own headers (servoflow/core/tensor.h)
// and is not part of libsfb200's build; tests/binding compiles it against
// them and runs it on the GPU.
//
// Errors become C++ exceptions, as the reference backend raises them:
// std::invalid_argument for unusable arguments (cuda_backend.cu:156-161),
// std::runtime_error for a failed status (the SF_CUDA_CHECK style of
// cuda_backend.cu:22-40).
#pragma once

#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "servoflow/core/tensor.h"
#include "sfb200.h"

namespace sfb_servoflow {

inline void check(int status, const char* what) {
    if (status != SFB_OK)
        throw std::runtime_error(std::string(what) + ": " + sfb_status_string(status) + " " +
                                 sfb_last_error());
}

// servoflow tensors carry byte strides; the C ABI takes element strides.
inline int64_t elem_stride(const sf::Tensor& t, int dim) {
    return t.strides()[dim] / static_cast<int64_t>(sf::dtype_size(t.dtype()));
}

// IBackend::attention (include/servoflow/backend/backend.h:102-110) over
// sfb_attention_fwd. Q [B, H, Sq, D], K/V [B, Hk, Sk, D] (any strides with a
// contiguous last dimension), out like Q. The mask is read by its dtype and
// rank, each form the reference's interfaces use:
//   Bool / Int8 [B, Sk]             key padding, nonzero = keep
//                                   (models/rdt1b/dit_block.h:141,153);
//   Int32 [B]                       valid key lengths;
//   Float32 / Float16 / BFloat16 [B|1, 1, Sq|1, Sk]
//                                   additive, added to the scaled logits
//                                   (ops/attention.h:16, backend.h:104; the
//                                   zero fp16 mask of octo.cpp:79,209).
inline void attention(const sf::Tensor& Q, const sf::Tensor& K, const sf::Tensor& V, sf::Tensor& out,
                      const sf::Tensor* mask, float scale, bool is_causal, cudaStream_t stream) {
    if (Q.ndim() != 4 || K.ndim() != 4 || V.ndim() != 4 || out.ndim() != 4)
        throw std::invalid_argument("attention: Q, K, V and out must be 4-D [B, H, S, D]");
    sfb_attn_args a{};
    a.q = Q.raw_data_ptr(); a.k = K.raw_data_ptr(); a.v = V.raw_data_ptr();
    a.out = out.raw_data_ptr();
    for (int i = 0; i < 3; ++i) {
        a.q_stride[i] = elem_stride(Q, i); a.k_stride[i] = elem_stride(K, i);
        a.v_stride[i] = elem_stride(V, i); a.out_stride[i] = elem_stride(out, i);
    }
    a.batch = static_cast<int32_t>(Q.shape()[0]); a.heads = static_cast<int32_t>(Q.shape()[1]);
    a.seq_q = static_cast<int32_t>(Q.shape()[2]); a.head_dim = static_cast<int32_t>(Q.shape()[3]);
    a.heads_kv = static_cast<int32_t>(K.shape()[1]); a.seq_k = static_cast<int32_t>(K.shape()[2]);
    a.dtype = static_cast<int32_t>(Q.dtype());             // sf::DType values are the SFB_* codes
    if (V.dtype() != Q.dtype()) a.v_dtype = static_cast<int32_t>(V.dtype());
    a.scale = scale;
    a.is_causal = is_causal ? 1 : 0;
    if (mask != nullptr && mask->numel() > 0) {
        const sf::Shape& ms = mask->shape();
        switch (mask->dtype()) {
            case sf::DType::Bool:
            case sf::DType::Int8:
                if (mask->ndim() != 2 || ms[0] != a.batch || ms[1] != a.seq_k ||
                    (a.seq_k > 1 && elem_stride(*mask, 1) != 1))
                    throw std::invalid_argument("attention: a key-padding mask is [B, Sk], keys contiguous");
                a.key_mask = static_cast<const uint8_t*>(mask->raw_data_ptr());
                a.key_mask_stride_b = elem_stride(*mask, 0);
                break;
            case sf::DType::Int32:
                if (mask->ndim() != 1 || ms[0] != a.batch || !mask->is_contiguous())
                    throw std::invalid_argument("attention: a length mask is contiguous Int32 [B]");
                a.kv_len = static_cast<const int32_t*>(mask->raw_data_ptr());
                break;
            case sf::DType::Float32:
            case sf::DType::Float16:
            case sf::DType::BFloat16:
                if (mask->ndim() != 4 || (ms[0] != 1 && ms[0] != a.batch) || ms[1] != 1 ||
                    (ms[2] != 1 && ms[2] != a.seq_q) || ms[3] != a.seq_k ||
                    (a.seq_k > 1 && elem_stride(*mask, 3) != 1))
                    throw std::invalid_argument("attention: an additive mask is [B|1, 1, Sq|1, Sk], keys contiguous");
                a.attn_mask = mask->raw_data_ptr();
                a.attn_mask_dtype = static_cast<int32_t>(mask->dtype());
                a.attn_mask_stride[0] = ms[0] == 1 ? 0 : elem_stride(*mask, 0);
                a.attn_mask_stride[1] = ms[2] == 1 ? 0 : elem_stride(*mask, 2);
                break;
            default:
                throw std::invalid_argument("attention: unsupported mask dtype");
        }
    }
    check(sfb_attention_fwd(&a, stream), "attention");        // no workspace, nothing allocated
}

// IBackend::dequantize (backend.h:201-206) over sfb_dequantize_int8: Int8
// [N, K] with a per-tensor or per-output-channel scale.
inline void dequantize(const sf::Tensor& in, const sf::Tensor& scale, sf::Tensor& out, cudaStream_t stream) {
    if (in.dtype() != sf::DType::Int8) throw std::invalid_argument("dequantize: input must be Int8");
    if (in.numel() == 0) return;
    const int64_t rows = in.shape()[0], cols = in.numel() / rows;
    check(sfb_dequantize_int8(static_cast<const int8_t*>(in.raw_data_ptr()), scale.raw_data_ptr(),
                              static_cast<int32_t>(scale.dtype()), scale.numel(), out.raw_data_ptr(),
                              static_cast<int32_t>(out.dtype()), rows, cols, stream),
          "dequantize");
}

}  // namespace sfb_servoflow
