// ref_shim.cu — TEST INFRASTRUCTURE ONLY. A C entry point around the
// reference's own CUDA attention and dequant ops, compiled together with the
// reference sources (src/backend/cuda/ops/attention.cu, quantization.cu) into
// oracle/_ref/libsfref.so so the GPU tests can pin the CPU oracle against the
// reference's kernels themselves. Without SF_USE_FLASH_ATTN the reference's
// cuda_ops::flash_attention runs its naive online-softmax kernel
// (attention.cu:141-181) for every dtype.
#include <cuda_runtime.h>
#include <memory>
#include "servoflow/core/tensor.h"
#include "backend/cuda/ops/attention.h"
#include "backend/cuda/ops/quantization.cuh"

namespace {
sf::Tensor wrap(const void* p, std::initializer_list<int64_t> shape, sf::DType dt) {
    auto st = std::make_shared<sf::Storage>(const_cast<void*>(p), 0, sf::kCUDA0, nullptr);
    return sf::Tensor(st, sf::Shape(shape), dt);
}
}  // namespace

extern "C" int sfref_attention(const void* q, const void* k, const void* v, void* out, int dtype,
                               int B, int H, int Lq, int Lk, int D, float scale, int causal,
                               void* stream) {
    try {
        const auto dt = static_cast<sf::DType>(dtype);
        sf::Tensor Q = wrap(q, {B, H, Lq, D}, dt), K = wrap(k, {B, H, Lk, D}, dt);
        sf::Tensor V = wrap(v, {B, H, Lk, D}, dt), O = wrap(out, {B, H, Lq, D}, dt);
        sf::cuda_ops::flash_attention(Q, K, V, O, nullptr, scale, causal != 0, nullptr, 0,
                                      static_cast<cudaStream_t>(stream));
        return cudaGetLastError() == cudaSuccess ? 0 : -6;
    } catch (...) {
        return -1;
    }
}

extern "C" int sfref_dequantize(const void* in, const void* scale_f16, long scale_numel, void* out_f16,
                                long rows, long cols, void* stream) {
    try {
        sf::Tensor I = wrap(in, {rows, cols}, sf::DType::Int8);
        sf::Tensor S = wrap(scale_f16, {scale_numel}, sf::DType::Float16);
        sf::Tensor O = wrap(out_f16, {rows, cols}, sf::DType::Float16);
        sf::cuda_ops::dequantize_int8(I, S, O, static_cast<cudaStream_t>(stream));
        return 0;
    } catch (...) {
        return -1;
    }
}
