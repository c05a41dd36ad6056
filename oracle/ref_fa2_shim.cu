// ref_fa2_shim.cu — TEST AND BENCHMARK INFRASTRUCTURE ONLY. C entry points
// around the reference's FlashAttention-2 forward (its vendored copy under
// src/backend/cuda/flash_attn/, SM80 mma.sync kernels, compiled here for
// sm_100a against the CUTLASS/CuTe headers of the image; FA2/CUTLASS pins are
// unknown), built into oracle/_ref/libsfref_fa2.so. bench.py times it beside
// this library's attention on configs 1-3; tests compare it with the oracle.
//
// fp16 goes through the reference's own stock path: cuda_ops::flash_attention
// (src/backend/cuda/ops/attention.cu:183-197, built with SF_USE_FLASH_ATTN) →
// flash_attn_dispatch (:29-80, LSE memset, mask dropped) → flash_attn::mha_fwd
// (flash_attn_adapter.cu:11-155). bf16 cannot go that way: the adapter prints
// "Unsupported BF16" and writes nothing (flash_attn_adapter.cu:144). For bf16
// this shim fills Flash_fwd_params the way the adapter's BHSD branch does
// (flash_attn_adapter.cu:22-130) and calls the bf16 hdim-64 instantiation
// (flash_fwd_hdim64_bf16_sm80.cu) directly.
#include <cuda_runtime.h>
#include <cmath>
#include <cstring>
#include <memory>

#include "servoflow/core/tensor.h"
#include "backend/cuda/ops/attention.h"
#include "flash_attn/flash_api.h"

namespace {
sf::Tensor wrap(const void* p, std::initializer_list<int64_t> shape, sf::DType dt) {
    auto st = std::make_shared<sf::Storage>(const_cast<void*>(p), 0, sf::kCUDA0, nullptr);
    return sf::Tensor(st, sf::Shape(shape), dt);
}
}  // namespace

// Bytes of workspace the reference's dispatcher demands (attention.cu:49-60).
extern "C" long sfref_fa2_workspace_bytes(int B, int H, int Lq) {
    return static_cast<long>(B) * H * Lq * 4 + 128 * 1024;
}

// Contiguous BHSD q/k/v/out, D == 64. dtype 1 (fp16) or 2 (bf16), as sf::DType.
extern "C" int sfref_fa2_attention(const void* q, const void* k, const void* v, void* out, int dtype,
                                   int B, int H, int Lq, int Lk, int D, float scale, int causal,
                                   void* workspace, long workspace_bytes, void* stream) {
    try {
        if (D != 64) return -3;
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (dtype == 1) {
            const auto dt = sf::DType::Float16;
            sf::Tensor Q = wrap(q, {B, H, Lq, D}, dt), K = wrap(k, {B, H, Lk, D}, dt);
            sf::Tensor V = wrap(v, {B, H, Lk, D}, dt), O = wrap(out, {B, H, Lq, D}, dt);
            sf::cuda_ops::flash_attention(Q, K, V, O, nullptr, scale, causal != 0, workspace,
                                          static_cast<size_t>(workspace_bytes), s);
            return cudaGetLastError() == cudaSuccess ? 0 : -6;
        }
        if (dtype != 2) return -2;
        if (workspace_bytes < sfref_fa2_workspace_bytes(B, H, Lq)) return -5;
        if (scale == 0.f) scale = 1.f / sqrtf(static_cast<float>(D));
        cudaMemsetAsync(workspace, 0, static_cast<size_t>(workspace_bytes), s);
        FLASH_NAMESPACE::Flash_fwd_params p;
        std::memset(&p, 0, sizeof(p));
        p.is_bf16 = true;
        p.q_ptr = const_cast<void*>(q); p.k_ptr = const_cast<void*>(k); p.v_ptr = const_cast<void*>(v);
        p.o_ptr = out; p.softmax_lse_ptr = workspace;
        p.b = B; p.h = H; p.h_k = H; p.h_h_k_ratio = 1;
        p.seqlen_q = Lq; p.seqlen_k = Lk; p.seqlen_q_rounded = Lq; p.seqlen_k_rounded = Lk;
        p.d = D; p.d_rounded = D;
        p.q_row_stride = D; p.k_row_stride = D; p.v_row_stride = D; p.o_row_stride = D;
        p.q_head_stride = static_cast<int64_t>(Lq) * D; p.o_head_stride = static_cast<int64_t>(Lq) * D;
        p.k_head_stride = static_cast<int64_t>(Lk) * D; p.v_head_stride = static_cast<int64_t>(Lk) * D;
        p.q_batch_stride = static_cast<int64_t>(H) * Lq * D; p.o_batch_stride = p.q_batch_stride;
        p.k_batch_stride = static_cast<int64_t>(H) * Lk * D; p.v_batch_stride = p.k_batch_stride;
        p.scale_softmax = scale;
        p.scale_softmax_log2 = scale * static_cast<float>(M_LOG2E);
        p.is_causal = causal != 0;
        p.window_size_left = -1;
        p.window_size_right = causal ? 0 : -1;
        p.softcap = 0.f;
        p.p_dropout = 0.f; p.rp_dropout = 1.f; p.scale_softmax_rp_dropout = scale;
        if (causal)
            FLASH_NAMESPACE::run_mha_fwd_<cutlass::bfloat16_t, 64, true>(p, s);
        else
            FLASH_NAMESPACE::run_mha_fwd_<cutlass::bfloat16_t, 64, false>(p, s);
        return cudaGetLastError() == cudaSuccess ? 0 : -6;
    } catch (...) {
        return -1;
    }
}
