// capi.cu — the extern "C" boundary (include/sfb200.h). Validates arguments,
// picks the kernel, and converts every failure into a status code; nothing
// here throws or allocates device memory.
#include "common.cuh"

namespace sfb {
int attention_tc_launch(const sfb_attn_args& a, cudaStream_t stream, const AttnOpts& o);
int attention_simt_launch(const sfb_attn_args& a, cudaStream_t stream);
int w8a16_gemm_launch(const void* x, int64_t ldx, const int8_t* w, const float* w_scale,
                      const void* bias, const void* residual, int64_t ldr, void* y, int64_t ldy,
                      int32_t y_dtype, int32_t M, int32_t N, int32_t K, int32_t act,
                      int32_t num_splits, cudaStream_t stream, bool pdl);
size_t w8a16_mlp_workspace_bytes(int M, int F);
int w8a16_mlp_launch(const void* x, int64_t ldx, const int8_t* w1, const float* s1, const void* b1,
                     const int8_t* w2, const float* s2, const void* b2, const void* residual, int64_t ldr,
                     void* y, int64_t ldy, int32_t y_dtype, int32_t M, int32_t K, int32_t F, int32_t N,
                     int32_t act, void* workspace, size_t workspace_bytes, cudaStream_t stream);
int dequantize_int8_launch(const int8_t* in, const void* scale, int32_t scale_dtype,
                           int64_t scale_numel, void* out, int32_t out_dtype, int64_t rows,
                           int64_t cols, cudaStream_t stream);
}  // namespace sfb

extern "C" {

const char* sfb_status_string(int status) {
    switch (status) {
        case SFB_OK:                 return "ok";
        case SFB_ERR_INVALID:        return "invalid argument";
        case SFB_ERR_DTYPE:          return "unsupported dtype";
        case SFB_ERR_SHAPE:          return "unsupported or inconsistent shape";
        case SFB_ERR_ALIGN:          return "misaligned pointer or stride (16-byte rule)";
        case SFB_ERR_WORKSPACE:      return "workspace missing or too small";
        case SFB_ERR_LAUNCH:         return "kernel launch failed";
        case SFB_ERR_UNSUPPORTED:    return "requires an sm_100a (B200) device";
        case SFB_ERR_CUDA:           return "CUDA runtime error";
        case SFB_ERR_DEVICE_TIMEOUT: return "a bounded device-side wait expired";
        case SFB_ERR_RANGE:          return "input value outside the kernel's supported range";
        case SFB_ERR_IO:             return "file missing, unreadable or malformed";
        default:                     return "unknown status";
    }
}

const char* sfb_version(void) { return "0.1.0 sm_100a"; }

const char* sfb_last_error(void) { return sfb::last_error_buf(); }

int sfb_copy_device(void* dst, const void* src, int64_t bytes) {
    if ((dst == nullptr || src == nullptr) && bytes > 0) return SFB_ERR_INVALID;
    cudaError_t e = cudaMemcpy(dst, src, static_cast<size_t>(bytes), cudaMemcpyDefault);
    if (e != cudaSuccess) { sfb::record_cuda_error(e, "copy"); return SFB_ERR_CUDA; }
    return SFB_OK;
}

int sfb_device_error(int* code, int reset) {
    if (code == nullptr) return SFB_ERR_INVALID;
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, sfb::g_sfb_device_error, sizeof(int)) != cudaSuccess) return SFB_ERR_CUDA;
    *code = v;
    if (reset) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(sfb::g_sfb_device_error, &zero, sizeof(int)) != cudaSuccess) return SFB_ERR_CUDA;
    }
    return SFB_OK;
}

int sfb_selftest_bounded_wait(int64_t timeout_ns, int32_t* completed) {
    if (completed == nullptr || timeout_ns < 100000 || timeout_ns > 2000000000) return SFB_ERR_INVALID;
    if (!sfb::is_sm100(sfb::device_info())) return SFB_ERR_UNSUPPORTED;
    int32_t* d = nullptr;
    if (cudaMalloc(&d, sizeof(int32_t)) != cudaSuccess) { (void)cudaGetLastError(); return SFB_ERR_CUDA; }
    sfb::bounded_wait_selftest_kernel<<<1, 32>>>(static_cast<uint64_t>(timeout_ns), d);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    int32_t h = -1;
    if (e == cudaSuccess) e = cudaMemcpy(&h, d, sizeof(int32_t), cudaMemcpyDeviceToHost);
    cudaFree(d);
    if (e != cudaSuccess) { sfb::record_cuda_error(e, "bounded wait self-test"); return SFB_ERR_CUDA; }
    *completed = h;
    return SFB_OK;
}

int sfb_attention_fwd(const sfb_attn_args* a, void* stream) {
    if (a == nullptr || a->q == nullptr || a->k == nullptr || a->v == nullptr || a->out == nullptr)
        return SFB_ERR_INVALID;
    if (a->batch < 0 || a->heads <= 0 || a->heads_kv <= 0 || a->seq_q < 0 || a->seq_k < 0 ||
        a->head_dim <= 0)
        return SFB_ERR_SHAPE;
    if (a->heads % a->heads_kv != 0) return SFB_ERR_SHAPE;
    if (a->dtype != SFB_F32 && a->dtype != SFB_F16 && a->dtype != SFB_BF16) return SFB_ERR_DTYPE;
    if (a->num_splits < 0 || a->num_splits > 16) return SFB_ERR_INVALID;
    if (a->v_dtype != 0 && a->v_dtype != a->dtype && !(a->v_dtype == SFB_F16 && a->dtype == SFB_BF16))
        return SFB_ERR_DTYPE;
    if (a->attn_mask != nullptr && a->attn_mask_dtype != SFB_F32 && a->attn_mask_dtype != SFB_F16 &&
        a->attn_mask_dtype != SFB_BF16)
        return SFB_ERR_DTYPE;
    if (a->attn_mask != nullptr && (a->attn_mask_stride[0] < 0 || a->attn_mask_stride[1] < 0))
        return SFB_ERR_SHAPE;
    if (a->batch == 0 || a->seq_q == 0) return SFB_OK;
    const sfb::DeviceInfo& dev = sfb::device_info();
    if (!sfb::is_sm100(dev)) return SFB_ERR_UNSUPPORTED;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool tc = (a->dtype == SFB_F16 || a->dtype == SFB_BF16) && a->head_dim == 64;
    const bool v_f16 = a->v_dtype == SFB_F16 && a->dtype == SFB_BF16;
    if (v_f16 && !tc) return SFB_ERR_DTYPE;
    return tc ? sfb::attention_tc_launch(*a, s, [&] {
        // Programmatic dependent launch: before its dependency wait the kernel
        // only sets up barriers and TMEM (no reads of q, k, v, kv_len, masks),
        // so it may start while the stream's previous kernel finishes.
        sfb::AttnOpts o;
        o.v_f16 = v_f16;
        o.pdl = true;
        return o;
    }()) : sfb::attention_simt_launch(*a, s);
}

int sfb_attention_bhsd(const void* q, const void* k, const void* v, void* out, int32_t batch,
                       int32_t heads, int32_t heads_kv, int32_t seq_q, int32_t seq_k,
                       int32_t head_dim, int32_t dtype, const uint8_t* key_mask, float scale,
                       int32_t is_causal, void* stream) {
    sfb_attn_args a;
    std::memset(&a, 0, sizeof(a));
    a.q = q; a.k = k; a.v = v; a.out = out;
    const int64_t D = head_dim;
    a.q_stride[0] = (int64_t)heads * seq_q * D;    a.q_stride[1] = (int64_t)seq_q * D;  a.q_stride[2] = D;
    a.out_stride[0] = a.q_stride[0];              a.out_stride[1] = a.q_stride[1];     a.out_stride[2] = D;
    a.k_stride[0] = (int64_t)heads_kv * seq_k * D; a.k_stride[1] = (int64_t)seq_k * D;  a.k_stride[2] = D;
    for (int i = 0; i < 3; ++i) a.v_stride[i] = a.k_stride[i];
    a.batch = batch; a.heads = heads; a.heads_kv = heads_kv; a.seq_q = seq_q; a.seq_k = seq_k;
    a.head_dim = head_dim; a.dtype = dtype; a.is_causal = is_causal; a.scale = scale;
    a.key_mask = key_mask; a.key_mask_stride_b = seq_k;
    return sfb_attention_fwd(&a, stream);
}

int sfb_dequantize_int8(const int8_t* in, const void* scale, int32_t scale_dtype,
                        int64_t scale_numel, void* out, int32_t out_dtype, int64_t rows,
                        int64_t cols, void* stream) {
    return sfb::dequantize_int8_launch(in, scale, scale_dtype, scale_numel, out, out_dtype, rows,
                                       cols, static_cast<cudaStream_t>(stream));
}

int sfb_w8a16_linear(const void* x, int64_t ldx, const int8_t* w, const float* w_scale,
                     const void* bias, const void* residual, int64_t ldr, void* y, int64_t ldy,
                     int32_t y_dtype, int32_t M, int32_t N, int32_t K, int32_t act,
                     int32_t num_splits, void* stream) {
    return sfb::w8a16_gemm_launch(x, ldx, w, w_scale, bias, residual, ldr, y, ldy, y_dtype, M, N, K,
                                  act, num_splits, static_cast<cudaStream_t>(stream), false);
}

size_t sfb_w8a16_mlp_workspace_bytes(int32_t M, int32_t F) { return sfb::w8a16_mlp_workspace_bytes(M, F); }

int sfb_w8a16_mlp(const void* x, int64_t ldx, const int8_t* w1, const float* s1, const void* b1,
                  const int8_t* w2, const float* s2, const void* b2, const void* residual, int64_t ldr,
                  void* y, int64_t ldy, int32_t y_dtype, int32_t M, int32_t K, int32_t F, int32_t N,
                  int32_t act, void* workspace, size_t workspace_bytes, void* stream) {
    return sfb::w8a16_mlp_launch(x, ldx, w1, s1, b1, w2, s2, b2, residual, ldr, y, ldy, y_dtype, M, K, F, N,
                                 act, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
