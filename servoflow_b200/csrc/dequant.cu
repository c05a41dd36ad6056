// dequant.cu — standalone int8 → fp16/bf16/fp32 dequantisation.
//
// Semantics of the reference's IBackend::dequantize
// (src/backend/cuda/ops/quantization.cu:18-95): out[n,k] = q[n,k] · s[n]
// with a per-output-channel scale (scale numel == rows) or a per-tensor scale
// (numel 1). For an fp16 output the exact product is rounded once to fp16,
// which is what the reference's __hmul(__int2half_rn(q), s) produces (an
// int8 times an fp16 is exact in fp32). The reference accepts only fp16
// scale/output; bf16 and fp32 are added here.
//
// Layout of the work: one thread converts 16 consecutive int8 of a row
// (one 16-byte load, vectorised stores); grid-stride over rows × 16-byte
// chunks; a scalar tail handles cols % 16.
#include "common.cuh"

namespace sfb {
namespace dequant {

template <typename S> __device__ __forceinline__ float load_scale(const S* s, int64_t i);
template <> __device__ __forceinline__ float load_scale<float>(const float* s, int64_t i) { return s[i]; }
template <> __device__ __forceinline__ float load_scale<__half>(const __half* s, int64_t i) { return __half2float(s[i]); }

template <typename O> __device__ __forceinline__ O to_out(float x);
template <> __device__ __forceinline__ float to_out<float>(float x) { return x; }
template <> __device__ __forceinline__ __half to_out<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 to_out<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

template <typename S, typename O>
__global__ void dequant_int8_kernel(const int8_t* __restrict__ in, const S* __restrict__ scale,
                                    bool per_channel, O* __restrict__ out, int64_t rows,
                                    int64_t cols, bool vec_ok) {
    const int64_t chunks_per_row = vec_ok ? cols / 16 : 0;
    const int64_t nvec = rows * chunks_per_row;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < nvec; i += stride) {
        const int64_t r = i / chunks_per_row, c = (i - r * chunks_per_row) * 16;
        const float s = load_scale<S>(scale, per_channel ? r : 0);
        const int4 raw = *reinterpret_cast<const int4*>(in + r * cols + c);
        const int8_t* q = reinterpret_cast<const int8_t*>(&raw);
        alignas(16) O v[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) v[t] = to_out<O>(static_cast<float>(q[t]) * s);
        int4* dst = reinterpret_cast<int4*>(out + r * cols + c);
#pragma unroll
        for (int t = 0; t < static_cast<int>(sizeof(v) / 16); ++t) dst[t] = reinterpret_cast<const int4*>(v)[t];
    }
    // scalar remainder (all elements when the vector path is not usable)
    const int64_t done = chunks_per_row * 16;
    const int64_t tail = cols - done;
    const int64_t ntail = rows * tail;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < ntail; i += stride) {
        const int64_t r = i / tail, c = done + (i - r * tail);
        const float s = load_scale<S>(scale, per_channel ? r : 0);
        out[r * cols + c] = to_out<O>(static_cast<float>(in[r * cols + c]) * s);
    }
}

template <typename S, typename O>
int launch(const int8_t* in, const void* scale, bool per_channel, void* out, int64_t rows,
           int64_t cols, cudaStream_t stream) {
    const bool vec_ok = (reinterpret_cast<uintptr_t>(in) % 16 == 0) &&
                        (reinterpret_cast<uintptr_t>(out) % 16 == 0) && (cols % 16 == 0);
    const int64_t work = vec_ok ? rows * (cols / 16) : rows * cols;
    const int threads = 256;
    const DeviceInfo& dev = device_info();
    int64_t blocks = (work + threads - 1) / threads;
    blocks = std::min<int64_t>(blocks, static_cast<int64_t>(std::max(dev.num_sms, 1)) * 16);
    blocks = std::max<int64_t>(blocks, 1);
    prefer_max_shared(dequant_int8_kernel<S, O>);
    dequant_int8_kernel<S, O><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
        in, static_cast<const S*>(scale), per_channel, static_cast<O*>(out), rows, cols, vec_ok);
    return launch_status();
}

}  // namespace dequant

int dequantize_int8_launch(const int8_t* in, const void* scale, int32_t scale_dtype,
                           int64_t scale_numel, void* out, int32_t out_dtype, int64_t rows,
                           int64_t cols, cudaStream_t stream) {
    if (rows < 0 || cols < 0) return SFB_ERR_SHAPE;
    if (rows == 0 || cols == 0) return SFB_OK;   // reference: numel == 0 is a no-op
    if (in == nullptr || scale == nullptr || out == nullptr) return SFB_ERR_INVALID;
    bool per_channel;
    if (scale_numel == 1) per_channel = false;
    else if (scale_numel == rows) per_channel = true;
    else return SFB_ERR_SHAPE;   // reference: "scale dim 0 mismatch" (quantization.cu:75-78)
    using namespace dequant;
    if (scale_dtype == SFB_F16) {
        switch (out_dtype) {
            case SFB_F16:  return launch<__half, __half>(in, scale, per_channel, out, rows, cols, stream);
            case SFB_BF16: return launch<__half, __nv_bfloat16>(in, scale, per_channel, out, rows, cols, stream);
            case SFB_F32:  return launch<__half, float>(in, scale, per_channel, out, rows, cols, stream);
            default: return SFB_ERR_DTYPE;
        }
    } else if (scale_dtype == SFB_F32) {
        switch (out_dtype) {
            case SFB_F16:  return launch<float, __half>(in, scale, per_channel, out, rows, cols, stream);
            case SFB_BF16: return launch<float, __nv_bfloat16>(in, scale, per_channel, out, rows, cols, stream);
            case SFB_F32:  return launch<float, float>(in, scale, per_channel, out, rows, cols, stream);
            default: return SFB_ERR_DTYPE;
        }
    }
    return SFB_ERR_DTYPE;
}

}  // namespace sfb
