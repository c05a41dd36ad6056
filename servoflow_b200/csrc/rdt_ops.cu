// rdt_ops.cu — the small kernels around the attention and projection kernels
// in an RDT-1B denoising step (sm_100a). All are bandwidth- or latency-bound
// elementwise / row-reduction kernels; none allocates.
//
//   rms_norm        x / sqrt(mean(x²) + eps) · w over rows of D (RmsNorm of
//                   tests/alignment/test_rdt1b_alignment.py:73-80; the
//                   reference's rms_norm_kernel_impl, src/backend/cuda/ops/
//                   norm.cuh:89-122), fp32 math, bf16 in/out, warp per row.
//   head_rms_norm   the same per 64-wide head, in place on a strided
//                   [tokens, heads·64] block (the qk-norm of dit_block.cu:185-196,
//                   applied where the projection wrote Q/K — no layout copy).
//   sincos_embed    [cos(t·f_i), sin(t·f_i)], f_i = 10000^(−i/half)
//                   (dit_block.cu:58-72).
//   assemble_x      x = [t_emb, freq_emb, state_traj, action_traj] + x_pos_embed
//                   per session (rdt1b.cpp:305-340), into the fp32 residual stream.
//   adaptor_input   cat([state | x_t], ones) per session, the state-adaptor input
//                   (test_rdt1b_alignment.py:204-209).
//   add_rows        cond += pos (condition position embeddings).
//   dpm_update      x ← a·x + b·x0 + c·x0_prev (one DPM-Solver++ step; the
//                   coefficients are computed on the host).
//   bf16_to_f16     in place on the cross-attention V cache once per control
//                   tick, so every denoising step reads V in the P·V operand
//                   type (exact for |v| <= 65504, else SFB_ERR_RANGE).
#include "common.cuh"
#include "sm100_ptx.cuh"

namespace sfb {
namespace rdt {

__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }

// Eight consecutive values of a bf16 or fp32 row as fp32.
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int k = 0; k < 4; ++k) { const float2 f = __bfloat1622float2(h[k]); v[2 * k] = f.x; v[2 * k + 1] = f.y; }
}
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// x (bf16 or fp32), out (bf16): [rows, D] with row strides; w: [D]; D % 256 == 0.
template <typename TX>
__global__ void rms_norm_kernel(const TX* __restrict__ x, int64_t ldx,
                                const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                int64_t ldo, int rows, int D, float eps) {
    pdl_trigger();
    pdl_wait();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const TX* xr = x + warp * ldx;
    float ss = 0.f;
    for (int c = lane * 8; c < D; c += 256) {
        float f[8];
        load8(xr + c, f);
#pragma unroll
        for (int i = 0; i < 4; ++i) ss = fmaf(f[2 * i], f[2 * i], fmaf(f[2 * i + 1], f[2 * i + 1], ss));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.f / sqrtf(ss / static_cast<float>(D) + eps);
    __nv_bfloat16* orow = out + warp * ldo;
    for (int c = lane * 8; c < D; c += 256) {
        float f[8];
        load8(xr + c, f);
        const uint4 g = *reinterpret_cast<const uint4*>(w + c);
        const __nv_bfloat162* gw = reinterpret_cast<const __nv_bfloat162*>(&g);
        uint4 r;
        __nv_bfloat162* ro = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 gg = __bfloat1622float2(gw[i]);
            // (x / rms) · w, the order of the reference's RmsNorm
            ro[i] = __floats2bfloat162_rn(f[2 * i] * inv * gg.x, f[2 * i + 1] * inv * gg.y);
        }
        *reinterpret_cast<uint4*>(orow + c) = r;
    }
}

// rms_norm for D = 32·8·kC (kC 16-byte chunks per lane): the constant weight
// is read before the dependency wait and the row is kept in registers, so the
// kernel's critical path is one load of x, the reduction and the store. Same
// operation order as rms_norm_kernel (identical results).
template <int kC, typename TX>
__global__ void rms_norm_reg_kernel(const TX* __restrict__ x, int64_t ldx,
                                    const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                    int64_t ldo, int rows, float eps) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    uint4 g[kC];
#pragma unroll
    for (int i = 0; i < kC; ++i) g[i] = *reinterpret_cast<const uint4*>(w + (i * 32 + lane) * 8);
    pdl_trigger();
    pdl_wait();
    if (warp >= rows) return;
    const TX* xr = x + warp * ldx;
    float u[kC][8];
#pragma unroll
    for (int i = 0; i < kC; ++i) load8(xr + (i * 32 + lane) * 8, u[i]);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kC; ++i) {
#pragma unroll
        for (int k = 0; k < 4; ++k) ss = fmaf(u[i][2 * k], u[i][2 * k], fmaf(u[i][2 * k + 1], u[i][2 * k + 1], ss));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.f / sqrtf(ss / static_cast<float>(kC * 256) + eps);
    __nv_bfloat16* orow = out + warp * ldo;
#pragma unroll
    for (int i = 0; i < kC; ++i) {
        const __nv_bfloat162* gw = reinterpret_cast<const __nv_bfloat162*>(&g[i]);
        uint4 r;
        __nv_bfloat162* ro = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 gg = __bfloat1622float2(gw[k]);
            ro[k] = __floats2bfloat162_rn(u[i][2 * k] * inv * gg.x, u[i][2 * k + 1] * inv * gg.y);
        }
        *reinterpret_cast<uint4*>(orow + (i * 32 + lane) * 8) = r;
    }
}

// In place: for each token row and each head h in [0, heads), the 64 values at
// x[row·ld + h·64 ...] are RMS-normalised with weight w[64]. 8 threads per head.
__global__ void head_rms_norm_kernel(__nv_bfloat16* __restrict__ x, int64_t ld, int rows, int heads,
                                     const __nv_bfloat16* __restrict__ w, float eps) {
    pdl_trigger();
    pdl_wait();
    const int g = (blockIdx.x * blockDim.x + threadIdx.x) >> 3, sub = threadIdx.x & 7;
    if (g >= rows * heads) return;
    const int row = g / heads, h = g - row * heads;
    __nv_bfloat16* p = x + row * ld + h * 64 + sub * 8;
    uint4 u = *reinterpret_cast<const uint4*>(p);
    __nv_bfloat162* v = reinterpret_cast<__nv_bfloat162*>(&u);
    float f[8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = __bfloat1622float2(v[i]);
        f[2 * i] = t.x; f[2 * i + 1] = t.y;
        ss = fmaf(t.x, t.x, fmaf(t.y, t.y, ss));
    }
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    ss += __shfl_xor_sync(0xffffffffu, ss, 4);
    const float inv = 1.f / sqrtf(ss / 64.f + eps);
    const uint4 gu = *reinterpret_cast<const uint4*>(w + sub * 8);
    const __nv_bfloat162* gw = reinterpret_cast<const __nv_bfloat162*>(&gu);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 gg = __bfloat1622float2(gw[i]);
        v[i] = __floats2bfloat162_rn(f[2 * i] * inv * gg.x, f[2 * i + 1] * inv * gg.y);
    }
    *reinterpret_cast<uint4*>(p) = u;
}

// out[0:half] = cos(t·f_i), out[half:2half] = sin(t·f_i), f_i = exp(−ln(10000)·i/half)
__global__ void sincos_kernel(float t, int dim, __nv_bfloat16* __restrict__ out) {
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int half = dim / 2;
    if (i >= half) return;
    const float freq = expf(-logf(10000.f) * static_cast<float>(i) / static_cast<float>(half));
    const float a = t * freq;
    out[i] = __float2bfloat16_rn(cosf(a));
    out[half + i] = __float2bfloat16_rn(sinf(a));
}

// x[b, 0] = t_emb + pos[0]; x[b, 1] = f_emb + pos[1]; x[b, 2 + i] = seq[b, i] + pos[2 + i]
__global__ void assemble_x_kernel(const __nv_bfloat16* __restrict__ t_emb,
                                  const __nv_bfloat16* __restrict__ f_emb,
                                  const __nv_bfloat16* __restrict__ seq,   // [B·(S−2), D]
                                  const __nv_bfloat16* __restrict__ pos,   // [S, D]
                                  float* __restrict__ x, int B, int S, int D) {   // fp32 residual stream
    pdl_trigger();
    pdl_wait();
    const int64_t n8 = static_cast<int64_t>(B) * S * D / 8;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n8;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t e = i * 8;
        const int col = static_cast<int>(e % D);
        const int64_t r = e / D;
        const int b = static_cast<int>(r / S), s = static_cast<int>(r % S);
        const __nv_bfloat16* src = s == 0 ? t_emb + col
                                 : s == 1 ? f_emb + col
                                          : seq + (static_cast<int64_t>(b) * (S - 2) + (s - 2)) * D + col;
        const uint4 a = *reinterpret_cast<const uint4*>(src);
        const uint4 p = *reinterpret_cast<const uint4*>(pos + static_cast<int64_t>(s) * D + col);
        const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&a);
        const __nv_bfloat162* hp = reinterpret_cast<const __nv_bfloat162*>(&p);
        float o[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 fa = __bfloat1622float2(ha[k]), fp = __bfloat1622float2(hp[k]);
            o[2 * k] = fa.x + fp.x; o[2 * k + 1] = fa.y + fp.y;
        }
        *reinterpret_cast<float4*>(x + e) = make_float4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<float4*>(x + e + 4) = make_float4(o[4], o[5], o[6], o[7]);
    }
}

// out[b, 0] = [state[b], 1...1]; out[b, 1 + i] = [x_t[b, i], 1...1]   (A = action dim)
__global__ void adaptor_input_kernel(const __nv_bfloat16* __restrict__ state,  // [B, A]
                                     const float* __restrict__ x_t,            // [B, T, A]
                                     __nv_bfloat16* __restrict__ out,          // [B·(T+1), 2A]
                                     int B, int T, int A) {
    pdl_trigger();
    pdl_wait();
    const int64_t n = static_cast<int64_t>(B) * (T + 1) * 2 * A;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % (2 * A));
        const int64_t r = i / (2 * A);
        const int b = static_cast<int>(r / (T + 1)), s = static_cast<int>(r % (T + 1));
        float v;
        if (c >= A) v = 1.f;
        else if (s == 0) v = bf(state[static_cast<int64_t>(b) * A + c]);
        else v = x_t[(static_cast<int64_t>(b) * T + (s - 1)) * A + c];
        out[i] = __float2bfloat16_rn(v);
    }
}

// cond[b, s, :] += pos[s, :]   for s < S (rows of cond per session: S, row stride D)
__global__ void add_rows_kernel(__nv_bfloat16* __restrict__ cond, const __nv_bfloat16* __restrict__ pos,
                                int B, int S, int D) {
    pdl_trigger();
    pdl_wait();
    const int64_t n8 = static_cast<int64_t>(B) * S * D / 8;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n8;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t e = i * 8;
        const int64_t s = (e / D) % S;
        const int col = static_cast<int>(e % D);
        uint4 a = *reinterpret_cast<const uint4*>(cond + e);
        const uint4 p = *reinterpret_cast<const uint4*>(pos + s * D + col);
        __nv_bfloat162* ha = reinterpret_cast<__nv_bfloat162*>(&a);
        const __nv_bfloat162* hp = reinterpret_cast<const __nv_bfloat162*>(&p);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 fa = __bfloat1622float2(ha[k]), fp = __bfloat1622float2(hp[k]);
            ha[k] = __floats2bfloat162_rn(fa.x + fp.x, fa.y + fp.y);
        }
        *reinterpret_cast<uint4*>(cond + e) = a;
    }
}

// One DPM-Solver++ update over [B, T, A]: x0 rows are rows 3..3+T−1 of each
// session's final-layer output [B, S, A] (fp32). x ← a·x + b·x0 + c·x0_prev,
// then x0_prev ← x0.
__global__ void dpm_update_kernel(float* __restrict__ x, const float* __restrict__ y_final,
                                  float* __restrict__ x0_prev, float a, float bcoef, float c,
                                  int B, int T, int A, int S) {
    pdl_trigger();
    pdl_wait();
    const int64_t n = static_cast<int64_t>(B) * T * A;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int col = static_cast<int>(i % A);
        const int64_t r = i / A;
        const int b = static_cast<int>(r / T), t = static_cast<int>(r % T);
        const float x0 = y_final[(static_cast<int64_t>(b) * S + (S - T) + t) * A + col];
        x[i] = a * x[i] + bcoef * x0 + c * x0_prev[i];
        x0_prev[i] = x0;
    }
}

// In place on a strided [rows, cols] block (cols % 8 == 0): bf16 → fp16, exact
// for |v| <= 65504 (fp16 has more mantissa bits); larger magnitudes set
// SFB_ERR_RANGE in the device error flag.
__global__ void bf16_to_f16_kernel(__nv_bfloat16* __restrict__ x, int64_t ld, int rows, int cols) {
    pdl_trigger();
    pdl_wait();
    const int per_row = cols / 8;
    const int64_t n = static_cast<int64_t>(rows) * per_row;
    bool bad = false;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / per_row, c = (i - r * per_row) * 8;
        uint4* p = reinterpret_cast<uint4*>(x + r * ld + c);
        uint4 u = *p;
        uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float lo = __uint_as_float(w[e] << 16), hi = __uint_as_float(w[e] & 0xffff0000u);
            bad |= (fabsf(lo) > 65504.f) | (fabsf(hi) > 65504.f);
            const __half2 h = __floats2half2_rn(lo, hi);
            w[e] = *reinterpret_cast<const uint32_t*>(&h);
        }
        *p = u;
    }
    if (bad) atomicExch(&g_sfb_device_error, SFB_ERR_RANGE);
}

// The inputs of a norm folded into the next projection (the persistent
// projection kernel): per row m, ss[m] = Σ_k x[m,k]² (fp32 of the bf16
// values) and xg[m, :] = bf16(x[m, :] · g). Warp per row; D % 256 == 0.
__global__ void norm_prep_kernel(const float* __restrict__ x, int64_t ldx,
                                 const __nv_bfloat16* __restrict__ g, __nv_bfloat16* __restrict__ xg,
                                 int64_t ldg, float* __restrict__ ss, int rows, int D) {
    pdl_trigger();
    pdl_wait();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const float* xr = x + warp * ldx;
    float a = 0.f;
    for (int c = lane * 8; c < D; c += 256) {
        float f[8];
        load8(xr + c, f);
        const uint4 gu = *reinterpret_cast<const uint4*>(g + c);
        const __nv_bfloat162* gg = reinterpret_cast<const __nv_bfloat162*>(&gu);
        uint4 o;
        __nv_bfloat162* ho = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 w = __bfloat1622float2(gg[i]);
            a = fmaf(f[2 * i], f[2 * i], fmaf(f[2 * i + 1], f[2 * i + 1], a));
            ho[i] = __floats2bfloat162_rn(f[2 * i] * w.x, f[2 * i + 1] * w.y);
        }
        *reinterpret_cast<uint4*>(xg + warp * ldg + c) = o;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0) ss[warp] = a;
}

}  // namespace rdt

// One warp waits, with the bounded mbarrier wait every kernel uses, on a
// barrier that nothing arrives at: the wait must give up after timeout_ns and
// the kernel must record SFB_ERR_DEVICE_TIMEOUT and return (the failure
// path of the kernels, exercised without a fault). out = 1 if the wait
// completed, 0 if it gave up.
__global__ void bounded_wait_selftest_kernel(uint64_t timeout_ns, int32_t* out) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        ptx::mbar_init(&bar, 1);
        ptx::fence_mbarrier_init();
    }
    __syncthreads();
    const bool done = ptx::mbar_wait(&bar, 0, timeout_ns);
    if (threadIdx.x == 0) {
        *out = done ? 1 : 0;
        if (!done) atomicExch(&g_sfb_device_error, SFB_ERR_DEVICE_TIMEOUT);
    }
}

namespace rdt {

inline unsigned grid_for(int64_t n, int threads) {
    int64_t g = (n + threads - 1) / threads;
    return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(g, 148 * 32)));
}

}  // namespace rdt

int rms_norm_launch(const void* x, int64_t ldx, const void* w, void* out, int64_t ldo, int rows,
                    int D, float eps, cudaStream_t s, bool x_f32) {
    if (D % 256 != 0 || (ldx % 8) || (ldo % 8)) return SFB_ERR_SHAPE;
    if (rows <= 0) return SFB_OK;
    const int warps_per_block = 4;
    const unsigned grid = (rows + warps_per_block - 1) / warps_per_block;
    if (x_f32) {
        if (D == 2048) {
            prefer_max_shared(rdt::rms_norm_reg_kernel<8, float>);
            return launch_kernel(rdt::rms_norm_reg_kernel<8, float>, grid, 32 * warps_per_block, 0, s, true,
                                 static_cast<const float*>(x), ldx, static_cast<const __nv_bfloat16*>(w),
                                 static_cast<__nv_bfloat16*>(out), ldo, rows, eps);
        }
        prefer_max_shared(rdt::rms_norm_kernel<float>);
        return launch_kernel(rdt::rms_norm_kernel<float>, grid, 32 * warps_per_block, 0, s, true,
                             static_cast<const float*>(x), ldx, static_cast<const __nv_bfloat16*>(w),
                             static_cast<__nv_bfloat16*>(out), ldo, rows, D, eps);
    }
    if (D == 2048) {
        prefer_max_shared(rdt::rms_norm_reg_kernel<8, __nv_bfloat16>);
        return launch_kernel(rdt::rms_norm_reg_kernel<8, __nv_bfloat16>, grid, 32 * warps_per_block, 0, s, true,
                             static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(w),
                             static_cast<__nv_bfloat16*>(out), ldo, rows, eps);
    }
    prefer_max_shared(rdt::rms_norm_kernel<__nv_bfloat16>);
    return launch_kernel(rdt::rms_norm_kernel<__nv_bfloat16>, grid, 32 * warps_per_block, 0, s, true,
                         static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(w),
                         static_cast<__nv_bfloat16*>(out), ldo, rows, D, eps);
}

int head_rms_norm_launch(void* x, int64_t ld, int rows, int heads, const void* w, float eps,
                         cudaStream_t s) {
    if (ld % 8) return SFB_ERR_SHAPE;
    if (rows <= 0 || heads <= 0) return SFB_OK;
    const int64_t threads = static_cast<int64_t>(rows) * heads * 8;
    prefer_max_shared(rdt::head_rms_norm_kernel);
    return launch_kernel(rdt::head_rms_norm_kernel, static_cast<unsigned>((threads + 255) / 256), 256, 0, s,
                         true, static_cast<__nv_bfloat16*>(x), ld, rows, heads,
                         static_cast<const __nv_bfloat16*>(w), eps);
}

int bf16_to_f16_launch(void* x, int64_t ld, int rows, int cols, cudaStream_t s) {
    if (cols % 8 || ld % 8) return SFB_ERR_SHAPE;
    if (rows <= 0) return SFB_OK;
    prefer_max_shared(rdt::bf16_to_f16_kernel);
    return launch_kernel(rdt::bf16_to_f16_kernel, rdt::grid_for(static_cast<int64_t>(rows) * cols / 8, 256), 256,
                         0, s, true, static_cast<__nv_bfloat16*>(x), ld, rows, cols);
}

}  // namespace sfb
