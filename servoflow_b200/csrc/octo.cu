// octo.cu — the Octo policy runtime over the libsfb200 kernels: a pre-LN
// transformer backbone, the MLP diffusion head, and the flow-matching
// sampling loop captured once into a CUDA graph.
//
// Follows the reference model (src/models/octo/octo.cpp,
// include/servoflow/models/octo/{octo,config}.h):
//   * OctoBlock::forward (octo.cpp:46-122): x += proj(attn(LN1(x))),
//     x += fc2(GELU(fc1(LN2(x)))), LayerNorm eps 1e-5, SDPA with scale
//     1/sqrt(head_dim) and no mask (the reference passes an all-zero additive
//     mask that its attention drops, attention.cu:30);
//   * OctoDiffusionHead::forward (octo.cpp:144-177): input = [x_t flattened,
//     a 128-wide time embedding filled with 0.1, the context], then
//     fc1 → GELU → fc2 → GELU → fc3. The reference ignores t (its time
//     embedding is the constant fill, octo.cpp:147-148); so does this one;
//   * OctoModel::encode_condition (octo.cpp:196-224) runs the blocks over
//     `seq_len` tokens (a 0.1 fill when the caller passes none) and returns a
//     readout that is a 0.1 fill, not taken from the blocks. readout_token < 0
//     keeps that behaviour; readout_token >= 0 takes that backbone output
//     token as the condition instead;
//   * the sampler is FlowMatchingSampler::sample (src/sampling/
//     flow_matching.cpp:25-93): timesteps linspace(t_start = 1, t_end = 0,
//     num_steps + 1) in fp32, x ← x + (t_{i+1} − t_i)·v, the loop in one graph.
// Changes for this runtime: projection weights are int8 per output channel
// (s_n = max|w_n| / 127) run through the fused sfb_w8a16_linear kernel
// (dequant + GEMM + bias + GELU + residual); activations are bf16 (the
// reference computes in fp16); the QKV projection output is read in place by
// the attention kernel through strides and the attention writes the
// projection's input layout directly (no unpack_qkv / permute kernels,
// octo.cpp:73-87); sessions are batched. The head's input width
// A·H + 128 + hidden is padded with zero weight columns to a multiple of 64
// (the GEMM's K step) and fc3's A·H outputs with zero rows to a multiple of
// 128 (one full 128-channel weight tile); padded lanes never reach the caller.
//
// Weights are random (seeded, generated on the device; the reference leaves
// them uninitialised until a checkpoint loader it does not have, octo.cpp:
// 247-260); sfb_octo_param exposes every tensor so a test can run the CPU
// oracle on the same values.
#include <map>
#include <string>
#include <vector>

#include "common.cuh"

namespace sfb {
int attention_simt_launch(const sfb_attn_args& a, cudaStream_t stream);

namespace octo {

using rdt::Linear;
using rdt::grid_for;

constexpr float kLnEps = 1e-5f;      // octo.cpp:56,102
constexpr float kFill = 0.1f;        // the reference's placeholder fills (octo.cpp:148,206,220)
constexpr int kTimeDim = 128;        // OctoDiffusionHead time_dim (octo.cpp:127)

// ── kernels ─────────────────────────────────────────────────────────────────

// LayerNorm over rows of D (D % 8 == 0, D <= 256·kC): y = (x − μ)·rstd·γ + β,
// μ and the population variance in fp32, two passes over the row held in
// registers. One warp per row; lane l holds the 8-wide chunks l + 32i.
template <int kC>
__global__ void layer_norm_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                  const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ b,
                                  __nv_bfloat16* __restrict__ out, int64_t ldo, int rows, int D, float eps) {
    pdl_trigger();
    pdl_wait();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const __nv_bfloat16* xr = x + warp * ldx;
    float v[kC][8];
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < kC; ++i) {
        const int c = (i * 32 + lane) * 8;
        if (c < D) {
            const uint4 u = *reinterpret_cast<const uint4*>(xr + c);
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = __bfloat1622float2(h[k]);
                v[i][2 * k] = f.x; v[i][2 * k + 1] = f.y;
                sum += f.x + f.y;
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = sum / static_cast<float>(D);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kC; ++i)
        if ((i * 32 + lane) * 8 < D) {
#pragma unroll
            for (int k = 0; k < 8; ++k) { const float d = v[i][k] - mean; ss = fmaf(d, d, ss); }
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rstd = 1.f / sqrtf(ss / static_cast<float>(D) + eps);
    __nv_bfloat16* orow = out + warp * ldo;
#pragma unroll
    for (int i = 0; i < kC; ++i) {
        const int c = (i * 32 + lane) * 8;
        if (c >= D) continue;
        const uint4 gu = *reinterpret_cast<const uint4*>(g + c);
        const uint4 bu = *reinterpret_cast<const uint4*>(b + c);
        const __nv_bfloat162* gg = reinterpret_cast<const __nv_bfloat162*>(&gu);
        const __nv_bfloat162* bb = reinterpret_cast<const __nv_bfloat162*>(&bu);
        uint4 r;
        __nv_bfloat162* ro = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 gf = __bfloat1622float2(gg[k]), bf = __bfloat1622float2(bb[k]);
            ro[k] = __floats2bfloat162_rn((v[i][2 * k] - mean) * rstd * gf.x + bf.x,
                                          (v[i][2 * k + 1] - mean) * rstd * gf.y + bf.y);
        }
        *reinterpret_cast<uint4*>(orow + c) = r;
    }
}

// out[i] = value for i < n (the reference's backend->fill, in bf16)
__global__ void fill_bf16_kernel(__nv_bfloat16* __restrict__ out, int64_t n, float value) {
    pdl_trigger();
    pdl_wait();
    const __nv_bfloat16 v = __float2bfloat16_rn(value);
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = v;
}

// Head input row b (octo.cpp:150-160): [x_t[b] (HA values) | 0.1 × tdim |
// cond[b] (D values) | zeros up to Kp].
__global__ void head_input_kernel(const float* __restrict__ x_t, const __nv_bfloat16* __restrict__ cond,
                                  __nv_bfloat16* __restrict__ out, int B, int HA, int tdim, int D, int Kp,
                                  float t_fill) {
    pdl_trigger();
    pdl_wait();
    const int64_t n = static_cast<int64_t>(B) * Kp;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % Kp), b = static_cast<int>(i / Kp);
        __nv_bfloat16 v;
        if (c < HA) v = __float2bfloat16_rn(x_t[static_cast<int64_t>(b) * HA + c]);
        else if (c < HA + tdim) v = __float2bfloat16_rn(t_fill);
        else if (c < HA + tdim + D) v = cond[static_cast<int64_t>(b) * D + (c - HA - tdim)];
        else v = __float2bfloat16_rn(0.f);
        out[i] = v;
    }
}

// Euler step of the flow-matching sampler (flow_matching.cpp:69-74):
// x ← x + dt·v, the product rounded before the sum as the reference's
// scale-then-add does. v rows have stride ldv (fc3's padded width).
__global__ void euler_kernel(float* __restrict__ x, const float* __restrict__ v, int64_t ldv, int B, int HA,
                             float dt) {
    pdl_trigger();
    pdl_wait();
    const int64_t n = static_cast<int64_t>(B) * HA;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = i / HA, c = i % HA;
        x[i] = __fadd_rn(x[i], __fmul_rn(dt, v[b * ldv + c]));
    }
}

// The Euler step of one sampling step fused with the head input of the next
// (euler_kernel then head_input_kernel in one pass): the thread of column
// c < HA updates x[b, c] exactly as euler_kernel does and writes its bf16
// copy into the next input row; the other columns are filled as
// head_input_kernel fills them.
__global__ void euler_input_kernel(float* __restrict__ x, const float* __restrict__ v, int64_t ldv,
                                   const __nv_bfloat16* __restrict__ cond, __nv_bfloat16* __restrict__ out,
                                   int B, int HA, int tdim, int D, int Kp, float t_fill, float dt) {
    pdl_trigger();
    pdl_wait();
    const int64_t n = static_cast<int64_t>(B) * Kp;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % Kp), b = static_cast<int>(i / Kp);
        __nv_bfloat16 o;
        if (c < HA) {
            const int64_t xi = static_cast<int64_t>(b) * HA + c;
            const float nx = __fadd_rn(x[xi], __fmul_rn(dt, v[b * ldv + c]));
            x[xi] = nx;
            o = __float2bfloat16_rn(nx);
        } else if (c < HA + tdim) {
            o = __float2bfloat16_rn(t_fill);
        } else if (c < HA + tdim + D) {
            o = cond[static_cast<int64_t>(b) * D + (c - HA - tdim)];
        } else {
            o = __float2bfloat16_rn(0.f);
        }
        out[i] = o;
    }
}

// velocity[b, c] = v[b·ldv + c] for c < HA (drops fc3's padded lanes)
__global__ void copy_velocity_kernel(const float* __restrict__ v, int64_t ldv, float* __restrict__ out, int B,
                                     int HA) {
    pdl_trigger();
    pdl_wait();
    const int64_t n = static_cast<int64_t>(B) * HA;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = v[(i / HA) * ldv + i % HA];
}

// cond[b] = x[b, token] (rows of D; the readout_token >= 0 mode)
__global__ void gather_token_kernel(const __nv_bfloat16* __restrict__ x, int S, int D, int token,
                                    __nv_bfloat16* __restrict__ cond, int B) {
    pdl_trigger();
    pdl_wait();
    const int64_t n = static_cast<int64_t>(B) * D;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = i / D, c = i % D;
        cond[i] = x[(b * S + token) * D + c];
    }
}

// One block per output row of a [N, K] int8 weight whose columns k >= Kv and
// rows r >= Nv are zero padding: the valid part is w ~ N(0, std²) (element
// (r, k) drawn at index r·Kv + k), s = max|w| / 127 (1 for a zero row),
// q = round(w / s). Padded rows get s = 1.
__global__ void init_int8_padded_kernel(int8_t* q, float* s, int K, int Kv, int Nv, uint64_t seed, float std) {
    const int r = blockIdx.x;
    __shared__ float red[32];
    const bool row_ok = r < Nv;
    float mx = 0.f;
    if (row_ok)
        for (int k = threadIdx.x; k < Kv; k += blockDim.x)
            mx = fmaxf(mx, fabsf(std * rdt::normal_at(seed, static_cast<uint64_t>(r) * Kv + k)));
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x < 32) {
        mx = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (threadIdx.x == 0) red[0] = mx;
    }
    __syncthreads();
    const float sc = red[0] > 0.f ? red[0] / 127.f : 1.f;
    if (threadIdx.x == 0) s[r] = sc;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        float qv = 0.f;
        if (row_ok && k < Kv)
            qv = fminf(127.f, fmaxf(-127.f, rintf(std * rdt::normal_at(seed, static_cast<uint64_t>(r) * Kv + k) / sc)));
        q[static_cast<int64_t>(r) * K + k] = static_cast<int8_t>(qv);
    }
}

// zero bias entries [nv, n) of a padded bias vector
__global__ void zero_tail_kernel(__nv_bfloat16* b, int nv, int n) {
    const int i = nv + blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) b[i] = __float2bfloat16_rn(0.f);
}

// ── model ───────────────────────────────────────────────────────────────────

struct Block {
    __nv_bfloat16 *ln1_g, *ln1_b, *ln2_g, *ln2_b;
    Linear qkv, proj, fc1, fc2;
};

struct Model {
    sfb_octo_config c{};
    int device = 0;
    std::vector<void*> allocs;
    std::map<std::string, std::pair<void*, std::pair<int64_t, int32_t>>> params;
    uint64_t seed = 0, counter = 0;

    std::vector<Block> blocks;
    Linear h1, h2, h3;                       // diffusion head
    int kin = 0, kin_pad = 0, out_pad = 0;   // head input width (valid / padded), fc3 rows (padded)
    int hh_pad = 0;                          // head hidden width padded to 64 (zero rows / columns)

    __nv_bfloat16 *x, *xn, *qkv, *attn, *mid;          // backbone [B·S, ·]
    __nv_bfloat16 *cond, *hin, *hh1, *hh2;             // head
    float *xact, *vel;                                  // x_t [B, H·A], fc3 output [B, out_pad]
    std::vector<float> ts;                              // num_steps + 1 timesteps
    std::recursive_mutex mu;                  // entry points of one handle are serialised
    std::map<int, cudaGraphExec_t> graphs;
    std::map<int, int64_t> graph_kernels;
    cudaStream_t own = nullptr;
    cudaEvent_t ev_in = nullptr, ev_out = nullptr;

    int HA() const { return c.action_dim * c.action_horizon; }
};

static int dalloc(Model& m, void** p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) { record_cuda_error(e, "octo allocation"); return SFB_ERR_CUDA; }
    m.allocs.push_back(*p);
    return SFB_OK;
}

static int new_bf16(Model& m, __nv_bfloat16** p, int64_t n, const std::string& name, float mean, float std) {
    SFB_TRY(dalloc(m, reinterpret_cast<void**>(p), n * 2));
    rdt::init_bf16_kernel<<<grid_for(n, 256), 256>>>(*p, n, m.seed + (++m.counter) * 0x1000193ull, mean, std);
    m.params[name] = {*p, {n, SFB_BF16}};
    return launch_status();
}

// [N, K] int8 linear layer whose valid block is [Nv, Kv] (padding is zero)
static int new_linear(Model& m, Linear& L, int N, int K, const std::string& name, int Nv = -1, int Kv = -1) {
    if (Nv < 0) Nv = N;
    if (Kv < 0) Kv = K;
    L.N = N; L.K = K;
    SFB_TRY(dalloc(m, reinterpret_cast<void**>(&L.w), static_cast<size_t>(N) * K));
    SFB_TRY(dalloc(m, reinterpret_cast<void**>(&L.s), static_cast<size_t>(N) * 4));
    init_int8_padded_kernel<<<N, 256>>>(L.w, L.s, K, Kv, Nv, m.seed + (++m.counter) * 0x1000193ull, m.c.weight_std);
    SFB_TRY(launch_status());
    m.params[name + ".weight_q"] = {L.w, {static_cast<int64_t>(N) * K, SFB_I8}};
    m.params[name + ".weight_scale"] = {L.s, {N, SFB_F32}};
    SFB_TRY(new_bf16(m, &L.b, N, name + ".bias", 0.f, m.c.weight_std));
    if (Nv < N) {
        zero_tail_kernel<<<(N - Nv + 127) / 128, 128>>>(L.b, Nv, N);
        SFB_TRY(launch_status());
    }
    return SFB_OK;
}

static int linear(const Linear& L, const __nv_bfloat16* x, int64_t ldx, int M, void* y, int64_t ldy, int act,
                  const __nv_bfloat16* residual, cudaStream_t s, bool y_f32 = false) {
    return w8a16_gemm_launch(x, ldx, L.w, L.s, L.b, residual, residual ? ldy : 0, y, ldy,
                             y_f32 ? SFB_F32 : SFB_BF16, M, L.N, L.K, act, 0, s, true);
}

static int layer_norm(const __nv_bfloat16* x, int64_t ldx, const __nv_bfloat16* g, const __nv_bfloat16* b,
                      __nv_bfloat16* out, int64_t ldo, int rows, int D, cudaStream_t s) {
    const unsigned grid = static_cast<unsigned>((rows + 3) / 4);
    if (D <= 256) {
        prefer_max_shared(layer_norm_kernel<1>);
        return launch_kernel(layer_norm_kernel<1>, grid, 128, 0, s, true, x, ldx, g, b, out, ldo, rows, D, kLnEps);
    }
    if (D <= 512) {
        prefer_max_shared(layer_norm_kernel<2>);
        return launch_kernel(layer_norm_kernel<2>, grid, 128, 0, s, true, x, ldx, g, b, out, ldo, rows, D, kLnEps);
    }
    if (D <= 1024) {
        prefer_max_shared(layer_norm_kernel<4>);
        return launch_kernel(layer_norm_kernel<4>, grid, 128, 0, s, true, x, ldx, g, b, out, ldo, rows, D, kLnEps);
    }
    prefer_max_shared(layer_norm_kernel<8>);
    return launch_kernel(layer_norm_kernel<8>, grid, 128, 0, s, true, x, ldx, g, b, out, ldo, rows, D, kLnEps);
}

static int create(Model& m) {
    const auto& c = m.c;
    const int D = c.hidden, F = c.intermediate, B = c.max_sessions, S = c.seq_len, HA = m.HA();
    m.blocks.resize(c.num_layers);
    for (int l = 0; l < c.num_layers; ++l) {
        Block& bl = m.blocks[l];
        const std::string p = "blocks." + std::to_string(l) + ".";
        SFB_TRY(new_bf16(m, &bl.ln1_g, D, p + "norm1.weight", 1.f, 0.1f));
        SFB_TRY(new_bf16(m, &bl.ln1_b, D, p + "norm1.bias", 0.f, 0.1f));
        SFB_TRY(new_linear(m, bl.qkv, 3 * D, D, p + "attn.qkv"));
        SFB_TRY(new_linear(m, bl.proj, D, D, p + "attn.proj"));
        SFB_TRY(new_bf16(m, &bl.ln2_g, D, p + "norm2.weight", 1.f, 0.1f));
        SFB_TRY(new_bf16(m, &bl.ln2_b, D, p + "norm2.bias", 0.f, 0.1f));
        SFB_TRY(new_linear(m, bl.fc1, F, D, p + "mlp.fc1"));
        SFB_TRY(new_linear(m, bl.fc2, D, F, p + "mlp.fc2"));
    }
    m.kin = HA + kTimeDim + D;
    m.kin_pad = (m.kin + 63) / 64 * 64;
    m.out_pad = (HA + 127) / 128 * 128;
    m.hh_pad = (c.head_hidden + 63) / 64 * 64;
    SFB_TRY(new_linear(m, m.h1, m.hh_pad, m.kin_pad, "head.fc1", c.head_hidden, m.kin));
    SFB_TRY(new_linear(m, m.h2, m.hh_pad, m.hh_pad, "head.fc2", c.head_hidden, c.head_hidden));
    SFB_TRY(new_linear(m, m.h3, m.out_pad, m.hh_pad, "head.fc3", HA, c.head_hidden));

    auto bf = [&](__nv_bfloat16** p, int64_t n) { return dalloc(m, reinterpret_cast<void**>(p), n * 2); };
    auto f32 = [&](float** p, int64_t n) { return dalloc(m, reinterpret_cast<void**>(p), n * 4); };
    const int64_t BS = static_cast<int64_t>(B) * S;
    SFB_TRY(bf(&m.x, BS * D)); SFB_TRY(bf(&m.xn, BS * D)); SFB_TRY(bf(&m.qkv, BS * 3 * D));
    SFB_TRY(bf(&m.attn, BS * D)); SFB_TRY(bf(&m.mid, BS * F));
    SFB_TRY(bf(&m.cond, static_cast<int64_t>(B) * D));
    SFB_TRY(bf(&m.hin, static_cast<int64_t>(B) * m.kin_pad));
    SFB_TRY(bf(&m.hh1, static_cast<int64_t>(B) * m.hh_pad));
    SFB_TRY(bf(&m.hh2, static_cast<int64_t>(B) * m.hh_pad));
    SFB_TRY(f32(&m.xact, static_cast<int64_t>(B) * HA));
    SFB_TRY(f32(&m.vel, static_cast<int64_t>(B) * m.out_pad));
    // the condition starts as the reference's readout: a 0.1 fill
    fill_bf16_kernel<<<grid_for(static_cast<int64_t>(B) * D, 256), 256>>>(m.cond, static_cast<int64_t>(B) * D, kFill);
    SFB_TRY(launch_status());
    // Schedule::linspace (flow_matching.cpp:10-17), fp32 as the reference
    m.ts.resize(c.num_steps + 1);
    for (int i = 0; i <= c.num_steps; ++i) {
        const float alpha = static_cast<float>(i) / static_cast<float>(c.num_steps);
        m.ts[i] = 1.f + alpha * (0.f - 1.f);
    }
    if (cudaStreamCreateWithFlags(&m.own, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&m.ev_in, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&m.ev_out, cudaEventDisableTiming) != cudaSuccess) {
        record_cuda_error(cudaGetLastError(), "octo stream");
        return SFB_ERR_CUDA;
    }
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { record_cuda_error(e, "octo init"); return SFB_ERR_CUDA; }
    return SFB_OK;
}

// The backbone (OctoBlock::forward × num_layers) in place on m.x [B·S, D].
static int backbone(Model& m, int B, cudaStream_t s) {
    const auto& c = m.c;
    const int D = c.hidden, F = c.intermediate, S = c.seq_len, M = B * S;
    for (int l = 0; l < c.num_layers; ++l) {
        const Block& bl = m.blocks[l];
        SFB_TRY(layer_norm(m.x, D, bl.ln1_g, bl.ln1_b, m.xn, D, M, D, s));
        SFB_TRY(linear(bl.qkv, m.xn, D, M, m.qkv, 3 * D, 0, nullptr, s));
        sfb_attn_args a;
        std::memset(&a, 0, sizeof(a));
        const int hd = c.head_dim;
        a.q = m.qkv; a.k = m.qkv + D; a.v = m.qkv + 2 * D; a.out = m.attn;
        const int64_t sb = static_cast<int64_t>(S) * 3 * D;
        a.q_stride[0] = sb; a.q_stride[1] = hd; a.q_stride[2] = 3 * D;
        for (int i = 0; i < 3; ++i) { a.k_stride[i] = a.q_stride[i]; a.v_stride[i] = a.q_stride[i]; }
        a.out_stride[0] = static_cast<int64_t>(S) * D; a.out_stride[1] = hd; a.out_stride[2] = D;
        a.batch = B; a.heads = c.heads; a.heads_kv = c.heads; a.seq_q = S; a.seq_k = S;
        a.head_dim = hd; a.dtype = SFB_BF16;               // scale 0: 1/sqrt(head_dim)
        if (hd == 64) {
            AttnOpts o;
            o.pdl = true;
            SFB_TRY(attention_tc_launch(a, s, o));
        } else {
            SFB_TRY(attention_simt_launch(a, s));
        }
        SFB_TRY(linear(bl.proj, m.attn, D, M, m.x, D, 0, m.x, s));
        SFB_TRY(layer_norm(m.x, D, bl.ln2_g, bl.ln2_b, m.xn, D, M, D, s));
        SFB_TRY(linear(bl.fc1, m.xn, D, M, m.mid, F, 1, nullptr, s));
        SFB_TRY(linear(bl.fc2, m.mid, F, M, m.x, D, 0, m.x, s));
    }
    return SFB_OK;
}

// The head's input rows from m.xact and the current condition (octo.cpp:150-160).
static int head_input(Model& m, int B, cudaStream_t s) {
    prefer_max_shared(head_input_kernel);
    return launch_kernel(head_input_kernel, grid_for(static_cast<int64_t>(B) * m.kin_pad, 256), 256, 0, s, true,
        m.xact, m.cond, m.hin, B, m.HA(), kTimeDim, m.c.hidden, m.kin_pad, kFill);
}

// fc1 → GELU → fc2 → GELU → fc3 of OctoDiffusionHead::forward on m.hin → m.vel.
static int head_mlp(Model& m, int B, cudaStream_t s) {
    SFB_TRY(linear(m.h1, m.hin, m.kin_pad, B, m.hh1, m.hh_pad, 1, nullptr, s));
    SFB_TRY(linear(m.h2, m.hh1, m.hh_pad, B, m.hh2, m.hh_pad, 1, nullptr, s));
    return linear(m.h3, m.hh2, m.hh_pad, B, m.vel, m.out_pad, 0, nullptr, s, true);
}

// num_steps head evaluations and Euler steps; the Euler step of step i and the
// head input of step i + 1 run as one kernel (4 kernels per step, plus one).
static int sample_loop(Model& m, int B, cudaStream_t s) {
    prefer_max_shared(euler_kernel);
    prefer_max_shared(euler_input_kernel);
    SFB_TRY(head_input(m, B, s));
    for (int i = 0; i < m.c.num_steps; ++i) {
        SFB_TRY(head_mlp(m, B, s));
        const float dt = m.ts[i + 1] - m.ts[i];
        if (i + 1 < m.c.num_steps) {
            SFB_TRY(launch_kernel(euler_input_kernel, grid_for(static_cast<int64_t>(B) * m.kin_pad, 256), 256, 0, s,
                true, m.xact, static_cast<const float*>(m.vel), static_cast<int64_t>(m.out_pad),
                static_cast<const __nv_bfloat16*>(m.cond), m.hin, B, m.HA(), kTimeDim, m.c.hidden, m.kin_pad,
                kFill, dt));
        } else {
            SFB_TRY(launch_kernel(euler_kernel, grid_for(static_cast<int64_t>(B) * m.HA(), 256), 256, 0, s, true,
                m.xact, static_cast<const float*>(m.vel), static_cast<int64_t>(m.out_pad), B, m.HA(), dt));
        }
    }
    return SFB_OK;
}

static Model* get(void* h) { return static_cast<Model*>(h); }

}  // namespace octo
}  // namespace sfb

// ── C ABI ───────────────────────────────────────────────────────────────────
extern "C" {

int sfb_octo_default_config(sfb_octo_config* c) {
    if (c == nullptr) return SFB_ERR_INVALID;
    std::memset(c, 0, sizeof(*c));
    // OctoConfig defaults (include/servoflow/models/octo/config.h:15-46),
    // Schedule::num_steps (sampler.h:24)
    c->num_layers = 12; c->hidden = 384; c->heads = 6; c->head_dim = 64; c->intermediate = 1536;
    c->action_dim = 7; c->action_horizon = 4; c->head_hidden = 256; c->seq_len = 64;
    c->max_sessions = 1; c->num_steps = 10; c->readout_token = -1; c->weight_std = 0.02f;
    return SFB_OK;
}

int sfb_octo_create(const sfb_octo_config* cfg, uint64_t seed, void** handle) {
    using namespace sfb;
    if (cfg == nullptr || handle == nullptr) return SFB_ERR_INVALID;
    const auto& c = *cfg;
    // head_dim 64 runs the tensor-core attention, 16/32/128 the CUDA-core one
    // (the reference's unit-test model has hidden 64 = 4 heads × 16,
    // tests/models/test_octo.cpp:17-25); head_hidden is padded to 64 inside
    if ((c.head_dim != 16 && c.head_dim != 32 && c.head_dim != 64 && c.head_dim != 128) || c.heads < 1 ||
        c.hidden != c.heads * c.head_dim || c.hidden % 64 || c.num_layers < 1 ||
        c.intermediate < 64 || c.intermediate % 64 || c.head_hidden < 1 ||
        c.action_dim < 1 || c.action_horizon < 1 || c.seq_len < 1 || c.max_sessions < 1 ||
        c.num_steps < 1 || c.num_steps > 1000 || c.hidden > 2048 || c.readout_token >= c.seq_len)
        return SFB_ERR_SHAPE;
    if (!is_sm100(device_info())) return SFB_ERR_UNSUPPORTED;
    auto* m = new (std::nothrow) octo::Model();
    if (m == nullptr) return SFB_ERR_CUDA;
    m->c = c;
    m->seed = seed;
    cudaGetDevice(&m->device);
    const int rc = octo::create(*m);
    if (rc != SFB_OK) {
        for (void* ptr : m->allocs) cudaFree(ptr);
        if (m->ev_in) cudaEventDestroy(m->ev_in);
        if (m->ev_out) cudaEventDestroy(m->ev_out);
        if (m->own) cudaStreamDestroy(m->own);
        delete m;
        return rc;
    }
    *handle = m;
    return SFB_OK;
}

int sfb_octo_destroy(void* handle) {
    auto* m = sfb::octo::get(handle);
    if (m == nullptr) return SFB_ERR_INVALID;
    DeviceGuard _sfb_dev(m->device);
    cudaDeviceSynchronize();
    for (auto& g : m->graphs) cudaGraphExecDestroy(g.second);
    if (m->ev_in) cudaEventDestroy(m->ev_in);
    if (m->ev_out) cudaEventDestroy(m->ev_out);
    if (m->own) cudaStreamDestroy(m->own);
    for (void* ptr : m->allocs) cudaFree(ptr);
    delete m;
    return SFB_OK;
}

int sfb_octo_encode(void* handle, int32_t sessions, const void* tokens, void* features, void* stream) {
    using namespace sfb;
    auto* m = octo::get(handle);
    if (m == nullptr) return SFB_ERR_INVALID;
    SFB_MODEL_ENTRY(m);
    if (sessions < 1 || sessions > m->c.max_sessions) return SFB_ERR_SHAPE;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int D = m->c.hidden, S = m->c.seq_len;
    const int64_t n = static_cast<int64_t>(sessions) * S * D;
    if (tokens != nullptr) {
        cudaError_t e = cudaMemcpyAsync(m->x, tokens, n * 2, cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) { record_cuda_error(e, "octo encode copy"); return SFB_ERR_CUDA; }
    } else {
        SFB_TRY(launch_kernel(octo::fill_bf16_kernel, octo::grid_for(n, 256), 256, 0, s, true, m->x, n, octo::kFill));
    }
    SFB_TRY(octo::backbone(*m, sessions, s));
    if (features != nullptr) {
        cudaError_t e = cudaMemcpyAsync(features, m->x, n * 2, cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) { record_cuda_error(e, "octo encode features"); return SFB_ERR_CUDA; }
    }
    const int64_t nc = static_cast<int64_t>(sessions) * D;
    if (m->c.readout_token < 0)
        return launch_kernel(octo::fill_bf16_kernel, octo::grid_for(nc, 256), 256, 0, s, true, m->cond, nc, octo::kFill);
    return launch_kernel(octo::gather_token_kernel, octo::grid_for(nc, 256), 256, 0, s, true,
                         static_cast<const __nv_bfloat16*>(m->x), S, D, m->c.readout_token, m->cond, sessions);
}

int sfb_octo_set_condition(void* handle, int32_t sessions, const void* context, void* stream) {
    using namespace sfb;
    auto* m = octo::get(handle);
    if (m == nullptr || context == nullptr) return SFB_ERR_INVALID;
    SFB_MODEL_ENTRY(m);
    if (sessions < 1 || sessions > m->c.max_sessions) return SFB_ERR_SHAPE;
    cudaError_t e = cudaMemcpyAsync(m->cond, context, static_cast<size_t>(sessions) * m->c.hidden * 2,
                                    cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) { record_cuda_error(e, "octo condition"); return SFB_ERR_CUDA; }
    return SFB_OK;
}

int sfb_octo_denoise_step(void* handle, int32_t sessions, const float* x_t, float t, float* velocity,
                          void* stream) {
    using namespace sfb;
    (void)t;   // the reference's head embeds a constant, not t (octo.cpp:147-148)
    auto* m = octo::get(handle);
    if (m == nullptr || x_t == nullptr || velocity == nullptr) return SFB_ERR_INVALID;
    SFB_MODEL_ENTRY(m);
    if (sessions < 1 || sessions > m->c.max_sessions) return SFB_ERR_SHAPE;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int HA = m->HA();
    cudaError_t e = cudaMemcpyAsync(m->xact, x_t, static_cast<size_t>(sessions) * HA * 4,
                                    cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) { record_cuda_error(e, "octo denoise copy"); return SFB_ERR_CUDA; }
    SFB_TRY(octo::head_input(*m, sessions, s));
    SFB_TRY(octo::head_mlp(*m, sessions, s));
    return launch_kernel(octo::copy_velocity_kernel, octo::grid_for(static_cast<int64_t>(sessions) * HA, 256), 256, 0, s,
                         true, static_cast<const float*>(m->vel), static_cast<int64_t>(m->out_pad), velocity,
                         sessions, HA);
}

int sfb_octo_sample(void* handle, int32_t sessions, const float* noise, float* actions, int32_t use_graph,
                    void* stream) {
    using namespace sfb;
    auto* m = octo::get(handle);
    if (m == nullptr || noise == nullptr || actions == nullptr) return SFB_ERR_INVALID;
    SFB_MODEL_ENTRY(m);
    if (sessions < 1 || sessions > m->c.max_sessions) return SFB_ERR_SHAPE;
    cudaStream_t caller = static_cast<cudaStream_t>(stream);
    cudaStream_t s = m->own;
    if (cudaEventRecord(m->ev_in, caller) != cudaSuccess || cudaStreamWaitEvent(s, m->ev_in, 0) != cudaSuccess) {
        record_cuda_error(cudaGetLastError(), "octo sample ordering");
        return SFB_ERR_CUDA;
    }
    const size_t bytes = static_cast<size_t>(sessions) * m->HA() * 4;
    // the initial-noise copy stays outside the graph (flow_matching.cpp:48-50)
    if (cudaMemcpyAsync(m->xact, noise, bytes, cudaMemcpyDefault, s) != cudaSuccess) {
        record_cuda_error(cudaGetLastError(), "octo sample input");
        return SFB_ERR_CUDA;
    }
    if (!use_graph) {
        SFB_TRY(octo::sample_loop(*m, sessions, s));
    } else {
        auto it = m->graphs.find(sessions);
        if (it == m->graphs.end()) {
            // first call for this session count: eager (this call's result), then capture
            SFB_TRY(octo::sample_loop(*m, sessions, s));
            cudaGraph_t g = nullptr;
            cudaError_t e = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
            if (e != cudaSuccess) { record_cuda_error(e, "begin capture"); return SFB_ERR_CUDA; }
            // capturing records the loop without running it
            const int rc = octo::sample_loop(*m, sessions, s);
            e = cudaStreamEndCapture(s, &g);
            if (rc != SFB_OK) { if (g) cudaGraphDestroy(g); return rc; }
            if (e != cudaSuccess) { record_cuda_error(e, "end capture"); return SFB_ERR_CUDA; }
            size_t nn = 0;
            int64_t nk = 0;
            if (cudaGraphGetNodes(g, nullptr, &nn) == cudaSuccess && nn > 0) {
                std::vector<cudaGraphNode_t> nodes(nn);
                if (cudaGraphGetNodes(g, nodes.data(), &nn) == cudaSuccess)
                    for (size_t i = 0; i < nn; ++i) {
                        cudaGraphNodeType ty;
                        if (cudaGraphNodeGetType(nodes[i], &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) ++nk;
                    }
            }
            m->graph_kernels[sessions] = nk;
            cudaGraphExec_t ge = nullptr;
            e = cudaGraphInstantiate(&ge, g, 0);
            cudaGraphDestroy(g);
            if (e != cudaSuccess) { record_cuda_error(e, "graph instantiate"); return SFB_ERR_CUDA; }
            m->graphs[sessions] = ge;
        } else {
            cudaError_t e = cudaGraphLaunch(it->second, s);
            if (e != cudaSuccess) { record_cuda_error(e, "graph launch"); return SFB_ERR_CUDA; }
        }
    }
    if (cudaMemcpyAsync(actions, m->xact, bytes, cudaMemcpyDefault, s) != cudaSuccess ||
        cudaEventRecord(m->ev_out, s) != cudaSuccess || cudaStreamWaitEvent(caller, m->ev_out, 0) != cudaSuccess) {
        record_cuda_error(cudaGetLastError(), "octo sample output");
        return SFB_ERR_CUDA;
    }
    return SFB_OK;
}

int sfb_octo_timesteps(void* handle, float* timesteps, int32_t n) {
    auto* m = sfb::octo::get(handle);
    if (m == nullptr || timesteps == nullptr || n != m->c.num_steps + 1) return SFB_ERR_INVALID;
    SFB_MODEL_ENTRY(m);
    for (int i = 0; i < n; ++i) timesteps[i] = m->ts[i];
    return SFB_OK;
}

int sfb_octo_param(void* handle, const char* name, void** ptr, int64_t* numel, int32_t* dtype) {
    auto* m = sfb::octo::get(handle);
    if (m == nullptr || name == nullptr || ptr == nullptr || numel == nullptr || dtype == nullptr)
        return SFB_ERR_INVALID;
    SFB_MODEL_ENTRY(m);
    auto it = m->params.find(name);
    if (it == m->params.end()) return SFB_ERR_INVALID;
    *ptr = it->second.first;
    *numel = it->second.second.first;
    *dtype = it->second.second.second;
    return SFB_OK;
}

int sfb_octo_graph_kernels(void* handle, int32_t sessions, int64_t* kernels) {
    auto* m = sfb::octo::get(handle);
    if (m == nullptr || kernels == nullptr) return SFB_ERR_INVALID;
    SFB_MODEL_ENTRY(m);
    auto it = m->graph_kernels.find(sessions);
    if (it == m->graph_kernels.end()) return SFB_ERR_INVALID;
    *kernels = it->second;
    return SFB_OK;
}

}  // extern "C"
