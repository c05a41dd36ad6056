// w8a16_gemm.cu — int8-weight GEMM with the dequantisation fused in, for the
// RDT-1B projections (sm_100a, tcgen05 + TMA).
//
//   Y[m, n] = act( s[n] · Σ_k X[m, k] · Wq[n, k] + bias[n] ) + R[m, n]
//
// X: bf16 activations [M, K] (row stride ldx); Wq: int8 weights [N, K]
// (row-major, one row per output channel, contiguous); s: fp32 per-output-
// channel scales; bias: optional bf16 [N]; act: none, GELU (tanh form) or SiLU;
// R: optional bf16 residual [M, N] (may alias Y); Y: bf16 or fp32 [M, N].
//
// It replaces the reference's two-step path — dequantise the whole weight
// (src/backend/cuda/ops/quantization.cu:18-95), then cuBLASLt GEMM + bias/GELU
// epilogue (src/backend/cuda/cuda_backend.cu:337-467) — with one pass over the
// int8 weights. The result equals dequant-then-GEMM up to fp32 summation
// order: int8 values are exact in bf16, products are exact in fp32, and the
// scale is applied once per output (y_n = s_n · Σ_k x_k q_nk).
//
// Design:
//   * Swap-AB: weight rows are the MMA M dimension (128 per CTA) and tokens
//     the MMA N dimension (N = tokens rounded up to 32, at most 256 per CTA),
//     so a 67-token denoising step does not pad an M=128 tile.
//   * Warp roles per CTA (6 warps): warp 0 issues TMA (int8 weight tile
//     [128 × 64] without swizzle, bf16 activation tile [N × 64] with 128-byte
//     swizzle), warp 1 issues tcgen05.mma from one elected lane of a
//     converged warp, warps 2..5 convert each int8 tile into a bf16 SW128
//     operand tile (exactly: bytes re-biased into fp32 with a byte permute,
//     one FADD, top 16 bits kept) and afterwards run the epilogue.
//   * Split-K over a thread-block cluster when M is small: each CTA
//     accumulates a K range in TMEM, pushes its fp32 partial into the owning
//     CTA's shared memory (owner = a block of token columns) with remote
//     stores, and each owner sums, applies the epilogue and stores coalesced
//     rows of Y. No global scratch.
//   * Every mbarrier wait is bounded (1 s) and records SFB_ERR_DEVICE_TIMEOUT.
#include "common.cuh"
#include "sm100_ptx.cuh"

namespace sfb {

struct W8Params {
    const float*   w_scale;
    const void*    bias;          // bf16 [N] or nullptr
    const void*    residual;      // bf16 [M, N] (row stride ldr) or nullptr
    void*          y;             // bf16 or fp32
    int64_t        ldy, ldr;
    int32_t        M, N, K;
    int32_t        bn;            // MMA N (tokens per CTA), multiple of 32, <= 256
    int32_t        kchunks;       // K / 64
    int32_t        splits;        // cluster size along grid.x
    int32_t        act;           // 0 none, 1 GELU (tanh), 2 SiLU
    int32_t        y_f32;         // 1: fp32 output
};

namespace w8 {

constexpr int kThreads  = 6 * 32;
constexpr int kStages   = 4;
constexpr int kWBytes   = 128 * 64;            // int8 weight tile
constexpr int kWbBytes  = 128 * 128;           // bf16 weight tile (SW128)
constexpr int kXBytes   = 256 * 128;           // bf16 activation tile, up to 256 rows
constexpr int kOffX     = 0;
constexpr int kOffWb    = kOffX + kStages * kXBytes;
constexpr int kOffW     = kOffWb + kStages * kWbBytes;
constexpr int kOffBar   = kOffW + kStages * kWBytes;
constexpr int kOffTmem  = kOffBar + 8 * 24;
constexpr int kSmemUsed = kOffTmem + 16;
constexpr int kSmemBytes = kSmemUsed + 1024;
// Split-K merge buffer (only when splits > 1, bn <= 128) reuses the X ring:
// [C sources][128 rows][ceil(bn/C) + 1 columns] fp32 <= 128 · 160 · 4 bytes.
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

__host__ __device__ constexpr int bar_full(int s)  { return s; }                 // W int8 + X landed
__host__ __device__ constexpr int bar_conv(int s)  { return kStages + s; }       // W bf16 ready
__host__ __device__ constexpr int bar_empty(int s) { return 2 * kStages + s; }   // stage consumed by MMA
constexpr int kBarAcc = 3 * kStages;                                             // accumulator done

__device__ __forceinline__ float gelu_tanh(float x) {
    const float k0 = 0.7978845608028654f, k1 = 0.044715f;   // sqrt(2/pi), GELU tanh form
    return 0.5f * x * (1.f + tanhf(k0 * fmaf(k1 * x * x, x, x)));
}

__global__ void __launch_bounds__(kThreads, 1)
w8a16_gemm_kernel(const __grid_constant__ CUtensorMap tmX,
                  const __grid_constant__ CUtensorMap tmW,
                  const W8Params p) {
    using namespace ptx;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kOffTmem);
    auto sX  = [&](int s) { return smem + kOffX + s * kXBytes; };
    auto sWb = [&](int s) { return smem + kOffWb + s * kWbBytes; };
    auto sW  = [&](int s) { return smem + kOffW + s * kWBytes; };

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = blockIdx.x;
    const int n0 = blockIdx.y * 128;
    const int m0 = blockIdx.z * p.bn;
    // this CTA's share of the 64-wide K chunks
    const int cbase = p.kchunks / p.splits, crem = p.kchunks - cbase * p.splits;
    const int c_begin = split * cbase + min(split, crem);
    const int nch = cbase + (split < crem ? 1 : 0);

    if (tid == 32) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars[bar_full(s)], 1);
            mbar_init(&bars[bar_conv(s)], 4);
            mbar_init(&bars[bar_empty(s)], 1);
        }
        mbar_init(&bars[kBarAcc], 1);
        fence_mbarrier_init();
        tma_prefetch_desc(&tmX);
        tma_prefetch_desc(&tmW);
    }
    if (warp == 0) {
        tmem_alloc(tmem_holder, 256);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem = *tmem_holder;

    bool ok = true;
    auto wait = [&](int bar, uint32_t parity) {
        if (!mbar_wait(&bars[bar], parity, ok ? 1000000000ull : 0ull)) ok = false;
    };
    const uint32_t xbytes = static_cast<uint32_t>(p.bn) * 128u;

    if (warp == 0) {
        // ── TMA producer ────────────────────────────────────────────────────
        for (int c = 0; c < nch; ++c) {
            const int s = c % kStages;
            if (c >= kStages) wait(bar_empty(s), ((c / kStages) - 1) & 1);
            if (elect_one()) {
                mbar_arrive_expect_tx(&bars[bar_full(s)], kWBytes + xbytes);
                const int k0 = (c_begin + c) * 64;
                tma_load_2d(sW(s), &tmW, &bars[bar_full(s)], k0, n0);
                tma_load_2d(sX(s), &tmX, &bars[bar_full(s)], k0, m0);
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        // ── MMA issuer ──────────────────────────────────────────────────────
        const uint32_t idesc = idesc_f16(128, static_cast<uint32_t>(p.bn), 1, 0, 0);
        for (int c = 0; c < nch; ++c) {
            const int s = c % kStages;
            wait(bar_conv(s), (c / kStages) & 1);
            tc_fence_after_sync();
            const uint32_t aw = smem_u32(sWb(s)), ax = smem_u32(sX(s));
            if (elect_one()) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    mma_f16_ss(tmem, smem_desc_sw128(aw + kk * 32, 16, 1024),
                               smem_desc_sw128(ax + kk * 32, 16, 1024), idesc,
                               (c > 0 || kk > 0) ? 1u : 0u);
                mma_commit(&bars[bar_empty(s)]);
                if (c == nch - 1) mma_commit(&bars[kBarAcc]);
            }
            __syncwarp();
        }
    } else {
        // ── converters: int8 [128 × 64] → bf16 SW128 [128 × 64] ──────────────
        const int ct = tid - 64;                       // 0..127
        for (int c = 0; c < nch; ++c) {
            const int s = c % kStages;
            wait(bar_full(s), (c / kStages) & 1);
            const uint8_t* src = sW(s);
            uint8_t* dst = sWb(s);
#pragma unroll 2
            for (int it = 0; it < 8; ++it) {
                const int unit = it * 128 + ct;        // (row, 8-element chunk)
                const int r = unit >> 3, ch = unit & 7;
                const uint2 raw = *reinterpret_cast<const uint2*>(src + r * 64 + ch * 8);
                uint32_t o[4];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t x = (h ? raw.y : raw.x) ^ 0x80808080u;   // q + 128, unsigned
                    // 0x4B0000bb = 2^23 + bb as fp32; minus (2^23 + 128) gives q exactly
                    const float f0 = __uint_as_float(ptx::prmt(x, 0x4B000000u, 0x7440u)) - 8388736.f;
                    const float f1 = __uint_as_float(ptx::prmt(x, 0x4B000000u, 0x7441u)) - 8388736.f;
                    const float f2 = __uint_as_float(ptx::prmt(x, 0x4B000000u, 0x7442u)) - 8388736.f;
                    const float f3 = __uint_as_float(ptx::prmt(x, 0x4B000000u, 0x7443u)) - 8388736.f;
                    o[2 * h]     = ptx::prmt(__float_as_uint(f0), __float_as_uint(f1), 0x7632u);
                    o[2 * h + 1] = ptx::prmt(__float_as_uint(f2), __float_as_uint(f3), 0x7632u);
                }
                *reinterpret_cast<uint4*>(dst + r * 128 + ((ch ^ (r & 7)) << 4)) =
                    make_uint4(o[0], o[1], o[2], o[3]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[bar_conv(s)]);
        }
    }

    // ── epilogue (warps 2..5: TMEM lane window = warp % 4) ───────────────────
    const bool epi = warp >= 2;
    const int win = warp & 3;
    const int nrow = n0 + win * 32 + lane;             // output channel of this thread
    const uint32_t lane_off = static_cast<uint32_t>(win * 32) << 16;
    float sc = 0.f, bi = 0.f;
    if (epi && nrow < p.N) {
        sc = p.w_scale[nrow];
        if (p.bias) bi = __bfloat162float(static_cast<const __nv_bfloat16*>(p.bias)[nrow]);
    }
    auto finish = [&](float acc, int m) {
        float y = fmaf(acc, sc, bi);
        if (p.act == 1) y = gelu_tanh(y);
        else if (p.act == 2) y = y / (1.f + expf(-y));          // SiLU
        if (p.residual)
            y += __bfloat162float(static_cast<const __nv_bfloat16*>(p.residual)[m * p.ldr + nrow]);
        if (p.y_f32) static_cast<float*>(p.y)[m * p.ldy + nrow] = y;
        else static_cast<__nv_bfloat16*>(p.y)[m * p.ldy + nrow] = __float2bfloat16_rn(y);
    };
    if (epi && nch > 0) {
        wait(kBarAcc, 0);
        tc_fence_after_sync();
    }
    const int mvalid = min(p.bn, p.M - m0);
    if (p.splits == 1) {
        if (epi) {
#pragma unroll 1
            for (int c0 = 0; c0 < p.bn; c0 += 32) {
                float v[32];
                if (nch > 0) { tmem_ld32(tmem + lane_off + c0, v); tmem_ld_wait(); }
                else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = 0.f;
                }
                if (nrow < p.N && ok) {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (c0 + i < mvalid) finish(v[i], m0 + c0 + i);
                }
            }
        }
    } else {
        // Split-K merge: CTA r owns token columns [bn·r/C, bn·(r+1)/C). Every CTA
        // pushes its partial rows of each owner's columns into that owner's
        // buffer [C sources][128 rows][cols]; one cluster barrier publishes them.
        const int C = p.splits;
        const int cs = (p.bn + C - 1) / C + 1;         // merge slice stride (floats)
        float* buf = reinterpret_cast<float*>(smem + kOffX);
        cluster_sync();   // every CTA's MMAs are done and its X ring is free
        if (epi) {
            const int row = win * 32 + lane;
#pragma unroll 1
            for (int c0 = 0; c0 < p.bn; c0 += 32) {
                float v[32];
                if (nch > 0) { tmem_ld32(tmem + lane_off + c0, v); tmem_ld_wait(); }
                else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = 0.f;
                }
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int col = c0 + i;
                    const int owner = (col * C) / p.bn;
                    const int lo = (p.bn * owner + C - 1) / C;
                    const uint32_t a = smem_u32(buf + (split * 128 + row) * cs + (col - lo));
                    dsmem_st_f32(dsmem_map(a, owner), v[i]);
                }
            }
        }
        cluster_sync();
        if (epi && nrow < p.N && ok) {
            const int row = win * 32 + lane;
            const int lo = (p.bn * split + C - 1) / C, hi = (p.bn * (split + 1) + C - 1) / C;
            for (int col = lo; col < hi && col < mvalid; ++col) {
                float acc = 0.f;
                for (int r = 0; r < C; ++r) acc += buf[(r * 128 + row) * cs + (col - lo)];
                finish(acc, m0 + col);
            }
        }
    }

    if (!ok) atomicExch(&g_sfb_device_error, SFB_ERR_DEVICE_TIMEOUT);
    tc_fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after_sync();
        tmem_dealloc(tmem, 256);
    }
}

}  // namespace w8

int w8a16_gemm_launch(const void* x, int64_t ldx, const int8_t* w, const float* w_scale,
                      const void* bias, const void* residual, int64_t ldr, void* y, int64_t ldy,
                      int32_t y_dtype, int32_t M, int32_t N, int32_t K, int32_t act,
                      int32_t num_splits, cudaStream_t stream) {
    if (x == nullptr || w == nullptr || w_scale == nullptr || y == nullptr) return SFB_ERR_INVALID;
    if (M < 0 || N <= 0 || K <= 0) return SFB_ERR_SHAPE;
    if (M == 0) return SFB_OK;
    if (K % 64 != 0 || N % 32 != 0) return SFB_ERR_SHAPE;
    if (y_dtype != SFB_BF16 && y_dtype != SFB_F32) return SFB_ERR_DTYPE;
    if (act < 0 || act > 2) return SFB_ERR_INVALID;
    auto aligned16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
    if (!aligned16(x) || !aligned16(w) || (ldx * 2) % 16 != 0) return SFB_ERR_ALIGN;
    if (residual != nullptr && ldr < N) return SFB_ERR_SHAPE;
    if (ldy < N) return SFB_ERR_SHAPE;
    const DeviceInfo& dev = device_info();
    if (!is_sm100(dev)) return SFB_ERR_UNSUPPORTED;

    W8Params p{};
    p.w_scale = w_scale; p.bias = bias; p.residual = residual; p.y = y;
    p.ldy = ldy; p.ldr = ldr; p.M = M; p.N = N; p.K = K;
    p.act = act; p.y_f32 = y_dtype == SFB_F32 ? 1 : 0;
    p.kchunks = K / 64;
    // tokens per CTA: round up to 32, at most 256
    p.bn = M >= 256 ? 256 : ((M + 31) / 32) * 32;
    const int ntile = (N + 127) / 128, mtile = (M + p.bn - 1) / p.bn;
    int splits = num_splits;
    if (splits <= 0) {
        splits = 1;
        if (p.bn <= 128) {
            const int units = ntile * mtile;
            splits = std::max(1, dev.num_sms / std::max(units, 1));
            splits = std::min(splits, 8);
            splits = std::min(splits, std::max(1, p.kchunks / 2));
        }
    }
    if (splits > 1 && p.bn > 128) return SFB_ERR_INVALID;
    p.splits = std::min(std::min(splits, 16), p.kchunks);

    CUtensorMap mx, mw;
    {
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
        cuuint64_t str[1] = {(cuuint64_t)(ldx * 2)};
        cuuint32_t box[2] = {64, (cuuint32_t)p.bn};
        cuuint32_t es[2] = {1, 1};
        int rc = encode_tensor_map(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x),
                                   dims, str, box, es, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc != SFB_OK) return rc;
    }
    {
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
        cuuint64_t str[1] = {(cuuint64_t)K};
        cuuint32_t box[2] = {64, 128};
        cuuint32_t es[2] = {1, 1};
        int rc = encode_tensor_map(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(w),
                                   dims, str, box, es, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc != SFB_OK) return rc;
    }
    static bool attr_done[64] = {};
    if (!attr_done[dev.ordinal & 63]) {
        cudaError_t e1 = cudaFuncSetAttribute(w8::w8a16_gemm_kernel,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, w8::kSmemBytes);
        cudaError_t e2 = cudaFuncSetAttribute(w8::w8a16_gemm_kernel,
                                              cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e1 != cudaSuccess || e2 != cudaSuccess) {
            (void)cudaGetLastError();
            record_cuda_error(e1 != cudaSuccess ? e1 : e2, "w8a16 kernel attributes");
            return SFB_ERR_CUDA;
        }
        attr_done[dev.ordinal & 63] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.splits, ntile, mtile);
    cfg.blockDim = dim3(w8::kThreads, 1, 1);
    cfg.dynamicSmemBytes = w8::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = p.splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, w8::w8a16_gemm_kernel, mx, mw, p);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        record_cuda_error(e, "w8a16 gemm launch");
        return SFB_ERR_LAUNCH;
    }
    return SFB_OK;
}

}  // namespace sfb
