// w8a16_gemm.cu — int8-weight GEMM with the dequantisation fused in, for the
// RDT-1B projections (sm_100a, tcgen05 + TMA).
//
//   Y[m, n] = act( s[n] · Σ_k X[m, k] · Wq[n, k] + bias[n] ) + R[m, n]
//
// X: bf16 activations [M, K] (row stride ldx); Wq: int8 weights [N, K]
// (row-major, one row per output channel, contiguous); s: fp32 per-output-
// channel scales; bias: optional bf16 [N]; act: none, GELU (tanh form) or SiLU;
// R: optional residual [M, N] in Y's dtype (may alias Y); Y: bf16 or fp32 [M, N].
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
//   * Warp roles per CTA (10 warps): warp 0 issues TMA (int8 weight tile
//     [128 × 64] without swizzle, bf16 activation tile [N × 64] with 128-byte
//     swizzle), warp 1 issues tcgen05.mma from one elected lane of a
//     converged warp, warps 2..9 convert each int8 tile into a bf16 SW128
//     operand tile (exactly: bytes re-biased into fp32 with a byte permute,
//     one FADD, top 16 bits kept) and afterwards run the epilogue, staged
//     through shared memory so that Y is written in 16-byte vectors.
//   * Split-K over a thread-block cluster when M is small: each CTA
//     accumulates a K range in TMEM and stores its scaled fp32 partial from
//     registers straight into the owning CTA's shared memory (owner = a
//     block of TM / C channel rows) with distributed-shared-memory stores;
//     one cluster barrier publishes them, and each owner sums, applies the
//     epilogue and stores coalesced rows of Y. No global scratch.
//   * Every mbarrier wait is bounded (1 s) and records SFB_ERR_DEVICE_TIMEOUT.
#include "common.cuh"
#include "sm100_ptx.cuh"

#include <mutex>
#include <utility>
#include <vector>

namespace sfb {

struct W8Params {
    const float*   w_scale;
    const void*    bias;          // bf16 [N] or nullptr
    const void*    residual;      // [M, N] (row stride ldr) in y's dtype, or nullptr
    void*          y;             // bf16 or fp32
    int64_t        ldy, ldr;
    int32_t        M, N, K;
    int32_t        bn;            // MMA N (tokens per CTA), multiple of 32, <= 256
    int32_t        kchunks;       // K / 64
    int32_t        splits;        // cluster size along grid.x
    int32_t        y_f32;         // 1: fp32 output
    int32_t        stages;        // pipeline depth, kRingBytes / stage bytes, at most kMaxStages
    int32_t        rcv_off;       // split-K: byte offset of the receive area (past the ring)
#ifdef SFB_TRACE
    unsigned long long* trace;
    unsigned long long* tl;
    int tl_launch;
#endif
};

namespace w8 {

#ifdef SFB_TRACE
#define W8_T(slot, i) do { if (p.trace && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && (i) < 64) \
        p.trace[(slot) * 64 + (i)] = ptx::global_timer_ns(); } while (0)
#else
#define W8_T(slot, i) do { } while (0)
#endif

constexpr int kThreads  = 10 * 32;        // TMA, MMA, 8 converter/epilogue warps
constexpr int kConvWarps = 8;
constexpr int kStageStride = 36;           // floats per row of an epilogue staging block
constexpr int kMaxStages = 8;
// Weight tiles are TM = 128 or 64 output channels (MMA M) × 64 K elements.
__host__ __device__ constexpr int w_bytes(int tm) { return tm * 64; }     // int8 weight tile
__host__ __device__ constexpr int wb_bytes(int tm) { return tm * 128; }   // bf16 weight tile (SW128)
// One ring area split into `stages` X tiles (bn · 128 B, bn <= 256), then as
// many bf16 and int8 weight tiles; the depth follows the token tile: 4 stages
// at bn = 256, 6 at 96, 8 at 64 and below.
constexpr int kRingBytes = 224 * 1024;
constexpr int kOffBar   = kRingBytes;
constexpr int kOffTmem  = kOffBar + 8 * (4 * kMaxStages + 2);
constexpr int kSmemUsed = kOffTmem + 16;
constexpr int kSmemBytes = kSmemUsed + 1024;
// Split-K (splits > 1, bn <= 128) shortens the ring by the stages that a
// TM × bn fp32 receive area needs; peers store their partials into it.
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

__host__ __device__ constexpr int stage_bytes(int bn, int tm) { return w_bytes(tm) + wb_bytes(tm) + bn * 128; }
__host__ __device__ constexpr int num_stages(int bn, int tm) {
    return kRingBytes / stage_bytes(bn, tm) < kMaxStages ? kRingBytes / stage_bytes(bn, tm) : kMaxStages;
}
static_assert(num_stages(256, 128) >= 4, "four stages at the widest token tile");

__host__ __device__ constexpr int bar_full_w(int s) { return s; }                    // W int8 landed
__host__ __device__ constexpr int bar_full_x(int s) { return kMaxStages + s; }       // X landed
__host__ __device__ constexpr int bar_conv(int s)  { return 2 * kMaxStages + s; }    // W bf16 ready
__host__ __device__ constexpr int bar_empty(int s) { return 3 * kMaxStages + s; }    // stage consumed by MMA
constexpr int kBarAcc = 4 * kMaxStages;                                              // accumulator done
constexpr int kBarDrain = kBarAcc + 1;             // failure path: every MMA issued so far has completed
constexpr uint64_t kDrainNs = 100000000ull;        // bound of each wait for in-flight copies/MMAs after a failure

__device__ __forceinline__ float gelu_tanh(float x) {
    const float k0 = 0.7978845608028654f, k1 = 0.044715f;   // sqrt(2/pi), GELU tanh form
    return 0.5f * x * (1.f + tanhf(k0 * fmaf(k1 * x * x, x, x)));
}

// Eight residual values R[m, n..n+7] in fp32 (R has Y's dtype); zeros when !use.
__device__ __forceinline__ void load_res8(const W8Params& p, int m, int n, bool use, float (&r)[8]) {
    if (!use) {
#pragma unroll
        for (int k = 0; k < 8; ++k) r[k] = 0.f;
        return;
    }
    if (p.y_f32) {
        const float* src = static_cast<const float*>(p.residual) + static_cast<int64_t>(m) * p.ldr + n;
        const float4 a = *reinterpret_cast<const float4*>(src);
        const float4 b = *reinterpret_cast<const float4*>(src + 4);
        r[0] = a.x; r[1] = a.y; r[2] = a.z; r[3] = a.w; r[4] = b.x; r[5] = b.y; r[6] = b.z; r[7] = b.w;
    } else {
        const uint4 u = *reinterpret_cast<const uint4*>(
            static_cast<const __nv_bfloat16*>(p.residual) + static_cast<int64_t>(m) * p.ldr + n);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int k = 0; k < 4; ++k) { const float2 f = __bfloat1622float2(h[k]); r[2 * k] = f.x; r[2 * k + 1] = f.y; }
    }
}

// kAct: 0 none, 1 GELU (tanh), 2 SiLU; kSplit: K split across a cluster;
// kTM: output channels per CTA (MMA M), 128 or 64. With M = 64 the
// accumulator row r sits in TMEM lane 32·(r / 16) + r % 16 (lanes 16..31 of
// each 32-lane window unused; measured on B200). Each instantiation carries
// only its own epilogue path.
template <int kAct, bool kSplit, int kTM>
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
    const int nst = p.stages;
    const int xtile = p.bn * 128;
    auto sX  = [&](int s) { return smem + s * xtile; };
    constexpr int kWB = w_bytes(kTM), kWBB = wb_bytes(kTM);
    constexpr int kRowsPerWin = kTM / 4;               // accumulator rows per 32-lane TMEM window
    auto sWb = [&](int s) { return smem + nst * xtile + s * kWBB; };
    auto sW  = [&](int s) { return smem + nst * (xtile + kWBB) + s * kWB; };

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = blockIdx.x;
    const int n0 = blockIdx.y * kTM;
    const int m0 = blockIdx.z * p.bn;
    // this CTA's share of the 64-wide K chunks
    const int cbase = p.kchunks / p.splits, crem = p.kchunks - cbase * p.splits;
    const int c_begin = split * cbase + min(split, crem);
    const int nch = cbase + (split < crem ? 1 : 0);
    // CTAs of different channel tiles walk their K range from different
    // chunks, so the activation tile each one loads at a given moment differs
    // (all channel tiles read the same activations; in lockstep they queue on
    // the same L2 slices).
    const int rot = nch > 0 ? static_cast<int>(blockIdx.y) % nch : 0;
    auto kchunk = [&](int c) { const int r = c + rot; return c_begin + (r >= nch ? r - nch : r); };

#ifdef SFB_TRACE
    const uint64_t cta_t0 = ptx::global_timer_ns();
#endif
    if (tid == 32) {
        for (int s = 0; s < nst; ++s) {
            mbar_init(&bars[bar_full_w(s)], 1);
            mbar_init(&bars[bar_full_x(s)], 1);
            mbar_init(&bars[bar_conv(s)], kConvWarps / 2);
            mbar_init(&bars[bar_empty(s)], 1);
        }
        mbar_init(&bars[kBarAcc], 1);
        mbar_init(&bars[kBarDrain], 1);
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
    // split-K: announce this CTA as started; the wait before the first store
    // into a peer's shared memory then guarantees every peer is running
    if constexpr (kSplit) cluster_arrive_relaxed();
    pdl_trigger();                                     // TMEM is held: the next kernel may start

#ifdef SFB_TRACE
    unsigned long long tl_t1 = 0;
#endif
    bool ok = true;
    auto wait = [&](int bar, uint32_t parity) {
        if (!mbar_wait(&bars[bar], parity, ok ? 1000000000ull : 0ull)) ok = false;
    };
    const uint32_t xbytes = static_cast<uint32_t>(p.bn) * 128u;

    if (warp == 0) {
        // ── TMA producer ────────────────────────────────────────────────────
        // The int8 weights of the first stages are constant and are fetched
        // before waiting for the previous kernel; activations after.
        const int pre = min(nch, nst);
        const uint64_t wpol = l2_evict_first_policy();   // weights are read once per step
        if (elect_one()) {
            for (int c = 0; c < pre; ++c) {
                mbar_arrive_expect_tx(&bars[bar_full_w(c)], kWB);
                tma_load_2d_hint(sW(c), &tmW, &bars[bar_full_w(c)], kchunk(c) * 64, n0, wpol);
            }
        }
        __syncwarp();
        pdl_wait();
#ifdef SFB_TRACE
        tl_t1 = ptx::global_timer_ns();
#endif
        int issued = 0;                                 // chunks whose X load (and W load) is issued
        for (int c = 0; c < nch; ++c) {
            const int s = c % nst;
            if (c >= nst) wait(bar_empty(s), ((c / nst) - 1) & 1);
            if (!ok) break;                             // a wait expired: issue nothing more
            issued = c + 1;
            if (elect_one()) {
                const int k0 = kchunk(c) * 64;
                if (c >= nst) {
                    mbar_arrive_expect_tx(&bars[bar_full_w(s)], kWB);
                    tma_load_2d_hint(sW(s), &tmW, &bars[bar_full_w(s)], k0, n0, wpol);
                }
                mbar_arrive_expect_tx(&bars[bar_full_x(s)], xbytes);
                tma_load_2d(sX(s), &tmX, &bars[bar_full_x(s)], k0, m0);
                W8_T(0, c);
            }
            __syncwarp();
        }
        // Copies in flight must land before the CTA releases its shared memory:
        // wait (bounded, also after a failure) for the last stages issued. On the
        // normal path the MMA warp has consumed them all and these return at once.
        const int wissued = max(issued, pre);
        for (int c = max(0, wissued - nst); c < wissued; ++c)
            if (!mbar_wait(&bars[bar_full_w(c % nst)], (c / nst) & 1, kDrainNs)) ok = false;
        for (int c = max(0, issued - nst); c < issued; ++c)
            if (!mbar_wait(&bars[bar_full_x(c % nst)], (c / nst) & 1, kDrainNs)) ok = false;
    } else if (warp == 1) {
        // ── MMA issuer ──────────────────────────────────────────────────────
        const uint32_t idesc = idesc_f16(kTM, static_cast<uint32_t>(p.bn), 1, 0, 0);
        for (int c = 0; c < nch; ++c) {
            const int s = c % nst;
            wait(bar_conv(s), (c / nst) & 1);
            wait(bar_full_x(s), (c / nst) & 1);
            if (!ok) break;                             // a wait expired: issue nothing more
            tc_fence_after_sync();
            const uint32_t aw = smem_u32(sWb(s)), ax = smem_u32(sX(s));
            if (elect_one()) {
                W8_T(3, c);
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
        if (!ok) {
            // every MMA issued so far completes before TMEM is released
            if (elect_one()) mma_commit(&bars[kBarDrain]);
            __syncwarp();
            mbar_wait(&bars[kBarDrain], 0, kDrainNs);
        }
    } else {
        // ── converters: int8 [TM × 64] → bf16 SW128 [TM × 64] ────────────────
        // Two groups of four warps take alternate chunks, so the conversion
        // latency of one chunk overlaps the next.
        const int grp = (warp - 2) >> 2;
        const int ct = tid - 64 - grp * 128;           // 0..127
        for (int c = grp; c < nch; c += 2) {
            const int s = c % nst;
            wait(bar_full_w(s), (c / nst) & 1);
            if (ct == 0) W8_T(1, c);
            const uint8_t* src = sW(s);
            uint8_t* dst = sWb(s);
            constexpr int kIt = kTM / 16;              // 8-byte units per thread
            uint2 raw[kIt];
#pragma unroll
            for (int it = 0; it < kIt; ++it) {         // all loads first: independent
                const int unit = it * 128 + ct;        // (row, 8-element chunk)
                raw[it] = *reinterpret_cast<const uint2*>(src + (unit >> 3) * 64 + (unit & 7) * 8);
            }
#pragma unroll
            for (int it = 0; it < kIt; ++it) {
                const int unit = it * 128 + ct;
                const int r = unit >> 3, ch = unit & 7;
                uint32_t o[4];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t x = (h ? raw[it].y : raw[it].x) ^ 0x80808080u;   // q + 128, unsigned
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
            if (ct == 0) W8_T(2, c);
        }
    }

    // ── epilogue (warps 2..9: TMEM lane window = warp % 4, column half hh) ───
    const bool epi = warp >= 2;
    const int win = warp & 3;
    const int hh = (warp - 2) >> 2;                    // 0: warps 2..5, 1: warps 6..9
    const bool lane_ok = kTM == 128 || lane < 16;     // lane holds an accumulator row
    const int trow = win * kRowsPerWin + lane;          // tile row (output channel) of this thread
    const int nrow = n0 + trow;
    const uint32_t lane_off = static_cast<uint32_t>(win * 32) << 16;
    float sc = 0.f, bi = 0.f;
    if (epi && lane_ok && nrow < p.N) {
        sc = p.w_scale[nrow];
        if (p.bias) bi = __bfloat162float(static_cast<const __nv_bfloat16*>(p.bias)[nrow]);
    }
    auto act = [](float y) {
        if constexpr (kAct == 1) return gelu_tanh(y);
        else if constexpr (kAct == 2) return y / (1.f + expf(-y));    // SiLU
        else return y;
    };
    if (tid == 64) W8_T(4, 0);
    pdl_wait();                                        // before the residual read and the output write
    const int mvalid = min(p.bn, p.M - m0);
    // Split-K owner pass: the residual rows this thread adds, loaded while the
    // MMAs finish.
    const int seg_per_row = (kTM / p.splits) / 8;      // 8-channel segments per owned row
    const int nunits = mvalid * seg_per_row;
    constexpr int kMaxIt = 4;                          // (128 tokens · 8 segs) / 256 threads
    float rres[kMaxIt][8];
    if constexpr (kSplit) {
        if (epi) {
            const int nb = n0 + split * (kTM / p.splits);
#pragma unroll
            for (int it = 0; it < kMaxIt; ++it) {
                const int u = tid - 64 + it * kConvWarps * 32;
                const int mm = u / seg_per_row, n = nb + (u - mm * seg_per_row) * 8;
                load_res8(p, m0 + mm, n, p.residual && u < nunits && n < p.N, rres[it]);
            }
        }
    }
    if (epi && nch > 0) {
        wait(kBarAcc, 0);
        tc_fence_after_sync();
    }
    if (tid == 64) W8_T(4, 1);
    if constexpr (!kSplit) {
        // Each warp takes 32-column blocks c0 = 32·hh, 32·hh + 64, ...: TMEM →
        // act(acc·s + b) staged as fp32 [32 tokens][32 channels] in shared memory
        // (the bf16 weight ring, idle now), then written as 16-byte vectors of 8
        // channels per token row, with the residual added in the same pass.
        if (epi) {
            float* stg = reinterpret_cast<float*>(smem) + (warp - 2) * 32 * kStageStride;
            const int nb = n0 + win * kRowsPerWin;      // first channel of this warp
            constexpr int kSegs = kRowsPerWin / 8;      // 8-channel segments per token row
            constexpr int kRowsPass = 32 / kSegs;       // token rows written per pass
#pragma unroll 1
            for (int c0 = 32 * hh; c0 < p.bn; c0 += 64) {
                float v[32];
                if (nch > 0) { tmem_ld32(tmem + lane_off + c0, v); tmem_ld_wait(); }
                else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = 0.f;
                }
#pragma unroll
                for (int i = 0; i < 32; ++i) stg[i * kStageStride + lane] = act(fmaf(v[i], sc, bi));
                __syncwarp();
#pragma unroll
                for (int j = 0; j < 32 / kRowsPass; ++j) {
                    const int r = j * kRowsPass + lane / kSegs, seg = (lane % kSegs) * 8;   // token row, 8 channels
                    const int m = m0 + c0 + r, n = nb + seg;
                    if (c0 + r < mvalid && n < p.N && ok) {
                        const float4 a = *reinterpret_cast<const float4*>(stg + r * kStageStride + seg);
                        const float4 b = *reinterpret_cast<const float4*>(stg + r * kStageStride + seg + 4);
                        float y[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
                        if (p.residual) {
                            float rr[8];
                            load_res8(p, m, n, true, rr);
#pragma unroll
                            for (int k = 0; k < 8; ++k) y[k] += rr[k];
                        }
                        if (p.y_f32) {
                            float* dst = static_cast<float*>(p.y) + m * p.ldy + n;
                            *reinterpret_cast<float4*>(dst) = make_float4(y[0], y[1], y[2], y[3]);
                            *reinterpret_cast<float4*>(dst + 4) = make_float4(y[4], y[5], y[6], y[7]);
                        } else {
                            uint4 o;
                            __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
                            for (int k = 0; k < 4; ++k) o2[k] = __floats2bfloat162_rn(y[2 * k], y[2 * k + 1]);
                            *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.y) + m * p.ldy + n) = o;
                        }
                    }
                }
                __syncwarp();
            }
        }
    } else {
        // Split-K merge. CTA r owns channel rows [r·R, (r+1)·R) of the
        // tile, R = TM / C; its receive area holds [C sources][bn tokens][R].
        const int C = p.splits, R = kTM / C;
        const int slice = p.bn * R;
        float* rcv = reinterpret_cast<float*>(smem + p.rcv_off);
        cluster_wait();                                 // every peer has started (arrived after its setup)
        if (epi) {
            const float bsplit = split == 0 ? bi : 0.f;     // the bias once, from CTA 0
            const int owner = trow / R, slot = trow - owner * R;
            float v[2][32];
            const int c0a = 32 * hh, c0b = 32 * hh + 64;
            if (nch > 0) {
                if (c0a < p.bn) tmem_ld32(tmem + lane_off + c0a, v[0]);
                if (c0b < p.bn) tmem_ld32(tmem + lane_off + c0b, v[1]);
                tmem_ld_wait();
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) { v[0][i] = 0.f; v[1][i] = 0.f; }
            }
            if (lane_ok) {
                // this thread's channel row, every token, into its owner's slot
                const uint32_t base = dsmem_map(smem_u32(rcv + split * slice + slot), static_cast<uint32_t>(owner));
                const uint32_t step = static_cast<uint32_t>(R) * 4u;
                if (c0a < p.bn) {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (c0a + i < p.bn) dsmem_st_f32(base + (c0a + i) * step, fmaf(v[0][i], sc, bsplit));
                }
                if (c0b < p.bn) {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (c0b + i < p.bn) dsmem_st_f32(base + (c0b + i) * step, fmaf(v[1][i], sc, bsplit));
                }
            }
        }
        if (tid == 64) W8_T(4, 3);
        cluster_sync();                                 // every partial is in its owner (release / acquire)
        if (tid == 64) W8_T(4, 5);
        if (epi) {
            const int nb = n0 + split * R;              // first channel owned here
#pragma unroll
            for (int it = 0; it < kMaxIt; ++it) {
                const int u = tid - 64 + it * kConvWarps * 32;
                const int mm = u / seg_per_row, seg = (u - mm * seg_per_row) * 8;
                const int n = nb + seg, m = m0 + mm;
                if (u >= nunits || n >= p.N || !ok) continue;
                float y[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) y[k] = 0.f;
#pragma unroll 1
                for (int r = 0; r < C; ++r) {
                    const float* src = rcv + r * slice + mm * R + seg;
                    const float4 a4 = *reinterpret_cast<const float4*>(src);
                    const float4 b4 = *reinterpret_cast<const float4*>(src + 4);
                    y[0] += a4.x; y[1] += a4.y; y[2] += a4.z; y[3] += a4.w;
                    y[4] += b4.x; y[5] += b4.y; y[6] += b4.z; y[7] += b4.w;
                }
#pragma unroll
                for (int k = 0; k < 8; ++k) y[k] = act(y[k]) + rres[it][k];   // zero without a residual
                if (p.y_f32) {
                    float* dst = static_cast<float*>(p.y) + m * p.ldy + n;
                    *reinterpret_cast<float4*>(dst) = make_float4(y[0], y[1], y[2], y[3]);
                    *reinterpret_cast<float4*>(dst + 4) = make_float4(y[4], y[5], y[6], y[7]);
                } else {
                    uint4 o;
                    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
                    for (int k = 0; k < 4; ++k) o2[k] = __floats2bfloat162_rn(y[2 * k], y[2 * k + 1]);
                    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.y) + m * p.ldy + n) = o;
                }
            }
        }
        if (tid == 64) W8_T(4, 6);
        // (no second barrier: nothing reads or writes another CTA's memory now)
    }

    if (tid == 64) W8_T(4, 2);
#ifdef SFB_TRACE
    if (p.trace && tid == 64) {
        const int cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
        if (cta < 1024) { p.trace[1024 + 2 * cta] = cta_t0; p.trace[1025 + 2 * cta] = ptx::global_timer_ns(); }
    }
#endif
    if (!ok) atomicExch(&g_sfb_device_error, SFB_ERR_DEVICE_TIMEOUT);
    tc_fence_before_sync();
    __syncthreads();
#ifdef SFB_TRACE
    tl_record(p.tl, p.tl_launch, kSplit ? 2 : 1, cta_t0, tl_t1);
#endif
    if (warp == 0) {
        tc_fence_after_sync();
        tmem_dealloc(tmem, 256);
    }
}

using KernFn = void (*)(CUtensorMap, CUtensorMap, W8Params);

inline KernFn pick(int act, bool split, int tm) {
    static const KernFn t[2][3][2] = {
        {{w8a16_gemm_kernel<0, false, 128>, w8a16_gemm_kernel<0, true, 128>},
         {w8a16_gemm_kernel<1, false, 128>, w8a16_gemm_kernel<1, true, 128>},
         {w8a16_gemm_kernel<2, false, 128>, w8a16_gemm_kernel<2, true, 128>}},
        {{w8a16_gemm_kernel<0, false, 64>, w8a16_gemm_kernel<0, true, 64>},
         {w8a16_gemm_kernel<1, false, 64>, w8a16_gemm_kernel<1, true, 64>},
         {w8a16_gemm_kernel<2, false, 64>, w8a16_gemm_kernel<2, true, 64>}}};
    return t[tm == 64 ? 1 : 0][act][split ? 1 : 0];
}


}  // namespace w8

#ifdef SFB_TRACE
static unsigned long long* g_w8_trace = nullptr;
static int g_w8_trace_launch = -1;        // trace only this timeline launch index (-1: every launch)
extern "C" void sfb_debug_set_w8_trace_launch(int i) { g_w8_trace_launch = i; }
extern "C" void sfb_debug_set_w8_trace(void* p) { g_w8_trace = static_cast<unsigned long long*>(p); }
#endif

// Clusters of `size` CTAs of the GEMM kernel that can be resident at once
// (cached per device and size; 0 when the query fails).
static int w8_max_clusters(const DeviceInfo& dev, int size) {
    static std::atomic<int> cache[64][17];            // 0: not queried yet (idempotent query)
    std::atomic<int>& slot = cache[dev.ordinal & 63][size < 0 ? 0 : (size > 16 ? 16 : size)];
    if (const int n = slot.load(std::memory_order_relaxed); n != 0) return n;
    const w8::KernFn kern = w8::pick(0, true, 128);   // the variants share their resource use
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             w8::kSmemBytes) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed,
                             1) != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(size, 1, 1);
    cfg.blockDim = dim3(w8::kThreads, 1, 1);
    cfg.dynamicSmemBytes = w8::kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = size;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
#ifdef SFB_TRACE
    fprintf(stderr, "w8a16: cluster size %d -> %d resident clusters\n", size, n);
#endif
    slot.store(n, std::memory_order_relaxed);
    return n;
}

int w8a16_gemm_launch(const void* x, int64_t ldx, const int8_t* w, const float* w_scale,
                      const void* bias, const void* residual, int64_t ldr, void* y, int64_t ldy,
                      int32_t y_dtype, int32_t M, int32_t N, int32_t K, int32_t act,
                      int32_t num_splits, cudaStream_t stream, bool pdl) {
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
    p.y_f32 = y_dtype == SFB_F32 ? 1 : 0;
    p.kchunks = K / 64;
    // tokens per CTA: round up to 32, at most 256 (16-token rounding measured
    // slower in the denoise: 67 tokens as N = 80 against N = 96)
    p.bn = M >= 256 ? 256 : ((M + 31) / 32) * 32;
    if (M >= 256) {
        // When 256-token tiles leave SMs idle in their single wave, take the
        // narrowest token tile whose grid still fits one wave (less MMA work
        // per CTA, the same single wave): M = 1072 → 9 tiles of 128 tokens,
        // 144 CTAs, instead of 5 of 256 (80 CTAs). Grids of several waves keep
        // 256 (per-CTA fixed costs favour the widest tile).
        const int64_t nt = (N + 127) / 128;
        auto ctas = [&](int bn) { return nt * ((M + bn - 1) / bn); };
        if (ctas(256) < dev.num_sms)
            for (int bn = 224; bn >= 32 && ctas(bn) <= dev.num_sms; bn -= 32) p.bn = bn;
    }
    const int mtile = (M + p.bn - 1) / p.bn;
    // Split K across a cluster only when the tiles alone leave most SMs idle,
    // and only as far as every cluster still fits in one wave: at one CTA per
    // SM the GPCs hold fewer 8-CTA clusters than SMs / 8, and a cluster left
    // over for a second wave doubles the kernel's time.
    auto auto_splits = [&](int units) {
        int sp = 1;
        while (p.bn <= 128 && sp < 8 && units * sp * 2 <= dev.num_sms &&
               p.kchunks / (sp * 2) >= 2 && units <= w8_max_clusters(dev, sp * 2))
            sp *= 2;
        return sp;
    };
    int tm = 128, ntile = (N + 127) / 128;
    int splits = num_splits;
    if (splits <= 0) {
        splits = auto_splits(ntile * mtile);
        // 64-channel tiles when 128-channel tiles cannot fill the GPU and the
        // halved tile gives more CTAs (N = 2048 at 67 tokens: 32 tiles × 4
        // splits instead of 16 × 4, 8-CTA clusters not fitting one wave)
        const int ntile64 = (N + 63) / 64, s64 = auto_splits(ntile64 * mtile);
        if (ntile * mtile * splits < dev.num_sms && ntile64 * mtile * s64 > ntile * mtile * splits &&
            ntile64 * mtile * s64 <= dev.num_sms) {           // and still one wave
            tm = 64; ntile = ntile64; splits = s64;
        }
    }
    if (splits != 1 && splits != 2 && splits != 4 && splits != 8 && splits != 16) return SFB_ERR_INVALID;
    if (splits > 1 && p.bn > 128) return SFB_ERR_INVALID;
    if (splits > p.kchunks || splits > tm / 8) return SFB_ERR_INVALID;
    p.splits = splits;
    p.stages = w8::num_stages(p.bn, tm);
    if (splits > 1) {
        // split-K: the receive area of the merge, TM × bn fp32, lies past the
        // ring's stages (at most 64 KB: four stages of the widest tile remain)
        const int sb = w8::stage_bytes(p.bn, tm), rcv = tm * p.bn * 4;
        p.stages = std::min(w8::kMaxStages, (w8::kRingBytes - rcv) / sb);
        p.rcv_off = p.stages * sb;
    }

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
        cuuint32_t box[2] = {64, (cuuint32_t)tm};
        cuuint32_t es[2] = {1, 1};
        int rc = encode_tensor_map(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(w),
                                   dims, str, box, es, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc != SFB_OK) return rc;
    }
    const w8::KernFn kern = w8::pick(act, p.splits > 1, tm);
    {
        static std::mutex mu;
        static std::vector<std::pair<int, w8::KernFn>> done;
        std::lock_guard<std::mutex> lock(mu);
        bool have = false;
        for (const auto& d : done) have = have || (d.first == dev.ordinal && d.second == kern);
        if (!have) {
            cudaError_t e1 = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  w8::kSmemBytes);
            cudaError_t e2 = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
            if (e1 != cudaSuccess || e2 != cudaSuccess) {
                (void)cudaGetLastError();
                record_cuda_error(e1 != cudaSuccess ? e1 : e2, "w8a16 kernel attributes");
                return SFB_ERR_CUDA;
            }
            done.emplace_back(dev.ordinal, kern);
        }
    }
#ifdef SFB_TRACE
    p.tl = tl_buf();
    p.tl_launch = tl_next();
    p.trace = (g_w8_trace_launch < 0 || g_w8_trace_launch == p.tl_launch) ? g_w8_trace : nullptr;
#endif
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.splits, ntile, mtile);
    cfg.blockDim = dim3(w8::kThreads, 1, 1);
    cfg.dynamicSmemBytes = w8::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = p.splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1 + pdl_attr(&attr[1], pdl);
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mx, mw, p);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        record_cuda_error(e, "w8a16 gemm launch");
        return SFB_ERR_LAUNCH;
    }
    return SFB_OK;
}

}  // namespace sfb
