// rdt_dense.cu — persistent multi-stage projection kernel for one RDT-1B
// session (M <= 80 tokens; sm_100a, tcgen05 + TMA + clusters).
//
// At one session the projections of a DiT block are a chain of small
// dependent GEMMs (M = 67 tokens × N = 2048 or 6144 × K = 2048), each far
// below the time its launch, its dependency release and its prologue take.
// This kernel runs a whole run of consecutive projections between two
// attention kernels as "stages" of one launch:
//
//   Y_s[m, n] = act( r_s[m] · w_scale[n] · Σ_k X_s[m, k] · Wq[n, k] + bias[n] ) + R[m, n]
//
// with the stages ordered by device-side completion counters instead of
// kernel boundaries. Each stage is the work of dequant + gemm_bias_act in the
// reference (src/backend/cuda/ops/quantization.cu:18-95 followed by
// src/backend/cuda/cuda_backend.cu:337-467) for one projection of
// RDTBlock::forward (src/models/rdt1b/dit_block.cu:349-387), with the block's
// pre-norm RMSNorm (norm.cuh:89-127; test_rdt1b_alignment.py:73-80) folded in:
//
//   * a stage that writes the residual stream x also writes, per token row,
//     partial sums of x² over its channels (ss_out) and xg = bf16(x · g) for
//     the next norm's weight g;
//   * the next stage multiplies X = xg by W and scales row m of the product
//     by r[m] = 1 / sqrt(Σ ss / K + eps) in its epilogue. Up to the rounding
//     point of the normalised activations (bf16(x·g) instead of
//     bf16(x·r·g), one bf16 rounding either way) this is RMSNorm → linear.
//
// Work of a stage: output tiles of TM = 64 or 128 weight rows; a 4-CTA
// thread-block cluster takes a tile and splits K four ways; clusters walk the
// tiles round-robin. Per CTA (11 warps):
//   warp 0      streams its int8 weight tiles [TM × 64] through a 6-slot ring,
//               running ahead across stages (weights depend on nothing);
//   warps 2..9  convert int8 → bf16 (two groups of four warps, alternating
//               chunks, exact), then run the epilogue;
//   warp 1      issues tcgen05.mma (M = TM weight rows, N = 80 tokens, K = 16)
//               into one of two TMEM accumulators;
//   warp 10     waits for the previous stage's counter (acquire, bounded),
//               then loads the CTA's activation slice [80 × K/4] by TMA.
// Split-K partials go from TMEM straight into the owning CTA's shared memory
// (the owner of a channel row is the cluster rank that equals its TMEM lane
// window), announced by remote mbarrier arrivals; owners sum the four
// partials, apply the epilogue and store coalesced 16-byte rows. Every
// CTA then bumps the stage's completion counter (release). No global scratch
// beyond the counters and the stage table.
//
// Every wait is bounded (1 s) and records SFB_ERR_DEVICE_TIMEOUT; after a
// failure a CTA stops issuing copies and MMAs, waits (bounded) for those in
// flight, still signals its counters so that no other CTA waits on it, and
// leaves through the final cluster barrier.
#include "common.cuh"
#include "sm100_ptx.cuh"

namespace sfb {

// One projection of a dense launch. Tensor maps first (64-byte aligned).
struct alignas(64) DenseStage {
    CUtensorMap tmW;                 // int8 [N, K], box {64, TM}, no swizzle
    CUtensorMap tmX;                 // bf16 [M, K] (row stride ldx), box {64, 80}, SWIZZLE_128B
    const float* w_scale;            // [N]
    const __nv_bfloat16* bias;       // [N] or null
    const void* residual;            // [M, N] (ldr) in y's dtype, or null; may alias y
    void* y;                         // [M, N] (ldy), bf16 or fp32
    const __nv_bfloat16* g_next;     // [N] or null: also write xg = bf16(y · g_next) (y as stored)
    __nv_bfloat16* xg;               // [M, N] (ldg)
    float* ss_out;                   // or null: [tiles · 4][80] partial Σ y² per token row (y as stored)
    const float* ss_in;              // or null: [n_ss_in][80] partials of X's rows; scales rows by r[m]
    const uint8_t* l2_prefetch;      // or null: a region the next kernel reads (a cross-attention
    uint64_t l2_bytes;               // K/V cache), pulled into L2 while this stage runs
    int64_t ldr, ldy, ldg;
    int32_t n_ss_in;
    int32_t N, K, TM, tiles, act, y_f32;
    float eps;
};

namespace dense {

constexpr int kThreads = 11 * 32;
// warp roles
constexpr int kWarpW = 0;                     // int8 weight stream (TMA)
constexpr int kWarpMma = 1;                   // tcgen05.mma issue
constexpr int kWarpX = 2;                     // stage dependency + activation loads (TMA)
constexpr int kWarpConv0 = 3;                 // warps 3..6: int8 → bf16 conversion
constexpr int kWarpEpi0 = 7;                  // warps 7..10: epilogue (TMEM quadrant = warp % 4)
constexpr int kEpiThreads = 128;
constexpr int kBN = 80;                       // tokens per tile (MMA N): M <= 80
constexpr int kSplit = 4;                     // cluster size = split-K ways
constexpr int kNW = 4;                        // int8 weight ring slots (TM × 64 B, TM <= 128)
constexpr int kNB = 4;                        // converted bf16 weight slots (SW128, TM × 128 B)
constexpr int kNX = 8;                        // activation chunks per CTA (K / 4 / 64 <= 8)
constexpr int kXBytes = kBN * 128;            // one activation chunk [80 × 64] bf16, SW128
constexpr int kWBytes = 128 * 64;             // int8 slot
constexpr int kWBBytes = 128 * 128;           // bf16 slot
constexpr int kOffX = 0;
constexpr int kOffWB = kOffX + kNX * kXBytes;                 // 81920
constexpr int kOffW = kOffWB + kNB * kWBBytes;                // 147456
constexpr int kOffRcv = kOffW + kNW * kWBytes;                // 180224
constexpr int kRcvBytes = kSplit * 32 * kBN * 4;              // [4 sources][R <= 32][80] fp32
constexpr int kOffRinv = kOffRcv + kRcvBytes;
constexpr int kOffRed = kOffRinv + kBN * 4;                   // [4 warps][80] partial row sums
constexpr int kOffBar = kOffRed + 4 * kBN * 4;
// barriers
constexpr int kBarWFull = 0;                                  // [kNW]
constexpr int kBarWFree = kBarWFull + kNW;                    // [kNW]
constexpr int kBarBFull = kBarWFree + kNW;                    // [kNB]
constexpr int kBarBFree = kBarBFull + kNB;                    // [kNB]
constexpr int kBarXFull = kBarBFree + kNB;                    // [kNX]
constexpr int kBarDep = kBarXFull + kNX;                      // stage dependency passed
constexpr int kBarAccFull = kBarDep + 1;                      // [2]
constexpr int kBarAccFree = kBarAccFull + 2;                  // [2]
constexpr int kBarRcv = kBarAccFree + 2;                      // partials of the four sources landed
constexpr int kBarRcvFree = kBarRcv + 1;                      // [4]: owner o has read the previous unit
constexpr int kBarDrain = kBarRcvFree + kSplit;
constexpr int kNumBars = kBarDrain + 1;
constexpr int kOffTmem = kOffBar + 8 * kNumBars;
constexpr int kOffGen = kOffTmem + 8;
constexpr int kSmemUsed = kOffGen + 8;
constexpr int kSmemBytes = kSmemUsed + 1024;                  // + alignment slack
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
static_assert(kOffWB % 1024 == 0 && kOffW % 1024 == 0 && kXBytes % 1024 == 0, "SW128 tile alignment");
static_assert(kOffBar % 8 == 0, "barrier alignment");
static_assert(kWarpEpi0 + 4 == kThreads / 32, "four epilogue warps last");
constexpr uint64_t kWaitNs = 1000000000ull;
constexpr uint64_t kDrainNs = 100000000ull;

__device__ __forceinline__ float gelu_tanh(float x) {
    const float k0 = 0.7978845608028654f, k1 = 0.044715f;
    return 0.5f * x * (1.f + tanhf(k0 * fmaf(k1 * x * x, x, x)));
}

__device__ __forceinline__ uint64_t ld_acquire_gpu(const unsigned long long* p) {
    uint64_t v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_gpu_add(unsigned long long* p, uint64_t v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void fence_acq_rel_cluster() {
    asm volatile("fence.acq_rel.cluster;" ::: "memory");
}
// Arrive (release at cluster scope) on the mbarrier at the same offset in the
// shared memory of cluster CTA `rank`.
__device__ __forceinline__ void mbar_arrive_remote(uint64_t* local_bar, uint32_t rank) {
    const uint32_t a = ptx::dsmem_map(ptx::smem_u32(local_bar), rank);
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(a) : "memory");
}
// Bounded wait with acquire at cluster scope (for arrivals made by peers).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, uint64_t timeout_ns) {
    const uint32_t a = ptx::smem_u32(bar);
    auto probe = [&]() {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred P;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 P, [%1], %2;\n\t"
            "selp.b32 %0, 1, 0, P;\n\t}"
            : "=r"(ok) : "r"(a), "r"(parity) : "memory");
        return ok != 0;
    };
    if (probe()) return true;
    const uint64_t t0 = ptx::global_timer_ns();
    for (uint32_t it = 0;; ++it) {
        if (probe()) return true;
        if ((it & 63u) == 63u && ptx::global_timer_ns() - t0 > timeout_ns) return false;
    }
}
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(p)), "r"(bytes)
                 : "memory");
}
// Asynchronous store into a peer's shared memory that completes `16` bytes
// of the transaction count of the peer's mbarrier at remote_bar.
__device__ __forceinline__ void st_async_v4(uint32_t addr, float4 v, uint32_t remote_bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];"
                 ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(remote_bar) : "memory");
}
__device__ __forceinline__ void dsmem_st_v4(uint32_t addr, float4 v) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};"
                 ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w) : "memory");
}

// The CTA's share of a stage: tiles t = cluster, cluster + nclusters, ...
__device__ __forceinline__ int units_of(const DenseStage& S, int cl, int ncl) {
    return cl < S.tiles ? (S.tiles - cl + ncl - 1) / ncl : 0;
}

// The kernel body: `stages` in global memory (a model's stage table) or in
// the parameter space of a launch (dense_pair_kernel).
#ifdef SFB_TRACE
// per launch slot: [CTA < 160][stage < 16, then 16 = setup][8] global-timer stamps
constexpr int kTrStages = 17;
#define DN_T(st, k) do { if (trace != nullptr && blockIdx.x < 160 && (st) < kTrStages) \
        trace[(blockIdx.x * kTrStages + (st)) * 8 + (k)] = ptx::global_timer_ns(); } while (0)
#else
#define DN_T(st, k) do { } while (0)
#endif

__device__ __forceinline__ void dense_run(const DenseStage* __restrict__ stages, int nst,
                                          unsigned long long* __restrict__ ctr, int M
#ifdef SFB_TRACE
                                          , unsigned long long* trace
#endif
                                          ) {
    using namespace ptx;
    if (threadIdx.x == 0) DN_T(16, 0);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kOffTmem);
    uint64_t* gen_slot = reinterpret_cast<uint64_t*>(smem + kOffGen);
    float* rcv = reinterpret_cast<float*>(smem + kOffRcv);
    float* rinv = reinterpret_cast<float*>(smem + kOffRinv);
    float* red = reinterpret_cast<float*>(smem + kOffRed);
    auto sX = [&](int c) { return smem + kOffX + c * kXBytes; };
    auto sWB = [&](int s) { return smem + kOffWB + s * kWBBytes; };
    auto sW = [&](int s) { return smem + kOffW + s * kWBytes; };

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rank = static_cast<int>(cluster_ctarank());
    const int ncl = gridDim.x / kSplit, cl = blockIdx.x / kSplit;
    const uint64_t ncta = gridDim.x;

    if (tid == 32) {
        for (int i = 0; i < kNW; ++i) { mbar_init(&bars[kBarWFull + i], 1); mbar_init(&bars[kBarWFree + i], 4); }
        for (int i = 0; i < kNB; ++i) { mbar_init(&bars[kBarBFull + i], 4); mbar_init(&bars[kBarBFree + i], 1); }
        for (int i = 0; i < kNX; ++i) mbar_init(&bars[kBarXFull + i], 1);
        mbar_init(&bars[kBarDep], 1);
        for (int i = 0; i < 2; ++i) { mbar_init(&bars[kBarAccFull + i], 1); mbar_init(&bars[kBarAccFree + i], 4); }
        mbar_init(&bars[kBarRcv], 1);                       // armed by the owner (expect_tx), filled by st.async
        for (int i = 0; i < kSplit; ++i) mbar_init(&bars[kBarRcvFree + i], 4);   // the owner's 4 warps
        mbar_init(&bars[kBarDrain], 1);
        fence_mbarrier_init();
    }
    if (tid == 0) {
        // this launch's generation: every CTA adds 1 to the start counter; a
        // launch adds exactly gridDim.x, so old / gridDim.x names the launch
        const unsigned long long old = atomicAdd(&ctr[0], 1ull);
        *gen_slot = old / ncta;
    }
    if (warp == 0) {
        tmem_alloc(tmem_holder, 256);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    // every peer of the cluster has initialised its barriers and runs
    cluster_arrive_relaxed();
    cluster_wait();
    const uint32_t tmem = *tmem_holder;
    const uint64_t target = (*gen_slot + 1) * ncta;     // a stage is done when every CTA added 1
    if (tid == 0) DN_T(16, 1);

    bool ok = true;
    auto wait = [&](int b, uint32_t parity) {
        if (!mbar_wait(&bars[b], parity, ok ? kWaitNs : 0ull)) ok = false;
    };

    if (warp == kWarpW) {
        // ── int8 weight stream, running ahead across stages ────────────────
        uint32_t gw = 0;
        const uint64_t pol = l2_evict_first_policy();
        for (int s = 0; s < nst && ok; ++s) {
            const DenseStage& S = stages[s];
            const int nu = units_of(S, cl, ncl), nk = S.K / 64 / kSplit;
            const uint32_t bytes = static_cast<uint32_t>(S.TM) * 64u;
            if (S.l2_prefetch != nullptr && lane == 0) {
                // this CTA's slice of the region, in 64 KB bulk prefetches (16-byte granules)
                const uint64_t total = S.l2_bytes & ~15ull;
                const uint64_t per = ((total + gridDim.x - 1) / gridDim.x + 15) & ~15ull;
                const uint64_t b0 = per * blockIdx.x;
                const uint64_t b1 = b0 + per < total ? b0 + per : total;
                for (uint64_t o = b0; o < b1; o += 65536) {
                    const uint64_t n = b1 - o < 65536 ? b1 - o : 65536;
                    prefetch_l2_bulk(S.l2_prefetch + o, static_cast<uint32_t>(n));
                }
            }
            __syncwarp();
            for (int j = 0; j < nu && ok; ++j) {
                const int n0 = (cl + j * ncl) * S.TM;
                for (int c = 0; c < nk; ++c, ++gw) {
                    const int slot = gw % kNW;
                    if (gw >= kNW) wait(kBarWFree + slot, ((gw / kNW) - 1) & 1);
                    if (!ok) break;
                    if (elect_one()) {
                        mbar_arrive_expect_tx(&bars[kBarWFull + slot], bytes);
                        tma_load_2d_hint(sW(slot), &S.tmW, &bars[kBarWFull + slot], (rank * nk + c) * 64, n0, pol);
                    }
                    __syncwarp();
                }
            }
        }
        // copies in flight land before the CTA leaves (bounded)
        for (uint32_t g = gw > kNW ? gw - kNW : 0; g < gw; ++g)
            if (!mbar_wait(&bars[kBarWFull + g % kNW], (g / kNW) & 1, kDrainNs)) ok = false;
    } else if (warp == kWarpX) {
        // ── dependency + activation loads ──────────────────────────────────
        // xmask bit c: parity of the next completion of activation slot c
        // (stages may load different numbers of chunks)
        uint32_t xmask = 0, last_mask = 0;
        int loaded = 0;                                    // chunks of the last load issued
        pdl_wait();                                        // everything earlier kernels wrote
        for (int s = 0; s < nst; ++s) {
            const DenseStage& S = stages[s];
            if (units_of(S, cl, ncl) == 0) continue;
            if (s > 0 && lane == 0) {
                const unsigned long long* c = &ctr[s];     // stage s-1's counter
                if (ld_acquire_gpu(c) < target) {
                    const uint64_t t0 = global_timer_ns();
                    for (uint32_t it = 0;; ++it) {
                        if (ld_acquire_gpu(c) >= target) break;
                        if ((it & 63u) == 63u && global_timer_ns() - t0 > (ok ? kWaitNs : 0ull)) { ok = false; break; }
                    }
                }
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0 && ok;
            if (lane == 0) DN_T(s, 0);
            fence_proxy_async_global();                    // generic writes of other CTAs → this TMA
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[kBarDep]);    // also after a failure: nobody waits in vain
            const int nk = S.K / 64 / kSplit;
            if (ok) {
                if (elect_one()) {
                    for (int c = 0; c < nk; ++c) {
                        mbar_arrive_expect_tx(&bars[kBarXFull + c], kXBytes);
                        tma_load_2d(sX(c), &S.tmX, &bars[kBarXFull + c], (rank * nk + c) * 64, 0);
                    }
                }
                __syncwarp();
                last_mask = xmask;
                loaded = nk;
                xmask ^= (nk >= 32 ? 0xffffffffu : ((1u << nk) - 1u));
            }
        }
        // the last loads land before the CTA leaves (bounded; immediate on the normal path)
        for (int c = 0; c < loaded; ++c)
            if (!mbar_wait(&bars[kBarXFull + c], (last_mask >> c) & 1u, kDrainNs)) ok = false;
    } else if (warp == kWarpMma) {
        // ── MMA issuer ──────────────────────────────────────────────────────
        uint32_t gm = 0, um = 0, xmask = 0;                // xmask as the activation loader's
        for (int s = 0; s < nst && ok; ++s) {
            const DenseStage& S = stages[s];
            const int nu = units_of(S, cl, ncl);
            if (nu == 0) continue;
            const int nk = S.K / 64 / kSplit;
            const uint32_t idesc = idesc_f16(static_cast<uint32_t>(S.TM), kBN, 1, 0, 0);
            for (int j = 0; j < nu && ok; ++j, ++um) {
                const int buf = um & 1;
                if (um >= 2) wait(kBarAccFree + buf, ((um >> 1) - 1) & 1);
                const uint32_t tacc = tmem + buf * 128;
                for (int c = 0; c < nk && ok; ++c, ++gm) {
                    const int bs = gm % kNB;
                    wait(kBarBFull + bs, (gm / kNB) & 1);
                    wait(kBarXFull + c, (xmask >> c) & 1u);
                    if (!ok) break;
                    tc_fence_after_sync();
                    const uint32_t aw = smem_u32(sWB(bs)), ax = smem_u32(sX(c));
                    if (elect_one()) {
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            mma_f16_ss(tacc, smem_desc_sw128(aw + kk * 32, 16, 1024),
                                       smem_desc_sw128(ax + kk * 32, 16, 1024), idesc,
                                       (c > 0 || kk > 0) ? 1u : 0u);
                        mma_commit(&bars[kBarBFree + bs]);
                        if (c == nk - 1) mma_commit(&bars[kBarAccFull + buf]);
                    }
                    __syncwarp();
                }
            }
            xmask ^= (nk >= 32 ? 0xffffffffu : ((1u << nk) - 1u));
        }
        if (!ok) {
            if (elect_one()) mma_commit(&bars[kBarDrain]);
            __syncwarp();
            mbar_wait(&bars[kBarDrain], 0, kDrainNs);
        }
    } else if (warp < kWarpEpi0) {
        // ── converters (warps 3..6): int8 [TM × 64] → bf16 SW128, running ahead
        //    of the MMAs by up to kNB chunks, across units and stages ─────────
        const int ct = tid - kWarpConv0 * 32;              // 0..127
        uint32_t gc = 0;
        for (int s = 0; s < nst; ++s) {
            const DenseStage& S = stages[s];
            const int nu = units_of(S, cl, ncl), nk = S.K / 64 / kSplit, TM = S.TM;
            for (int j = 0; j < nu; ++j) {
                for (int c = 0; c < nk; ++c, ++gc) {
                    const int ws = gc % kNW, bs = gc % kNB;
                    wait(kBarWFull + ws, (gc / kNW) & 1);
                    if (gc >= kNB) wait(kBarBFree + bs, ((gc / kNB) - 1) & 1);
                    const uint8_t* src = sW(ws);
                    uint8_t* dst = sWB(bs);
                    const int its = TM / 16;               // 8-byte units per thread
                    for (int it = 0; it < its; ++it) {
                        const int unit = it * 128 + ct;
                        const int r = unit >> 3, ch = unit & 7;
                        const uint2 raw = *reinterpret_cast<const uint2*>(src + r * 64 + ch * 8);
                        uint32_t o[4];
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const uint32_t x = (h ? raw.y : raw.x) ^ 0x80808080u;
                            // 0x4B0000bb = 2^23 + bb as fp32; minus (2^23 + 128) gives q exactly
                            const float f0 = __uint_as_float(prmt(x, 0x4B000000u, 0x7440u)) - 8388736.f;
                            const float f1 = __uint_as_float(prmt(x, 0x4B000000u, 0x7441u)) - 8388736.f;
                            const float f2 = __uint_as_float(prmt(x, 0x4B000000u, 0x7442u)) - 8388736.f;
                            const float f3 = __uint_as_float(prmt(x, 0x4B000000u, 0x7443u)) - 8388736.f;
                            o[2 * h]     = prmt(__float_as_uint(f0), __float_as_uint(f1), 0x7632u);
                            o[2 * h + 1] = prmt(__float_as_uint(f2), __float_as_uint(f3), 0x7632u);
                        }
                        *reinterpret_cast<uint4*>(dst + r * 128 + ((ch ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) { mbar_arrive(&bars[kBarWFree + ws]); mbar_arrive(&bars[kBarBFull + bs]); }
                }
            }
        }
    } else {
        // ── epilogue (warps 7..10; TMEM quadrant q = warp % 4 = owner rank) ──
        const int et = tid - kWarpEpi0 * 32;               // 0..127
        const int q = warp & 3;
        constexpr int kMaxIt = 3;                          // owner units (<= 80 · 32 / 8) / 128 threads
        uint32_t ue = 0, xs = 0;
        const int mvalid = min(M, kBN);
        for (int s = 0; s < nst; ++s) {
            const DenseStage& S = stages[s];
            const int nu = units_of(S, cl, ncl);
            const int TM = S.TM, RPW = TM / 4;             // rows per TMEM quadrant = rows per owner
            const int segs = RPW / 8;                      // 8-channel segments per owned row
            const int units = mvalid * segs;
            for (int j = 0; j < nu; ++j, ++ue) {
                const int n0 = (cl + j * ncl) * TM;
                const int nb = n0 + rank * RPW;            // first channel this CTA owns
                // (1) the stage's dependency (once per stage); rows' RMS factors
                if (j == 0) {
                    wait(kBarDep, xs & 1);
                    if (S.ss_in != nullptr) {
                        // warp w sums partials [w·np/4, (w+1)·np/4); lane l the rows l, l+32,
                        // l+64 (consecutive floats: one 128-byte line per warp load); the
                        // four warps' sums are then added in warp order
                        const int np = S.n_ss_in;
                        const int p0 = (q * np) / 4, p1 = ((q + 1) * np) / 4;
                        float a0 = 0.f, a1 = 0.f, a2 = 0.f;
#pragma unroll 4
                        for (int p = p0; p < p1; ++p) {
                            const float* row = S.ss_in + p * kBN;
                            a0 += row[lane];
                            a1 += row[lane + 32];
                            if (lane + 64 < kBN) a2 += row[lane + 64];
                        }
                        red[q * kBN + lane] = a0;
                        red[q * kBN + lane + 32] = a1;
                        if (lane + 64 < kBN) red[q * kBN + lane + 64] = a2;
                        named_bar_sync(1, kEpiThreads);
                        if (et < mvalid) {
                            const float tot = ((red[et] + red[kBN + et]) + red[2 * kBN + et]) + red[3 * kBN + et];
                            rinv[et] = 1.f / sqrtf(tot / static_cast<float>(S.K) + S.eps);
                        }
                    }
                    named_bar_sync(1, kEpiThreads);
                }
                // (2) this thread's owner-pass operands, loaded while the MMAs run
                float rres[kMaxIt][8];
                uint4 rbias[kMaxIt], rg[kMaxIt];
#pragma unroll
                for (int it = 0; it < kMaxIt; ++it) {
                    const int u = et + it * kEpiThreads;
                    const int m = u < units ? u / segs : 0, n = nb + (u < units ? (u - m * segs) * 8 : 0);
                    const bool use = u < units && n < S.N;
#pragma unroll
                    for (int k = 0; k < 8; ++k) rres[it][k] = 0.f;
                    rbias[it] = make_uint4(0u, 0u, 0u, 0u);
                    rg[it] = make_uint4(0u, 0u, 0u, 0u);
                    if (use && S.residual != nullptr) {
                        if (S.y_f32) {
                            const float* rp = static_cast<const float*>(S.residual) + m * S.ldr + n;
                            const float4 a = *reinterpret_cast<const float4*>(rp), b = *reinterpret_cast<const float4*>(rp + 4);
                            rres[it][0] = a.x; rres[it][1] = a.y; rres[it][2] = a.z; rres[it][3] = a.w;
                            rres[it][4] = b.x; rres[it][5] = b.y; rres[it][6] = b.z; rres[it][7] = b.w;
                        } else {
                            const uint4 ru = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(S.residual) + m * S.ldr + n);
                            const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&ru);
#pragma unroll
                            for (int k = 0; k < 4; ++k) { const float2 f = __bfloat1622float2(r2[k]); rres[it][2 * k] = f.x; rres[it][2 * k + 1] = f.y; }
                        }
                    }
                    if (use && S.bias != nullptr) rbias[it] = *reinterpret_cast<const uint4*>(S.bias + n);
                    if (use && S.g_next != nullptr) rg[it] = *reinterpret_cast<const uint4*>(S.g_next + n);
                }
                // (3) accumulator → scaled partials into the owner's receive area
                const int buf = ue & 1;
                const bool lane_ok = lane < RPW;
                const int trow = q * RPW + lane;               // tile row (owner q, slot lane)
                const float sc = (lane_ok && n0 + trow < S.N) ? S.w_scale[n0 + trow] : 0.f;
                // arm this CTA's receive barrier for the unit: the four sources' partials
                // of its RPW rows (this thread has passed the previous unit's phase)
                if (et == 0)
                    mbar_arrive_expect_tx(&bars[kBarRcv], static_cast<uint32_t>(kSplit * RPW * kBN * 4));
                if (ue >= 1) {
                    // the owner has read this area's previous contents
                    if (!mbar_wait_cluster(&bars[kBarRcvFree + q], (ue - 1) & 1, ok ? kWaitNs : 0ull)) ok = false;
                }
                wait(kBarAccFull + buf, (ue >> 1) & 1);
                if (et == 0 && j == 0) DN_T(s, 1);
                tc_fence_after_sync();
                const uint32_t tq = tmem + buf * 128 + (static_cast<uint32_t>(q * 32) << 16);
                const uint32_t base = dsmem_map(smem_u32(rcv + (rank * RPW + (lane_ok ? lane : 0)) * kBN),
                                                static_cast<uint32_t>(q));
                const uint32_t rbar = dsmem_map(smem_u32(&bars[kBarRcv]), static_cast<uint32_t>(q));
#pragma unroll 1
                for (int blk = 0; blk < 3; ++blk) {                 // 32 token columns at a time
                    float v[32];
                    tmem_ld32(tq + 32 * blk, v);
                    tmem_ld_wait();
                    if (lane_ok) {
#pragma unroll
                        for (int i = 0; i < 32; i += 4) {
                            if (blk * 32 + i < kBN)
                                st_async_v4(base + (blk * 32 + i) * 4,
                                            make_float4(v[i] * sc, v[i + 1] * sc, v[i + 2] * sc, v[i + 3] * sc), rbar);
                        }
                    }
                }
                tc_fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars[kBarAccFree + buf]);
                if (et == 0 && j == nu - 1) DN_T(s, 4);
                // (4) owner pass: rows [nb, nb + RPW) of the tile, every token
                if (!mbar_wait_cluster(&bars[kBarRcv], ue & 1, ok ? kWaitNs : 0ull)) ok = false;
                if (et == 0 && j == nu - 1) DN_T(s, 5);
                // sums of the four sources first, so the area is released before any
                // global store of this pass
                float ysum[kMaxIt][8];
#pragma unroll
                for (int it = 0; it < kMaxIt; ++it) {
                    const int u = et + it * kEpiThreads;
                    const int m = u < units ? u / segs : 0, seg = u < units ? u - (u / segs) * segs : 0;
#pragma unroll
                    for (int k = 0; k < 8; ++k) ysum[it][k] = 0.f;
                    if (u < units) {
#pragma unroll
                        for (int src = 0; src < kSplit; ++src) {
#pragma unroll
                            for (int k = 0; k < 8; ++k) ysum[it][k] += rcv[(src * RPW + seg * 8 + k) * kBN + m];
                        }
                    }
                }
                __syncwarp();
                if (lane < kSplit) mbar_arrive_remote(&bars[kBarRcvFree + rank], static_cast<uint32_t>(lane));
#pragma unroll
                for (int it = 0; it < kMaxIt; ++it) {
                    const int u = et + it * kEpiThreads;
                    if (it * kEpiThreads >= units) break;          // uniform over the CTA
                    const bool valid = u < units && ok;
                    const int m = valid ? u / segs : 0, seg = valid ? u - (u / segs) * segs : 0;
                    const int n = nb + seg * 8;
                    float outv[8];
                    float sq = 0.f;
                    if (valid && n < S.N) {
                        const float* yv = ysum[it];
                        const float r = S.ss_in != nullptr ? rinv[m] : 1.f;
                        const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&rbias[it]);
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const float2 bb = __bfloat1622float2(b2[k]);
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                float t = fmaf(yv[2 * k + h], r, h ? bb.y : bb.x);
                                if (S.act == 1) t = gelu_tanh(t);
                                else if (S.act == 2) t = t / (1.f + expf(-t));
                                outv[2 * k + h] = t + rres[it][2 * k + h];
                            }
                        }
                        if (S.y_f32) {
                            float* dst = static_cast<float*>(S.y) + m * S.ldy + n;
                            *reinterpret_cast<float4*>(dst) = make_float4(outv[0], outv[1], outv[2], outv[3]);
                            *reinterpret_cast<float4*>(dst + 4) = make_float4(outv[4], outv[5], outv[6], outv[7]);
                        } else {
                            uint4 o;
                            __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                o2[k] = __floats2bfloat162_rn(outv[2 * k], outv[2 * k + 1]);
                                const float2 f = __bfloat1622float2(o2[k]);      // the stored values
                                outv[2 * k] = f.x; outv[2 * k + 1] = f.y;
                            }
                            *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(S.y) + m * S.ldy + n) = o;
                        }
                        if (S.g_next != nullptr) {
                            const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&rg[it]);
                            uint4 qv;
                            __nv_bfloat162* q2 = reinterpret_cast<__nv_bfloat162*>(&qv);
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                const float2 g = __bfloat1622float2(g2[k]);
                                q2[k] = __floats2bfloat162_rn(outv[2 * k] * g.x, outv[2 * k + 1] * g.y);
                            }
                            *reinterpret_cast<uint4*>(S.xg + m * S.ldg + n) = qv;
                        }
#pragma unroll
                        for (int k = 0; k < 8; ++k) sq = fmaf(outv[k], outv[k], sq);
                    }
                    if (S.ss_out != nullptr) {
                        // the row's segments sit in adjacent lanes (segs divides 32)
                        for (int o = 1; o < segs; o <<= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
                        if (valid && seg == 0) S.ss_out[((n0 / TM) * kSplit + rank) * kBN + m] = sq;
                    }
                }
            }
            if (nu > 0) ++xs;
            // (5) this CTA is done with stage s: publish its writes, bump the counter
            named_bar_sync(1, kEpiThreads);
            if (et == 0) {
                // release at GPU scope: covers every epilogue thread's stores, which the
                // named barrier ordered before it; readers acquire and fence the
                // async proxy before their TMA loads
                DN_T(s, 2);
                red_release_gpu_add(&ctr[1 + s], 1ull);
                DN_T(s, 3);
            }
        }
    }

    if (!ok) atomicExch(&g_sfb_device_error, SFB_ERR_DEVICE_TIMEOUT);
    tc_fence_before_sync();
    __syncthreads();
    // no CTA leaves while a peer may still write its shared memory or arrive on its barriers
    cluster_arrive();
    cluster_wait();
    if (warp == 0) {
        tc_fence_after_sync();
        tmem_dealloc(tmem, 256);
    }
}

__global__ void __launch_bounds__(kThreads, 1)
rdt_dense_kernel(const DenseStage* __restrict__ stages, int nst, unsigned long long* __restrict__ ctr, int M
#ifdef SFB_TRACE
                 , unsigned long long* trace
#endif
                 ) {
    dense_run(stages, nst, ctr, M
#ifdef SFB_TRACE
              , trace
#endif
              );
}

// Two stages passed by value (tensor maps in the parameter space): a launch
// that needs no stage table in device memory.
struct DenseStagePair { DenseStage s[2]; };
__global__ void __launch_bounds__(kThreads, 1)
dense_pair_kernel(const __grid_constant__ DenseStagePair p, unsigned long long* __restrict__ ctr, int M) {
    dense_run(p.s, 2, ctr, M
#ifdef SFB_TRACE
              , nullptr
#endif
              );
}

}  // namespace dense

// Clusters of the dense kernel resident at once (one CTA per SM), cached.
int dense_clusters(const DeviceInfo& dev) {
    static std::atomic<int> cache[64];
    std::atomic<int>& slot = cache[dev.ordinal & 63];
    if (const int n = slot.load(std::memory_order_relaxed); n != 0) return n;
    auto kern = dense::rdt_dense_kernel;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, dense::kSmemBytes) != cudaSuccess ||
        cudaFuncSetAttribute(dense::dense_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             dense::kSmemBytes) != cudaSuccess) {
        (void)cudaGetLastError();
        return -1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(dense::kSplit, 1, 1);
    cfg.blockDim = dim3(dense::kThreads, 1, 1);
    cfg.dynamicSmemBytes = dense::kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = dense::kSplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        (void)cudaGetLastError();
        return -1;
    }
    slot.store(n, std::memory_order_relaxed);
    return n;
}

// Fills a stage's tensor maps and checks its shape. x: bf16 [M, K] (ldx);
// w: int8 [N, K].
int dense_stage_init(DenseStage& S, const void* x, int64_t ldx, int M, const int8_t* w, int N, int K, int TM) {
    if (M < 1 || M > dense::kBN) return SFB_ERR_SHAPE;
    if ((TM != 64 && TM != 128) || N % TM != 0 || K % (64 * dense::kSplit) != 0 ||
        K / 64 / dense::kSplit > dense::kNX)
        return SFB_ERR_SHAPE;
    S.N = N; S.K = K; S.TM = TM; S.tiles = N / TM;
    {
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
        cuuint64_t str[1] = {(cuuint64_t)(ldx * 2)};
        cuuint32_t box[2] = {64, (cuuint32_t)dense::kBN};
        cuuint32_t es[2] = {1, 1};
        SFB_TRY(encode_tensor_map(&S.tmX, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, str,
                                  box, es, CU_TENSOR_MAP_SWIZZLE_128B));
    }
    {
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
        cuuint64_t str[1] = {(cuuint64_t)K};
        cuuint32_t box[2] = {64, (cuuint32_t)TM};
        cuuint32_t es[2] = {1, 1};
        SFB_TRY(encode_tensor_map(&S.tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(w), dims, str,
                                  box, es, CU_TENSOR_MAP_SWIZZLE_NONE));
    }
    return SFB_OK;
}

// Launch configuration shared by both kernels (cluster of kSplit CTAs, one
// CTA per SM, as many clusters as are resident at once).
static cudaLaunchConfig_t dense_config(int ncl, cudaStream_t stream, cudaLaunchAttribute* attr, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ncl * dense::kSplit, 1, 1);
    cfg.blockDim = dim3(dense::kThreads, 1, 1);
    cfg.dynamicSmemBytes = dense::kSmemBytes;
    cfg.stream = stream;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = dense::kSplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1 + pdl_attr(&attr[1], pdl);
    return cfg;
}

// One launch over stages[0, nst) (device memory); ctr: nst + 1 counters of
// this launch slot (zero at allocation, never reset).
#ifdef SFB_TRACE
static unsigned long long* g_dense_trace = nullptr;
extern "C" void sfb_debug_set_dense_trace(void* p) { g_dense_trace = static_cast<unsigned long long*>(p); }
#endif

int dense_launch(const DenseStage* stages, int nst, unsigned long long* ctr, int M, cudaStream_t stream, bool pdl,
                 int trace_slot) {
    const DeviceInfo& dev = device_info();
    const int ncl = dense_clusters(dev);
    if (ncl <= 0) { record_cuda_error(cudaErrorInvalidConfiguration, "dense kernel clusters"); return SFB_ERR_LAUNCH; }
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = dense_config(ncl, stream, attr, pdl);
#ifdef SFB_TRACE
    unsigned long long* tr = (g_dense_trace != nullptr && trace_slot >= 0)
                                 ? g_dense_trace + static_cast<size_t>(trace_slot) * 160 * dense::kTrStages * 8 : nullptr;
    cudaError_t e = cudaLaunchKernelEx(&cfg, dense::rdt_dense_kernel, stages, nst, ctr, M, tr);
#else
    (void)trace_slot;
    cudaError_t e = cudaLaunchKernelEx(&cfg, dense::rdt_dense_kernel, stages, nst, ctr, M);
#endif
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        record_cuda_error(e, "dense kernel launch");
        return SFB_ERR_LAUNCH;
    }
    return SFB_OK;
}

// Counters of a two-stage launch: start + one per stage, padded to 256 B.
constexpr size_t kMlpCtrBytes = 256;

size_t w8a16_mlp_workspace_bytes(int M, int F) {
    const size_t h = static_cast<size_t>(std::max(M, 0)) * std::max(F, 0) * 2;
    return kMlpCtrBytes + ((h + 255) / 256) * 256;
}

// y = fc2(act(fc1(x))) [+ residual] as one launch of the persistent kernel:
// stage 0 writes h = act(x·W1ᵀ·s1 + b1) (bf16, [M, F]) into the workspace,
// stage 1 reads it. The workspace holds the counters (cleared on every call)
// and h.
int w8a16_mlp_launch(const void* x, int64_t ldx, const int8_t* w1, const float* s1, const void* b1,
                     const int8_t* w2, const float* s2, const void* b2, const void* residual, int64_t ldr,
                     void* y, int64_t ldy, int32_t y_dtype, int32_t M, int32_t K, int32_t F, int32_t N,
                     int32_t act, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    if (x == nullptr || w1 == nullptr || s1 == nullptr || w2 == nullptr || s2 == nullptr || y == nullptr ||
        workspace == nullptr)
        return SFB_ERR_INVALID;
    if (M < 1 || M > dense::kBN || K < 1 || F < 1 || N < 1) return SFB_ERR_SHAPE;
    if (N % 64 != 0 || F % 64 != 0) return SFB_ERR_SHAPE;
    if (y_dtype != SFB_BF16 && y_dtype != SFB_F32) return SFB_ERR_DTYPE;
    if (act < 0 || act > 2) return SFB_ERR_INVALID;
    if (ldy < N || (residual != nullptr && ldr < N) || ldx < K) return SFB_ERR_SHAPE;
    auto aligned16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    if (!aligned16(x) || !aligned16(w1) || !aligned16(w2) || (ldx * 2) % 16 != 0 ||
        (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
        return SFB_ERR_ALIGN;
    if (workspace_bytes < w8a16_mlp_workspace_bytes(M, F)) return SFB_ERR_WORKSPACE;
    const DeviceInfo& dev = device_info();
    if (!is_sm100(dev)) return SFB_ERR_UNSUPPORTED;
    const int ncl = dense_clusters(dev);
    if (ncl <= 0) { record_cuda_error(cudaErrorInvalidConfiguration, "dense kernel clusters"); return SFB_ERR_LAUNCH; }
    unsigned long long* ctr = static_cast<unsigned long long*>(workspace);
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(workspace) + kMlpCtrBytes);
    dense::DenseStagePair p;
    std::memset(&p, 0, sizeof(p));
    DenseStage& a = p.s[0];
    DenseStage& b = p.s[1];
    SFB_TRY(dense_stage_init(a, x, ldx, M, w1, F, K, 64));
    a.w_scale = s1; a.bias = static_cast<const __nv_bfloat16*>(b1); a.y = h; a.ldy = F; a.act = act; a.eps = 1e-6f;
    SFB_TRY(dense_stage_init(b, h, F, M, w2, N, F, 64));
    b.w_scale = s2; b.bias = static_cast<const __nv_bfloat16*>(b2); b.residual = residual; b.ldr = ldr;
    b.y = y; b.ldy = ldy; b.y_f32 = y_dtype == SFB_F32 ? 1 : 0; b.eps = 1e-6f;
    // every call starts its counters from zero (one generation per call)
    cudaError_t e = cudaMemsetAsync(ctr, 0, kMlpCtrBytes, stream);
    if (e != cudaSuccess) { record_cuda_error(e, "mlp counters"); return SFB_ERR_CUDA; }
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = dense_config(ncl, stream, attr, false);
    e = cudaLaunchKernelEx(&cfg, dense::dense_pair_kernel, p, ctr, M);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        record_cuda_error(e, "mlp launch");
        return SFB_ERR_LAUNCH;
    }
    return SFB_OK;
}

}  // namespace sfb
