// attn_tc.cu — tensor-core attention forward for sm_100a (head_dim 64,
// fp16/bf16 in, fp32 softmax/accumulate).
//
// Replaces the reference's FlashAttention-2 SM80 forward
// (src/backend/cuda/flash_attn/flash_fwd_kernel.h:52-497, reached through
// src/backend/cuda/ops/attention.cu:29-80) with a Blackwell design built for
// RDT-1B's shapes: Lq = 67 action tokens against Lk ∈ {67, 1024 (masked
// language), 4374 (image)}.
//
// One CTA = 128 query rows × a contiguous range of 128-key tiles, 9 warps:
//   * warp 8 (control): TMA loads (SWIZZLE_128B) of Q once and of K/V tiles
//     through a 4-deep ring, and every tcgen05.mma: S_j = Q·K_jᵀ (M=128,
//     N=128, K=64) into one of two TMEM S/P buffers, then O += P_j·V_j
//     (M=128, N=64, K=128) with P read from TMEM and O accumulated in TMEM
//     across all tiles.
//   * warps 0-7 (softmax): warps w and w+4 share TMEM lanes 32·(w%4)..+31
//     (query rows) and split the 128 key columns in halves; the row max is
//     exchanged through shared memory under a 64-thread named barrier.
//     P is written back over S in TMEM as two bf16 (or fp16) parts,
//     P = P_hi + P_lo, both multiplied into V, so the probabilities keep
//     ~16 significant bits (plain bf16 P costs up to 2^-9 relative per weight,
//     6e-3 absolute on few-key rows). The running max is a lazy reference:
//     O in TMEM is rescaled only when a tile raises the max by more than
//     8 (log2 units).
//   * Only warps whose rows hold queries work (Lq = 67 → 6 of 8).
//   * Split-K over Lk: the CTAs of one (batch, head, q-tile) form a thread-
//     block cluster; each keeps (O, m, l) for its key range, and the partials
//     are merged through distributed shared memory. No global scratch, no
//     atomics, no inter-CTA spin waits (cluster barriers are hardware).
//
// TMEM (512 columns): S/P buffer 0 at [0,128), buffer 1 at [128,256)
// (P_hi over columns [0,64) of a buffer, P_lo over [64,128)), O at [256,320).
//
// Every mbarrier wait is bounded (1 s); after an expiry a thread stops
// waiting, skips its output and records SFB_ERR_DEVICE_TIMEOUT in
// g_sfb_device_error; control flow stays uniform so no barrier is left
// half-arrived.
#include "common.cuh"
#include "sm100_ptx.cuh"

namespace sfb {

struct AttnTcParams {
    void*    out;
    int64_t  o_sb, o_sh, o_ss;       // element strides of out
    int32_t  B, H, Hkv, Lq, Lk, qtiles;
    int32_t  splits;                 // cluster size along grid.x
    int32_t  causal;
    float    sl2;                    // softmax scale · log2(e)
    const int32_t* kv_len;
    const uint8_t* key_mask;
    int64_t  mask_sb;
#ifdef SFB_TRACE
    unsigned long long* trace;
#endif
};

namespace attn_tc {

#ifdef SFB_TRACE
#define SFB_T(i) do { if (p.trace && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && \
                          (threadIdx.x == 0 || threadIdx.x == 256)) { \
        p.trace[(threadIdx.x == 0 ? 0 : 256) + (i)] = clock64(); } } while (0)
#else
#define SFB_T(i) do { } while (0)
#endif

constexpr int kSoftWarps = 8;
constexpr int kCtrlWarp  = 8;
constexpr int kThreads   = (kSoftWarps + 1) * 32;          // 288
constexpr int kStages    = 4;
constexpr int kTileKeys  = 128;
constexpr int kTileBytes = 128 * 128;                       // 128 rows × 64 halves
constexpr int kOffQ      = 0;
constexpr int kOffStage  = kOffQ + kTileBytes;              // [kStages] × (K, V)
constexpr int kOffBar    = kOffStage + kStages * 2 * kTileBytes;
constexpr int kNumBars   = 1 + 2 * kStages + 2 + 2 + 2;
constexpr int kOffTmem   = kOffBar + 8 * 16;
constexpr int kOffRed    = kOffTmem + 16;                   // float [2][2][128] row max
constexpr int kOffRedL   = kOffRed + 2 * 2 * 128 * 4;       // float [2][128] row sum
constexpr int kSmemUsed  = kOffRedL + 2 * 128 * 4;
constexpr int kSmemBytes = kSmemUsed + 1024;                // + alignment slack
constexpr int kTmemCols  = 512;
constexpr uint32_t kTmemO = 256;
// Split-K merge buffers reuse the stage region once the main loop is done.
constexpr int kOStride   = 68;                              // floats per row
constexpr int kOffCombO  = kOffStage;
// at most rows + C - 1 <= 143 row slots of (O row, m, l)
static_assert(143 * (kOStride + 2) * 4 <= kStages * 2 * kTileBytes, "merge buffers must fit in the stage region");
static_assert(kNumBars <= 16, "barrier area");

// barrier indices
constexpr int kBarQ = 0;
__host__ __device__ constexpr int bar_k(int s) { return 1 + s; }
__host__ __device__ constexpr int bar_v(int s) { return 1 + kStages + s; }
__host__ __device__ constexpr int bar_s(int b) { return 1 + 2 * kStages + b; }      // S_j ready
__host__ __device__ constexpr int bar_p(int b) { return 3 + 2 * kStages + b; }      // P_j written
__host__ __device__ constexpr int bar_o(int b) { return 5 + 2 * kStages + b; }      // PV_j done

template <typename T> struct HalfOps;
template <> struct HalfOps<__nv_bfloat16> {
    static constexpr uint32_t kFmt = 1;
    static __device__ __forceinline__ uint32_t pack(float a, float b) {
        __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    }
    static __device__ __forceinline__ float2 unpack(uint32_t u) {
        return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u));
    }
};
template <> struct HalfOps<__half> {
    static constexpr uint32_t kFmt = 0;
    static __device__ __forceinline__ uint32_t pack(float a, float b) {
        __half2 v = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    }
    static __device__ __forceinline__ float2 unpack(uint32_t u) {
        return __half22float2(*reinterpret_cast<__half2*>(&u));
    }
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                   const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV,
                   const AttnTcParams p) {
    using namespace ptx;
    using HO = HalfOps<T>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t*  sQ   = smem + kOffQ;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kOffTmem);
    float*    red  = reinterpret_cast<float*>(smem + kOffRed);     // [2 parity][2 half][128]
    float*    redl = reinterpret_cast<float*>(smem + kOffRedL);    // [2 half][128]
    auto sK = [&](int s) { return smem + kOffStage + (2 * s) * kTileBytes; };
    auto sV = [&](int s) { return smem + kOffStage + (2 * s + 1) * kTileBytes; };

    const int tid  = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int split = blockIdx.x;
    const int h     = blockIdx.y;
    const int b     = blockIdx.z / p.qtiles;
    const int qt    = blockIdx.z - b * p.qtiles;
    const int hk    = h / (p.H / p.Hkv);
    const int q0    = qt * 128;
    const int rows  = min(128, p.Lq - q0);
    const int groups = (rows + 31) >> 5;            // active 32-row groups
    const int nsoft  = 2 * groups;                  // active softmax warps

    // Key range of this (batch, q-tile), then this CTA's share of its tiles.
    int kend = p.Lk;
    if (p.kv_len != nullptr) kend = min(kend, max(0, p.kv_len[b]));
    if (p.causal) kend = min(kend, q0 + rows);
    const int ntiles  = (kend + kTileKeys - 1) / kTileKeys;
    const int tbase   = ntiles / p.splits;
    const int trem    = ntiles - tbase * p.splits;
    const int t_begin = split * tbase + min(split, trem);
    const int ntl     = tbase + (split < trem ? 1 : 0);

    SFB_T(0);
    if (tid == kCtrlWarp * 32) {
        mbar_init(&bars[kBarQ], 1);
        for (int s = 0; s < kStages; ++s) { mbar_init(&bars[bar_k(s)], 1); mbar_init(&bars[bar_v(s)], 1); }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars[bar_s(i)], 1);
            mbar_init(&bars[bar_p(i)], nsoft);
            mbar_init(&bars[bar_o(i)], 1);
        }
        fence_mbarrier_init();
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    if (warp == 0) {
        tmem_alloc(tmem_holder, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem = *tmem_holder;
    SFB_T(1);

    bool ok = true;
    auto wait = [&](int bar, uint32_t parity) {
        if (!mbar_wait(&bars[bar], parity, ok ? 1000000000ull : 0ull)) ok = false;
    };

    float o_part[32];                   // this thread's 32 output columns (softmax warps)
    float m_ref = -INFINITY, l_run = 0.f;
    const int grp  = warp & 3;          // row group
    const int half = warp >> 2;         // key-column half (softmax warps)
    const int row  = grp * 32 + lane;

    if (warp == kCtrlWarp) {
        // ── control warp: TMA + MMA issue (one thread) ──────────────────────
        if (lane == 0 && ntl > 0) {
            constexpr uint32_t idS  = idesc_f16(128, 128, HO::kFmt, 0, 0);  // Q·Kᵀ, both K-major
            constexpr uint32_t idPV = idesc_f16(128, 64, HO::kFmt, 0, 1);   // P(tmem)·V(MN-major)
            constexpr bool kSplitP  = std::is_same<T, __nv_bfloat16>::value;
            auto issue_kv = [&](int tile_idx) {
                const int s = tile_idx % kStages;
                const int key0 = (t_begin + tile_idx) * kTileKeys;
                mbar_arrive_expect_tx(&bars[bar_k(s)], kTileBytes);
                tma_load_4d(sK(s), &tmK, &bars[bar_k(s)], 0, key0, hk, b);
                mbar_arrive_expect_tx(&bars[bar_v(s)], kTileBytes);
                tma_load_4d(sV(s), &tmV, &bars[bar_v(s)], 0, key0, hk, b);
            };
            auto issue_pv = [&](int j) {
                const int bf = j & 1, s = j % kStages;
                wait(bar_p(bf), (j >> 1) & 1);
                wait(bar_v(s), (j / kStages) & 1);
                tc_fence_after_sync();
                const uint32_t tP = tmem + bf * 128;
                const uint32_t av = smem_u32(sV(s));
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    mma_f16_ts(tmem + kTmemO, tP + 8 * k, smem_desc_sw128(av + k * 2048, 8192, 1024),
                               idPV, (j > 0 || k > 0) ? 1u : 0u);
                if (kSplitP) {
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        mma_f16_ts(tmem + kTmemO, tP + 64 + 8 * k,
                                   smem_desc_sw128(av + k * 2048, 8192, 1024), idPV, 1u);
                }
                mma_commit(&bars[bar_o(bf)]);
            };
            mbar_arrive_expect_tx(&bars[kBarQ], kTileBytes);
            tma_load_4d(sQ, &tmQ, &bars[kBarQ], 0, q0, h, b);
            for (int t = 0; t < min(kStages, ntl); ++t) issue_kv(t);
            wait(kBarQ, 0);
            const uint32_t aq = smem_u32(sQ);
            for (int j = 0; j < ntl; ++j) {
                const int bf = j & 1, s = j % kStages;
                if (j >= 2) {
                    // PV_{j-2} done: S/P buffer bf and stage (j-2)%kStages are free
                    wait(bar_o(bf), ((j - 2) >> 1) & 1);
                    if (j + 2 < ntl && j + 2 >= kStages) issue_kv(j + 2);
                }
                wait(bar_k(s), (j / kStages) & 1);
                tc_fence_after_sync();
                const uint32_t ak = smem_u32(sK(s));
                const uint32_t tS = tmem + bf * 128;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    mma_f16_ss(tS, smem_desc_sw128(aq + kk * 32, 16, 1024),
                               smem_desc_sw128(ak + kk * 32, 16, 1024), idS, kk > 0 ? 1u : 0u);
                mma_commit(&bars[bar_s(bf)]);
                SFB_T(2 + 6 * j);
                if (j >= 1) issue_pv(j - 1);
                SFB_T(3 + 6 * j);
            }
            issue_pv(ntl - 1);
        }
    } else if (grp < groups) {
        // ── softmax warps ───────────────────────────────────────────────────
        const uint32_t lane_off = static_cast<uint32_t>(grp * 32) << 16;
        const int qi = q0 + row;
        const float sl2 = p.sl2;
        const bool use_mask = p.key_mask != nullptr;
        const uint32_t bar_id = 1 + grp;
        for (int j = 0; j < ntl; ++j) {
            const int bf = j & 1;
            const uint32_t tS = tmem + bf * 128 + lane_off;
            const int key0 = (t_begin + j) * kTileKeys + half * 64;
            SFB_T(2 + 6 * j);
            wait(bar_s(bf), (j >> 1) & 1);
            SFB_T(3 + 6 * j);
            tc_fence_after_sync();
            float sc[64];
            tmem_ld32(tS + half * 64, *reinterpret_cast<float(*)[32]>(&sc[0]));
            tmem_ld32(tS + half * 64 + 32, *reinterpret_cast<float(*)[32]>(&sc[32]));
            tmem_ld_wait();
            const bool full = (key0 + 64 <= kend) && !use_mask && !p.causal;
            if (!full) {
                const uint8_t* mrow = use_mask ? p.key_mask + static_cast<int64_t>(b) * p.mask_sb : nullptr;
#pragma unroll
                for (int i = 0; i < 64; ++i) {
                    const int key = key0 + i;
                    bool v = key < kend;
                    if (use_mask && v) v = mrow[key] != 0;
                    if (p.causal) v = v && key <= qi;
                    if (!v) sc[i] = -INFINITY;
                }
            }
            float mxa = sc[0], mxb = sc[1], mxc = sc[2], mxd = sc[3];
#pragma unroll
            for (int i = 4; i < 64; i += 4) {
                mxa = fmaxf(mxa, sc[i]); mxb = fmaxf(mxb, sc[i + 1]);
                mxc = fmaxf(mxc, sc[i + 2]); mxd = fmaxf(mxd, sc[i + 3]);
            }
            float mx = fmaxf(fmaxf(mxa, mxb), fmaxf(mxc, mxd));
            // exchange the half-row max with the partner warp
            red[(bf * 2 + half) * 128 + row] = mx;
            tc_fence_before_sync();
            SFB_T(4 + 6 * j);
            named_bar_sync(bar_id, 64);
            SFB_T(5 + 6 * j);
            tc_fence_after_sync();
            mx = fmaxf(mx, red[(bf * 2 + (half ^ 1)) * 128 + row]);
            const float m_tile = mx == -INFINITY ? -INFINITY : mx * sl2;
            if (m_tile > m_ref + 8.f) {          // also true when m_ref == -inf
                if (m_ref != -INFINITY) {
                    const float alpha = ptx::ex2(m_ref - m_tile);
                    l_run *= alpha;
                    // O holds PV_0..PV_{j-1}: wait for PV_{j-1}, rescale our 32 columns
                    wait(bar_o((j - 1) & 1), ((j - 1) >> 1) & 1);
                    tc_fence_after_sync();
                    float ot[32];
                    tmem_ld32(tmem + kTmemO + lane_off + half * 32, ot);
                    tmem_ld_wait();
                    uint32_t ou[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) ou[i] = __float_as_uint(ot[i] * alpha);
                    tmem_st32(tmem + kTmemO + lane_off + half * 32, ou);
                }
                m_ref = m_tile;
            }
            const float m_use = m_ref == -INFINITY ? 0.f : m_ref;
            uint32_t phi[32], plo[32];
            float lsum0 = 0.f, lsum1 = 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const float p0 = ptx::ex2(fmaf(sc[2 * i], sl2, -m_use));
                const float p1 = ptx::ex2(fmaf(sc[2 * i + 1], sl2, -m_use));
                lsum0 += p0;
                lsum1 += p1;
                if (std::is_same<T, __nv_bfloat16>::value) {
                    // hi = p truncated to bf16 (exact top 16 bits), lo = p - hi (exact in
                    // fp32), truncated to bf16 as well: hi + lo carries 16 significant bits.
                    const uint32_t u0 = __float_as_uint(p0), u1 = __float_as_uint(p1);
                    const float lo0 = p0 - __uint_as_float(u0 & 0xffff0000u);
                    const float lo1 = p1 - __uint_as_float(u1 & 0xffff0000u);
                    phi[i] = ptx::prmt(u0, u1, 0x7632u);
                    plo[i] = ptx::prmt(__float_as_uint(lo0), __float_as_uint(lo1), 0x7632u);
                } else {
                    phi[i] = HO::pack(p0, p1);
                }
            }
            const float lsum = lsum0 + lsum1;
            l_run += lsum;
            // P_hi over S columns [0,64), P_lo over [64,128) of this buffer; the
            // partner warp's S half was consumed before the named barrier.
            SFB_T(6 + 6 * j);
            tmem_st32(tS + half * 32, phi);
            if (std::is_same<T, __nv_bfloat16>::value) tmem_st32(tS + 64 + half * 32, plo);
            tmem_st_wait();
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[bar_p(bf)]);
            SFB_T(7 + 6 * j);
        }
        // final O: wait for the last PV, read our 32 columns
        if (ntl > 0) {
            wait(bar_o((ntl - 1) & 1), ((ntl - 1) >> 1) & 1);
            tc_fence_after_sync();
            tmem_ld32(tmem + kTmemO + lane_off + half * 32, o_part);
            tmem_ld_wait();
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) o_part[i] = 0.f;
        }
        // full row sum
        redl[half * 128 + row] = l_run;
        named_bar_sync(bar_id, 64);
        l_run += redl[(half ^ 1) * 128 + row];
    }
    SFB_T(200);

    // ── epilogue ────────────────────────────────────────────────────────────
    T* out = static_cast<T*>(p.out);
    const int64_t row_base = static_cast<int64_t>(b) * p.o_sb + static_cast<int64_t>(h) * p.o_sh;
    const bool has_rows = warp < kSoftWarps && grp < groups && row < rows;
    if (p.splits == 1) {
        if (has_rows && ok) {
            const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
            T* dst = out + row_base + static_cast<int64_t>(q0 + row) * p.o_ss + half * 32;
#pragma unroll
            for (int c = 0; c < 32; c += 8) {
                uint4 u;
                u.x = HO::pack(o_part[c + 0] * inv, o_part[c + 1] * inv);
                u.y = HO::pack(o_part[c + 2] * inv, o_part[c + 3] * inv);
                u.z = HO::pack(o_part[c + 4] * inv, o_part[c + 5] * inv);
                u.w = HO::pack(o_part[c + 6] * inv, o_part[c + 7] * inv);
                *reinterpret_cast<uint4*>(dst + c) = u;
            }
        }
    } else {
        // Row r is owned by CTA r % C at slot r / C. Every CTA pushes its partial
        // (O row, m, l) into the owner's shared memory with remote stores, one
        // cluster barrier publishes them, and each owner merges its rows locally.
        const int C = p.splits;
        const int slots = (rows + C - 1) / C;
        float* sO = reinterpret_cast<float*>(smem + kOffCombO);        // [C][slots][kOStride]
        float* sM = sO + C * slots * kOStride;                         // [C][slots]
        float* sL = sM + C * slots;                                    // [C][slots]
        cluster_sync();   // every CTA is past its main loop: stage regions are free
        if (has_rows) {
            const int owner = row % C, slot = row / C;
            const uint32_t dO = dsmem_map(smem_u32(sO + (split * slots + slot) * kOStride + half * 32), owner);
#pragma unroll
            for (int c = 0; c < 32; c += 4)
                dsmem_st_f32x4(dO + c * 4, make_float4(o_part[c], o_part[c + 1], o_part[c + 2], o_part[c + 3]));
            if (half == 0) {
                dsmem_st_f32(dsmem_map(smem_u32(sM + split * slots + slot), owner), m_ref);
                dsmem_st_f32(dsmem_map(smem_u32(sL + split * slots + slot), owner), l_run);
            }
        }
        cluster_sync();
        const int nsub = kThreads / 16;
        const int sub  = tid >> 4, c4 = (tid & 15) * 4;
        for (int slot = sub; slot < slots; slot += nsub) {
            const int r = slot * C + split;
            if (r >= rows) break;
            float M = -INFINITY;
            for (int k = 0; k < C; ++k) M = fmaxf(M, sM[k * slots + slot]);
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            float L = 0.f;
            if (M != -INFINITY) {
                for (int k = 0; k < C; ++k) {
                    const float w = ptx::ex2(sM[k * slots + slot] - M);
                    L += w * sL[k * slots + slot];
                    const float4 o = *reinterpret_cast<const float4*>(sO + (k * slots + slot) * kOStride + c4);
                    acc.x += w * o.x; acc.y += w * o.y; acc.z += w * o.z; acc.w += w * o.w;
                }
            }
            const float inv = L > 0.f ? 1.f / L : 0.f;
            if (ok) {
                T* dst = out + row_base + static_cast<int64_t>(q0 + r) * p.o_ss + c4;
                uint2 u;
                u.x = HO::pack(acc.x * inv, acc.y * inv);
                u.y = HO::pack(acc.z * inv, acc.w * inv);
                *reinterpret_cast<uint2*>(dst) = u;
            }
        }
    }

    SFB_T(201);
    if (!ok) atomicExch(&g_sfb_device_error, SFB_ERR_DEVICE_TIMEOUT);
    tc_fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after_sync();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace attn_tc

// ── host launcher ───────────────────────────────────────────────────────────
static int make_map_4d(CUtensorMap* map, const void* base, CUtensorMapDataType dt,
                       int64_t d0, int64_t d1, int64_t d2, int64_t d3,
                       int64_t s1_elems, int64_t s2_elems, int64_t s3_elems, int elem_bytes,
                       uint32_t box0, uint32_t box1) {
    cuuint64_t dims[4]    = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2, (cuuint64_t)d3};
    cuuint64_t strides[3] = {(cuuint64_t)(s1_elems * elem_bytes), (cuuint64_t)(s2_elems * elem_bytes),
                             (cuuint64_t)(s3_elems * elem_bytes)};
    cuuint32_t box[4]     = {box0, box1, 1, 1};
    cuuint32_t estr[4]    = {1, 1, 1, 1};
    return encode_tensor_map(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr,
                             CU_TENSOR_MAP_SWIZZLE_128B);
}

#ifdef SFB_TRACE
static unsigned long long* g_trace_ptr = nullptr;
extern "C" void sfb_debug_set_trace(void* p) { g_trace_ptr = static_cast<unsigned long long*>(p); }
#endif

// Cluster size along Lk: as many splits as keep every CTA co-resident in one
// wave (one CTA per SM), at least two key tiles per split.
int choose_attn_splits(int units, int ntiles_max, int num_sms) {
    int s = std::max(1, num_sms / std::max(units, 1));
    s = std::min(s, 16);
    s = std::min(s, std::max(1, ntiles_max / 2));
    return s;
}

int attention_tc_launch(const sfb_attn_args& a, cudaStream_t stream) {
    const int eb = 2;
    const CUtensorMapDataType dt =
        a.dtype == SFB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    // TMA: 16-byte aligned bases and byte strides.
    auto aligned16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
    if (!aligned16(a.q) || !aligned16(a.k) || !aligned16(a.v) || !aligned16(a.out)) return SFB_ERR_ALIGN;
    for (int i = 0; i < 3; ++i) {
        if ((a.q_stride[i] * eb) % 16 || (a.k_stride[i] * eb) % 16 || (a.v_stride[i] * eb) % 16 ||
            (a.out_stride[i] * eb) % 16)
            return SFB_ERR_ALIGN;
    }
    CUtensorMap mq, mk, mv;
    int rc;
    if ((rc = make_map_4d(&mq, a.q, dt, 64, a.seq_q, a.heads, a.batch, a.q_stride[2], a.q_stride[1],
                          a.q_stride[0], eb, 64, 128)) != SFB_OK) return rc;
    if ((rc = make_map_4d(&mk, a.k, dt, 64, a.seq_k, a.heads_kv, a.batch, a.k_stride[2], a.k_stride[1],
                          a.k_stride[0], eb, 64, 128)) != SFB_OK) return rc;
    if ((rc = make_map_4d(&mv, a.v, dt, 64, a.seq_k, a.heads_kv, a.batch, a.v_stride[2], a.v_stride[1],
                          a.v_stride[0], eb, 64, 128)) != SFB_OK) return rc;

    const DeviceInfo& dev = device_info();
    AttnTcParams p{};
    p.out = a.out;
    p.o_sb = a.out_stride[0]; p.o_sh = a.out_stride[1]; p.o_ss = a.out_stride[2];
    p.B = a.batch; p.H = a.heads; p.Hkv = a.heads_kv; p.Lq = a.seq_q; p.Lk = a.seq_k;
    p.qtiles = (a.seq_q + 127) / 128;
    p.causal = a.is_causal ? 1 : 0;
    const float scale = a.scale == 0.f ? 1.f / sqrtf(static_cast<float>(a.head_dim)) : a.scale;
    p.sl2 = scale * 1.4426950408889634f;
    p.kv_len = a.kv_len;
    p.key_mask = a.key_mask;
    p.mask_sb = a.key_mask_stride_b;
#ifdef SFB_TRACE
    p.trace = g_trace_ptr;
#endif
    const int units = a.batch * a.heads * p.qtiles;
    const int ntiles_max = (a.seq_k + 127) / 128;
    p.splits = a.num_splits > 0 ? std::min(a.num_splits, 16)
                                : choose_attn_splits(units, ntiles_max, dev.num_sms);
    if (p.splits > std::max(1, ntiles_max)) p.splits = std::max(1, ntiles_max);
    if ((p.o_ss % 8) != 0 && p.splits == 1) return SFB_ERR_ALIGN;

    auto kern = a.dtype == SFB_BF16 ? attn_tc::attn_fwd_tc_kernel<__nv_bfloat16>
                                    : attn_tc::attn_fwd_tc_kernel<__half>;
    static bool attr_done[2][64] = {};
    const int ki = a.dtype == SFB_BF16 ? 0 : 1;
    if (!attr_done[ki][dev.ordinal & 63]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 attn_tc::kSmemBytes) != cudaSuccess ||
            cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
            return SFB_ERR_CUDA;
        attr_done[ki][dev.ordinal & 63] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim  = dim3(p.splits, a.heads, a.batch * p.qtiles);
    cfg.blockDim = dim3(attn_tc::kThreads, 1, 1);
    cfg.dynamicSmemBytes = attn_tc::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = p.splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mq, mk, mv, p);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return SFB_ERR_LAUNCH;
    }
    return SFB_OK;
}

}  // namespace sfb
