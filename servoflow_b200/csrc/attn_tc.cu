// attn_tc.cu — tensor-core attention forward for sm_100a (head_dim 64,
// fp16/bf16 in, fp32 softmax/accumulate).
//
// Replaces the reference's FlashAttention-2 SM80 forward
// (src/backend/cuda/flash_attn/flash_fwd_kernel.h:52-497, reached through
// src/backend/cuda/ops/attention.cu:29-80) with a Blackwell design built for
// RDT-1B's shapes: Lq = 67 action tokens against Lk ∈ {67, 1024 (masked
// language), 4374 (image)}.
//
// One CTA = 128 query rows × a contiguous range of 128-key tiles, 12 warps:
//   * warp 11 (control): TMA loads (SWIZZLE_128B) of Q once and of K/V tiles
//     through a 5-deep ring, and every tcgen05.mma: S_j = Q·K_jᵀ (M=128,
//     N=128, K=64) into TMEM, then O_g += P_j·V_j (M=128, N=64, K=128) with
//     P read from TMEM. It runs an event loop (non-blocking mbarrier probes)
//     that issues whichever of {K/V refill, next S, next P·V} is ready, and it
//     sits alone on SM sub-partition 3 whenever Lq <= 96 (the softmax warps of
//     rows 96..127 are then idle), so its spinning steals no issue slots.
//   * Two softmax groups ping-pong over the key tiles, FlashAttention-4 style
//     but along Lk (there is a single 67-row Q tile): group g (warps 4g..4g+3)
//     takes the tiles j ≡ g (mod 2), owns accumulator O_g and keeps its own
//     running max / sum. Thread = query row = TMEM lane, so row reductions
//     are thread-local and the two groups never wait for each other; their
//     latencies overlap. O_A and O_B are merged once at the end.
//   * P is written to TMEM as fp16 (11 significant bits; a bf16 P, 8 bits,
//     costs up to 2^-9 relative per weight — 6e-3 absolute on few-key rows).
//     The P·V product therefore runs in fp16: for bf16 inputs, warps 8..10
//     convert each V tile to fp16 in shared memory (exact for |v| <= 65504;
//     larger values record SFB_ERR_RANGE). The running max is a lazy
//     reference: O_g in TMEM is rescaled only when a tile raises the max by
//     more than 8 (log2 units), which keeps P <= 256.
//   * Only warps whose rows hold queries work (Lq = 67 → 3 of 4 per group).
//   * Split-K over Lk: the CTAs of one (batch, head, q-tile) form a thread-
//     block cluster; each pushes its (O, m, l) rows into the owning CTA's
//     dedicated merge buffer with remote shared-memory stores, one cluster
//     barrier publishes them, and each owner merges its rows locally. No
//     global scratch, no atomics, no inter-CTA spin waits.
//
// TMEM (512 columns): three S/P buffers at [128u, 128u+128) — tile j uses
// buffer j mod 3, so a tile's S MMA waits only for the P·V three tiles back;
// the fp16 P of keys [32c, 32c+32) overwrites the first 16 of that chunk's
// own 32 S columns — and O_g at [384+64g, 448+64g). Three warps per SM
// sub-partition cap a thread at 168 registers: S is read in 32-column chunks,
// twice (row max, then exponentials), and the hot loop is kept compact
// (rolled chunk loops; masked keys are set to -inf in TMEM during the first
// pass), because instruction-fetch stalls dominated a fully unrolled form.
//
// Measured on B200 while designing this (microbenchmarks): MUFU ex2 runs at
// 16 results/clk/SM; tcgen05.mma M=128 at N=64 takes 48 cycles (66% of peak)
// and at N>=128 runs at full rate, with A from TMEM as fast as from smem.
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
    int32_t  v_f16;                  // bf16 Q/K with V already in fp16: no in-kernel conversion
    const __nv_bfloat16* qn_w;       // per-head RMSNorm weight [64] applied to Q rows, or null
    const __nv_bfloat16* kn_w;       // the same for K rows, or null
    float    norm_eps;
    int32_t  kv_stream;              // K/V read once per use (a per-tick cache): L2 evict-first
    const void* amask;               // additive mask, added to the scaled logits (keys contiguous)
    int32_t  am_dt;
    int64_t  am_sb, am_ss;           // element strides: batch, query row (0 = broadcast)
    float    inv_scale;              // 1 / softmax scale: the mask enters the raw logits as m / scale
#ifdef SFB_TRACE
    unsigned long long* trace;
    int dbg_skip;                    // timing experiments only: return at once
    unsigned long long* tl;
    int tl_launch;
#endif
};

namespace attn_tc {

#ifdef SFB_TRACE
#define SFB_T(i) do { if (p.trace && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && \
                          (threadIdx.x == 0 || threadIdx.x == 128 || threadIdx.x == 352)) { \
        p.trace[(threadIdx.x == 352 ? 2 : threadIdx.x / 128) * 170 + (i)] = ptx::global_timer_ns(); } } while (0)
#else
#define SFB_T(i) do { } while (0)
#endif

constexpr int kSoftWarps = 8;
constexpr int kConvWarp0 = 8;                               // warps 8..10: bf16 V → fp16
constexpr int kConvWarps = 3;
constexpr int kCtrlWarp  = 11;                              // 11 % 4 == 3
constexpr int kThreads   = 12 * 32;                         // 384
constexpr int kStages    = 5;
constexpr int kBufs      = 3;                               // TMEM S/P buffers
constexpr int kTileKeys  = 128;
constexpr int kTileBytes = 128 * 128;                       // 128 rows × 64 halves
constexpr int kMaxSplits = 16;
constexpr int kOStride   = 36;                              // floats per merge half-row
constexpr int kMergeRows = 128 + kMaxSplits - 1;            // row slots over all sources
constexpr int kOffQ      = 0;
constexpr int kOffStage  = kOffQ + kTileBytes;              // [kStages] × (K, V)
constexpr int kOffMerge  = kOffStage + kStages * 2 * kTileBytes;
constexpr int kMergeBytes = kMergeRows * (2 * kOStride + 2) * 4;
constexpr int kOffBar    = kOffMerge + kMergeBytes;
constexpr int kOffTmem   = kOffBar + 8 * 40;
constexpr int kOffRed    = kOffTmem + 16;                   // float [2 groups][m|l][128]
constexpr int kOffNormW  = (kOffRed + 2 * 2 * 128 * 4 + 15) & ~15;   // bf16 q/k norm weights [2][64]
constexpr int kSmemUsed  = kOffNormW + 2 * 64 * 2;
constexpr int kSmemBytes = kSmemUsed + 1024;                // + alignment slack
constexpr int kTmemCols  = 512;
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
static_assert(kOffNormW % 16 == 0 && kOffQ % 1024 == 0 && kOffStage % 1024 == 0, "vector/TMA alignment");
static_assert(kOffBar % 8 == 0, "barrier alignment");

// barrier indices
constexpr int kBarQ = 0;
__host__ __device__ constexpr int bar_k(int s) { return 1 + s; }
__host__ __device__ constexpr int bar_v(int s) { return 1 + kStages + s; }
__host__ __device__ constexpr int bar_vc(int s) { return 1 + 2 * kStages + s; }              // V in fp16
__host__ __device__ constexpr int bar_s(int u) { return 1 + 3 * kStages + u; }               // S_j ready
__host__ __device__ constexpr int bar_p(int u) { return 1 + 3 * kStages + kBufs + u; }       // P_j written
__host__ __device__ constexpr int bar_o(int u) { return 1 + 3 * kStages + 2 * kBufs + u; }   // PV_j done
__host__ __device__ constexpr int bar_og(int g) { return 1 + 3 * kStages + 3 * kBufs + g; }  // group's PV done
constexpr int kBarQn = 3 + 3 * kStages + 3 * kBufs;                                        // Q rows normalised
__host__ __device__ constexpr int bar_kn(int s) { return kBarQn + 1 + s; }                  // K rows normalised
constexpr int kBarDrain = kBarQn + 1 + kStages;                                            // failure path: MMAs done
constexpr int kNumBars = kBarDrain + 1;
static_assert(kNumBars <= 40, "barrier area");
constexpr uint64_t kDrainNs = 100000000ull;        // bound of each wait for in-flight copies/MMAs after a failure

// RMS-normalises row r (64 bf16) of a 128-byte-swizzled [128 × 64] tile in
// place: x · 1/sqrt(mean(x²) + eps) · w, fp32 math, bf16 result. The sum of
// squares is formed as 8 per-chunk partials combined pairwise, the order of
// the standalone per-head RMSNorm kernel, so both give identical bits.
__device__ __forceinline__ void norm_row_sw128(uint8_t* tile, int r, const __nv_bfloat16* w_smem, float eps) {
    uint4 c[8];
    float part[8];
#pragma unroll
    for (int lc = 0; lc < 8; ++lc) {                // logical 16-byte chunk lc sits at lc ^ (r & 7)
        c[lc] = *reinterpret_cast<const uint4*>(tile + r * 128 + ((lc ^ (r & 7)) << 4));
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&c[lc]);
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
        }
        part[lc] = ss;
    }
    const float ss = ((part[0] + part[1]) + (part[2] + part[3])) + ((part[4] + part[5]) + (part[6] + part[7]));
    const float inv = 1.f / sqrtf(ss / 64.f + eps);
#pragma unroll
    for (int lc = 0; lc < 8; ++lc) {
        const uint4 gu = *reinterpret_cast<const uint4*>(w_smem + lc * 8);
        const __nv_bfloat162* g = reinterpret_cast<const __nv_bfloat162*>(&gu);
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&c[lc]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]), gg = __bfloat1622float2(g[i]);
            h[i] = __floats2bfloat162_rn(f.x * inv * gg.x, f.y * inv * gg.y);
        }
        *reinterpret_cast<uint4*>(tile + r * 128 + ((lc ^ (r & 7)) << 4)) = c[lc];
    }
}

template <typename T> struct HalfOps;
template <> struct HalfOps<__nv_bfloat16> {
    static __device__ __forceinline__ uint32_t pack(float a, float b) {
        __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    }
};
template <> struct HalfOps<__half> {
    static __device__ __forceinline__ uint32_t pack(float a, float b) {
        __half2 v = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    }
};

// Validity bits of keys [key, key+32) for one query row: key < kend_row and,
// with a key-padding mask, a nonzero mask byte. Mask rows are read 16 bytes
// at a time when aligned.
// The session whose valid length (clamped to [0, Lk]) has rank `rank` in
// descending order (ties by index); every lane of the calling warp gets it.
__device__ __forceinline__ int session_by_length_rank(const int32_t* len, int B, int Lk, int rank, int lane) {
    int found = rank;
    for (int base = 0; base < B; base += 32) {
        const int s = base + lane;
        int r = -1;
        if (s < B) {
            const int ls = min(Lk, max(0, len[s]));
            r = 0;
            for (int t = 0; t < B; ++t) {
                const int lt = min(Lk, max(0, len[t]));
                r += (lt > ls || (lt == ls && t < s)) ? 1 : 0;
            }
        }
        const unsigned m = __ballot_sync(0xffffffffu, r == rank);
        if (m != 0u) found = base + __ffs(m) - 1;
    }
    return found;
}

__device__ __forceinline__ uint32_t key_bits(const AttnTcParams& p, int b, int key, int kend_row) {
    const int n = kend_row - key;
    uint32_t bits = n >= 32 ? 0xffffffffu : (n <= 0 ? 0u : ((1u << n) - 1u));
    if (p.key_mask != nullptr && bits != 0u) {
        const uint8_t* m = p.key_mask + static_cast<int64_t>(b) * p.mask_sb + key;
        uint32_t mb = 0;
        if ((reinterpret_cast<uintptr_t>(m) & 15u) == 0 && key + 32 <= p.Lk) {
            const uint4 w0 = *reinterpret_cast<const uint4*>(m);
            const uint4 w1 = *reinterpret_cast<const uint4*>(m + 16);
            const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                // one bit per nonzero byte, gathered into 4 bits
                const uint32_t nz = (__vcmpne4(w[q], 0u) & 0x01010101u) * 0x01020408u;
                mb |= ((nz >> 24) & 0xfu) << (4 * q);
            }
        } else {
#pragma unroll 1
            for (int i = 0; i < 32; ++i)
                if (key + i < p.Lk && m[i] != 0) mb |= 1u << i;
        }
        bits &= mb;
    }
    return bits;
}

// kAMask: the instantiation that applies an additive mask (sfb_attn_args.
// attn_mask); the other carries no mask code, so its softmax loop keeps the
// compact body it was tuned with.
template <typename T, bool kAMask>
__global__ void __launch_bounds__(kThreads, 1)
attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                   const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV,
                   const AttnTcParams p) {
    using namespace ptx;
    using HO = HalfOps<T>;
    constexpr bool kConvV = std::is_same<T, __nv_bfloat16>::value;   // bf16 V needs an fp16 copy
    constexpr uint32_t kFmtQK = kConvV ? 1u : 0u;
    const bool conv_v = kConvV && !p.v_f16;          // bf16 V converted to fp16 here
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t*  sQ   = smem + kOffQ;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kOffTmem);
    float*    red  = reinterpret_cast<float*>(smem + kOffRed);
    auto sK = [&](int s) { return smem + kOffStage + (2 * s) * kTileBytes; };
    auto sV = [&](int s) { return smem + kOffStage + (2 * s + 1) * kTileBytes; };

    const int tid  = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int split = blockIdx.x;
    const int h     = blockIdx.y;
    int b           = blockIdx.z / p.qtiles;       // remapped below when sessions have lengths
    const int qt    = blockIdx.z % p.qtiles;
    const int hk    = h / (p.H / p.Hkv);
    const int q0    = qt * 128;
    const int rows  = min(128, p.Lq - q0);
    const int groups = (rows + 31) >> 5;            // active 32-row windows per group


#ifdef SFB_TRACE
    if (p.dbg_skip) { pdl_trigger(); pdl_wait(); return; }
#endif
    SFB_T(0);
#ifdef SFB_TRACE
    const uint64_t cta_t0 = ptx::global_timer_ns();
#endif
    if (tid == kCtrlWarp * 32) {
        mbar_init(&bars[kBarQ], 1);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars[bar_k(s)], 1);
            mbar_init(&bars[bar_v(s)], 1);
            mbar_init(&bars[bar_vc(s)], kConvWarps);
        }
        for (int u = 0; u < kBufs; ++u) {
            mbar_init(&bars[bar_s(u)], 1);
            mbar_init(&bars[bar_p(u)], groups);
            mbar_init(&bars[bar_o(u)], 1);
        }
        mbar_init(&bars[bar_og(0)], 1);
        mbar_init(&bars[bar_og(1)], 1);
        mbar_init(&bars[kBarQn], 4);
        for (int s = 0; s < kStages; ++s) mbar_init(&bars[bar_kn(s)], kConvWarps);
        mbar_init(&bars[kBarDrain], 1);
        fence_mbarrier_init();
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    if (warp == 0) {
        tmem_alloc(tmem_holder, kTmemCols);
        tmem_relinquish();
    }
    // the q/k norm weights (constant parameters) staged in shared memory
    __nv_bfloat16* norm_w = reinterpret_cast<__nv_bfloat16*>(smem + kOffNormW);
    if (warp == 1 && lane < 16) {
        const __nv_bfloat16* src = lane < 8 ? p.qn_w : p.kn_w;
        if (src != nullptr)
            reinterpret_cast<uint4*>(norm_w)[lane] = reinterpret_cast<const uint4*>(src)[lane & 7];
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem = *tmem_holder;
    // split-K: announce this CTA as started; the wait before the first store
    // into a peer's merge buffer then guarantees every peer is running
    if (p.splits > 1) cluster_arrive_relaxed();
    pdl_trigger();                       // TMEM is held: the next kernel may start
    pdl_wait();                          // Q/K/V, key lengths and the output belong to earlier kernels
#ifdef SFB_TRACE
    const unsigned long long tl_t1 = ptx::global_timer_ns();
#endif
    SFB_T(1);

    // With per-session lengths, CTA row z of the grid takes the session of
    // rank z by descending length, so the longest sessions' CTAs are scheduled
    // first and the last wave holds the short ones.
    if (p.kv_len != nullptr && p.B > 1 && p.B <= 64) b = session_by_length_rank(p.kv_len, p.B, p.Lk, b, lane);
    // Key range of this (batch, q-tile), then this CTA's share of its tiles.
    int kend = p.Lk;
    if (p.kv_len != nullptr) kend = min(kend, max(0, p.kv_len[b]));
    if (p.causal) kend = min(kend, q0 + rows);
    const int ntiles  = (kend + kTileKeys - 1) / kTileKeys;
    const int tbase   = ntiles / p.splits;
    const int trem    = ntiles - tbase * p.splits;
    const int t_begin = split * tbase + min(split, trem);
    const int ntl     = tbase + (split < trem ? 1 : 0);

    bool ok = true;
    auto wait = [&](int bar, uint32_t parity) {
        if (!mbar_wait(&bars[bar], parity, ok ? 1000000000ull : 0ull)) ok = false;
    };

    const int win = warp & 3;            // 32-lane window = row block
    const int grp = (warp >> 2) & 1;     // softmax group (tile parity)
    const int row = win * 32 + lane;
    float m_ref = -INFINITY, l_run = 0.f;

    // qk-RMSNorm fused into the load (dit_block.cu:185-196 applies it as a
    // separate pass): warps 0..3 normalise the landed Q tile in place, one
    // row per thread, before the first Q·Kᵀ; the K tiles are done by the
    // V-conversion warps below.
    if (p.qn_w != nullptr && warp < 4 && ntl > 0) {
        wait(kBarQ, 0);
        norm_row_sw128(sQ, row, norm_w, p.norm_eps);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[kBarQn]);
    }

    if (warp == kCtrlWarp) {
        // ── control warp: TMA + MMA issue ───────────────────────────────────
        // All 32 lanes run the loop with identical, warp-uniform state; each
        // TMA / MMA / commit is issued by one elected lane. (Issuing from a
        // single divergent lane cost ~100 cycles per tcgen05.mma, measured.)
        if (ntl > 0) {
            constexpr uint32_t idS  = idesc_f16(128, 128, kFmtQK, 0, 0);  // Q·Kᵀ, both K-major
            constexpr uint32_t idPV = idesc_f16(128, 64, 0, 0, 1);        // P(tmem)·V(MN-major), fp16
            // a static K/V cache is streamed once per use: evict-first in L2
            const uint64_t kvpol = l2_evict_first_policy();
            auto issue_kv = [&](int t) {
                const int s = t % kStages;
                const int key0 = (t_begin + t) * kTileKeys;
                if (elect_one()) {
                    mbar_arrive_expect_tx(&bars[bar_k(s)], kTileBytes);
                    mbar_arrive_expect_tx(&bars[bar_v(s)], kTileBytes);
                    if (p.kv_stream) {
                        tma_load_4d_hint(sK(s), &tmK, &bars[bar_k(s)], 0, key0, hk, b, kvpol);
                        tma_load_4d_hint(sV(s), &tmV, &bars[bar_v(s)], 0, key0, hk, b, kvpol);
                    } else {
                        tma_load_4d(sK(s), &tmK, &bars[bar_k(s)], 0, key0, hk, b);
                        tma_load_4d(sV(s), &tmV, &bars[bar_v(s)], 0, key0, hk, b);
                    }
                }
                __syncwarp();
            };
            const uint32_t aq = smem_u32(sQ);
            auto issue_s = [&](int j) {
                const int u = j % kBufs, s = j % kStages;
                tc_fence_after_sync();
                const uint32_t ak = smem_u32(sK(s));
                if (elect_one()) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_f16_ss(tmem + u * 128, smem_desc_sw128(aq + kk * 32, 16, 1024),
                                   smem_desc_sw128(ak + kk * 32, 16, 1024), idS, kk > 0 ? 1u : 0u);
                    mma_commit(&bars[bar_s(u)]);
                }
                __syncwarp();
            };
            auto issue_pv = [&](int j) {
                const int u = j % kBufs, g = j & 1, s = j % kStages;
                tc_fence_after_sync();
                const uint32_t tP = tmem + u * 128, tO = tmem + 384 + g * 64;
                const uint32_t av = smem_u32(sV(s));
                // fp16 P of keys [32c, 32c+32) sits in columns 32c..32c+15
                if (elect_one()) {
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        mma_f16_ts(tO, tP + 32 * (k >> 1) + 8 * (k & 1),
                                   smem_desc_sw128(av + k * 2048, 8192, 1024), idPV,
                                   (j >= 2 || k > 0) ? 1u : 0u);
                    mma_commit(&bars[bar_o(u)]);
                    mma_commit(&bars[bar_og(g)]);
                }
                __syncwarp();
            };
            if (elect_one()) {
                mbar_arrive_expect_tx(&bars[kBarQ], kTileBytes);
                tma_load_4d(sQ, &tmQ, &bars[kBarQ], 0, q0, h, b);
            }
            __syncwarp();
            SFB_T(150);
            int nL = min(kStages, ntl);                // tiles whose K/V load is issued
            for (int t = 0; t < nL; ++t) issue_kv(t);
            SFB_T(151);
#ifdef SFB_TRACE
            wait(kBarQ, 0);
            SFB_T(152);
            wait(bar_k(0), 0);
            SFB_T(153);
#endif
            wait(p.qn_w ? kBarQn : kBarQ, 0);
            // Event loop. P·V completions are retired in issue order, so every
            // parity probe is at most one phase behind its barrier.
            int nS = 0, nP = 0, pv_done = 0;
            const uint64_t t_start = global_timer_ns();
            uint32_t idle = 0;
#ifdef SFB_TRACE
            long long seen_p = 0, seen_v = 0;
#endif
            long long last_iter = 0;
            while (nP < ntl && ok) {
#ifdef SFB_TRACE
                last_iter = clock64();
#endif
                bool progress = false;
                while (pv_done < nP && mbar_test(&bars[bar_o(pv_done % kBufs)], (pv_done / kBufs) & 1))
                    ++pv_done;
                // stage of tile t is free once P·V of tile t - kStages is done
                while (nL < ntl && nL - kStages < pv_done) { issue_kv(nL); ++nL; progress = true; }
                // S/P buffer of tile j is free once P·V of tile j - kBufs is done
                if (nS < ntl && (nS < kBufs || nS - kBufs < pv_done) &&
                    mbar_test(&bars[p.kn_w ? bar_kn(nS % kStages) : bar_k(nS % kStages)], (nS / kStages) & 1)) {
#ifdef SFB_TRACE
                    const long long ts0 = clock64();
#endif
                    issue_s(nS);
#ifdef SFB_TRACE
                    if (p.trace && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && nS < 40) {
                        p.trace[3400 + 2 * nS] = ts0; p.trace[3401 + 2 * nS] = clock64();
                    }
#endif
                    SFB_T(2 + 4 * nS);
                    ++nS;
                    progress = true;
                }
#ifdef SFB_TRACE
                if (nP < nS) {
                    if (!seen_p && mbar_test(&bars[bar_p(nP % kBufs)], (nP / kBufs) & 1)) seen_p = clock64();
                    if (!seen_v && mbar_test(&bars[conv_v ? bar_vc(nP % kStages) : bar_v(nP % kStages)],
                                             (nP / kStages) & 1)) seen_v = clock64();
                }
#endif
                if (nP < nS && mbar_test(&bars[bar_p(nP % kBufs)], (nP / kBufs) & 1) &&
                    mbar_test(&bars[conv_v ? bar_vc(nP % kStages) : bar_v(nP % kStages)],
                              (nP / kStages) & 1)) {
#ifdef SFB_TRACE
                    const long long tb0 = clock64();
#endif
                    issue_pv(nP);
#ifdef SFB_TRACE
                    const long long tb1 = clock64();
                    if (p.trace && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && nP < 40) {
                        p.trace[3200 + 4 * nP] = seen_p; p.trace[3201 + 4 * nP] = tb0;
                        p.trace[3202 + 4 * nP] = tb1; p.trace[3203 + 4 * nP] = last_iter;
                    }
                    seen_p = seen_v = 0;
#endif
                    SFB_T(3 + 4 * nP);
                    ++nP;
                    progress = true;
                }
                if (progress) { idle = 0; continue; }
                if ((++idle & 1023u) == 1023u) {
                    // lane 0 decides, so the whole warp leaves the loop together
                    const int expired = global_timer_ns() - t_start > 1000000000ull ? 1 : 0;
                    if (__shfl_sync(0xffffffffu, expired, 0)) ok = false;
                }
            }
            if (!ok) {
                // Failure path: the copies and MMAs this warp issued complete
                // before the CTA releases its shared memory and TMEM. Q; K of
                // the tiles whose S was not issued; V of those whose P·V was not
                // (each wait bounded); then one commit covering every MMA.
                mbar_wait(&bars[kBarQ], 0, kDrainNs);
                for (int t = max(nS, nL - kStages); t < nL; ++t)
                    mbar_wait(&bars[bar_k(t % kStages)], (t / kStages) & 1, kDrainNs);
                for (int t = max(nP, nL - kStages); t < nL; ++t)
                    mbar_wait(&bars[bar_v(t % kStages)], (t / kStages) & 1, kDrainNs);
                if (elect_one()) mma_commit(&bars[kBarDrain]);
                __syncwarp();
                mbar_wait(&bars[kBarDrain], 0, kDrainNs);
            }
        }
    } else if ((conv_v || p.kn_w != nullptr) && warp >= kConvWarp0 && warp < kConvWarp0 + kConvWarps) {
        // ── K-norm / V conversion warps: K rows RMS-normalised in place, bf16 V
        //    converted to fp16 in place (same swizzled layouts) ──
        const int ct = (warp - kConvWarp0) * 32 + lane;
        uint32_t bad = 0;
        for (int t = 0; t < ntl; ++t) {
            const int s = t % kStages;
            if (p.kn_w != nullptr) {
                wait(bar_k(s), (t / kStages) & 1);
                for (int r = ct; r < kTileKeys; r += kConvWarps * 32)
                    norm_row_sw128(sK(s), r, norm_w + 64, p.norm_eps);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars[bar_kn(s)]);
            }
            if (!conv_v) continue;
            wait(bar_v(s), (t / kStages) & 1);
            uint4* v4 = reinterpret_cast<uint4*>(sV(s));
#pragma unroll 2
            for (int i = ct; i < kTileBytes / 16; i += kConvWarps * 32) {
                uint4 w = v4[i];
                uint32_t* q = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float lo = __uint_as_float(q[e] << 16), hi = __uint_as_float(q[e] & 0xffff0000u);
                    bad |= (fabsf(lo) > 65504.f) | (fabsf(hi) > 65504.f);
                    q[e] = HalfOps<__half>::pack(lo, hi);
                }
                v4[i] = w;
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[bar_vc(s)]);
        }
        if (__any_sync(0xffffffffu, bad != 0) && lane == 0) atomicExch(&g_sfb_device_error, SFB_ERR_RANGE);
    } else if (warp < kSoftWarps && win < groups) {
        // ── softmax group grp: tiles j ≡ grp (mod 2) ────────────────────────
        const uint32_t lane_off = static_cast<uint32_t>(win * 32) << 16;
        const uint32_t tO = tmem + 384 + grp * 64 + lane_off;
        const int qi = q0 + row;
        const int kend_row = p.causal ? min(kend, qi + 1) : kend;
        const float sl2 = p.sl2;
        const bool use_mask = p.key_mask != nullptr;
        int uses = 0;
        for (int j = grp; j < ntl; j += 2, ++uses) {
            const int key0 = (t_begin + j) * kTileKeys;
            const int u = j % kBufs;
            const uint32_t tS = tmem + u * 128 + lane_off;
            SFB_T(2 + 4 * uses);
            wait(bar_s(u), (j / kBufs) & 1);
            SFB_T(3 + 4 * uses);
            tc_fence_after_sync();
            const bool full = (key0 + kTileKeys <= kend) && !use_mask && !p.causal && !kAMask;
            // pass 1: row max of the raw logits. In a tile with invalid keys
            // (beyond kv_len, masked, or causal) those logits are replaced by
            // -inf in TMEM first, so pass 2 is the same code for every tile.
            float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll 1
            for (int hh = 0; hh < 2; ++hh) {
                float a[32], bb[32];
                tmem_ld32(tS + 64 * hh, a);
                tmem_ld32(tS + 64 * hh + 32, bb);
                tmem_ld_wait();
                if (!full) {
                    const uint32_t va = key_bits(p, b, key0 + 64 * hh, kend_row);
                    const uint32_t vb = key_bits(p, b, key0 + 64 * hh + 32, kend_row);
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        a[i]  = (va >> i) & 1u ? a[i] : -INFINITY;
                        bb[i] = (vb >> i) & 1u ? bb[i] : -INFINITY;
                    }
                    if constexpr (kAMask) {
                        // additive mask: raw logit + m / scale, so that the later
                        // scaling gives scale·q·k + m (masked keys stay -inf)
                        if (qi < p.Lq) {
                            const int64_t mrow = static_cast<int64_t>(b) * p.am_sb + static_cast<int64_t>(qi) * p.am_ss;
                            const int ka = key0 + 64 * hh;
#pragma unroll 4
                            for (int i = 0; i < 32; ++i) {
                                if ((va >> i) & 1u) a[i] = fmaf(attn_mask_at(p.amask, p.am_dt, mrow + ka + i), p.inv_scale, a[i]);
                                if ((vb >> i) & 1u) bb[i] = fmaf(attn_mask_at(p.amask, p.am_dt, mrow + ka + 32 + i), p.inv_scale, bb[i]);
                            }
                        }
                    }
                    tmem_st32(tS + 64 * hh, *reinterpret_cast<uint32_t(*)[32]>(a));
                    tmem_st32(tS + 64 * hh + 32, *reinterpret_cast<uint32_t(*)[32]>(bb));
                }
#pragma unroll
                for (int i = 0; i < 32; ++i) { mx0 = fmaxf(mx0, a[i]); mx1 = fmaxf(mx1, bb[i]); }
            }
            if (!full) tmem_st_wait();
            const float mraw = fmaxf(mx0, mx1);
            const float m_tile = mraw == -INFINITY ? -INFINITY : mraw * sl2;
            if (m_tile > m_ref + 8.f) {          // also true when m_ref == -inf
                if (m_ref != -INFINITY) {
                    const float alpha = ptx::ex2(m_ref - m_tile);
                    l_run *= alpha;
                    // O_grp holds this group's earlier tiles: wait for its last PV
                    wait(bar_og(grp), (uses - 1) & 1);
                    tc_fence_after_sync();
#pragma unroll 1
                    for (int c = 0; c < 2; ++c) {
                        float ot[32];
                        tmem_ld32(tO + 32 * c, ot);
                        tmem_ld_wait();
                        uint32_t ou[32];
#pragma unroll
                        for (int i = 0; i < 32; ++i) ou[i] = __float_as_uint(ot[i] * alpha);
                        tmem_st32(tO + 32 * c, ou);
                    }
                }
                m_ref = m_tile;
            }
            const float m_use = m_ref == -INFINITY ? 0.f : m_ref;
            SFB_T(4 + 4 * uses);
            // pass 2: P = 2^(s·scale·log2e − m) in 32-key chunks; the next chunk's
            // TMEM load is in flight while the current one is computed. The fp16
            // P of chunk c overwrites S columns [32c, 32c+16), already read.
            float lacc0 = 0.f, lacc1 = 0.f;
            auto chunk = [&](const float (&v)[32], int c) {
                uint32_t ph[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float p0 = ptx::ex2(fmaf(v[2 * i], sl2, -m_use));
                    const float p1 = ptx::ex2(fmaf(v[2 * i + 1], sl2, -m_use));
                    lacc0 += p0;
                    lacc1 += p1;
                    ph[i] = HalfOps<__half>::pack(p0, p1);
                }
                tmem_st16(tS + 32 * c, ph);
            };
            float ca[32], cb[32];
            tmem_ld32(tS, ca);
            tmem_ld_wait();
#pragma unroll 1
            for (int c = 0; c < 4; c += 2) {
                tmem_ld32(tS + 32 * (c + 1), cb);
                chunk(ca, c);
                tmem_ld_wait();
                if (c + 2 < 4) tmem_ld32(tS + 32 * (c + 2), ca);
                chunk(cb, c + 1);
                if (c + 2 < 4) tmem_ld_wait();
            }
            l_run += lacc0 + lacc1;
            tmem_st_wait();
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[bar_p(u)]);
            SFB_T(5 + 4 * uses);
        }
        // publish (m, l) of this group for the in-CTA merge
        red[(grp * 2 + 0) * 128 + row] = m_ref;
        red[(grp * 2 + 1) * 128 + row] = l_run;
    }
    SFB_T(160);
    __syncthreads();    // (m, l) of both groups visible
    SFB_T(161);

    // ── merge O_A and O_B: group g's threads take output columns [32g, 32g+32)
    float o_row[32];
    const bool has_rows = warp < kSoftWarps && win < groups && row < rows;
    if (warp < kSoftWarps && win < groups) {
        const uint32_t lane_off = static_cast<uint32_t>(win * 32) << 16;
        const float mA = red[0 * 128 + row], lA = red[1 * 128 + row];
        const float mB = red[2 * 128 + row], lB = red[3 * 128 + row];
        const float M  = fmaxf(mA, mB);
        const float wA = (mA == -INFINITY) ? 0.f : ptx::ex2(mA - M);
        const float wB = (mB == -INFINITY) ? 0.f : ptx::ex2(mB - M);
        // wait for the last PV of each group that had tiles
        if (ntl >= 1) wait(bar_og(0), ((ntl + 1) / 2 - 1) & 1);
        if (ntl >= 2) wait(bar_og(1), (ntl / 2 - 1) & 1);
        tc_fence_after_sync();
        float a[32], bb[32];
        tmem_ld32(tmem + 384 + lane_off + 32 * grp, a);
        tmem_ld32(tmem + 448 + lane_off + 32 * grp, bb);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i)
            o_row[i] = (wA != 0.f ? wA * a[i] : 0.f) + (wB != 0.f ? wB * bb[i] : 0.f);
        m_ref = M;
        l_run = wA * lA + wB * lB;
    }
    SFB_T(162);

    // ── epilogue ────────────────────────────────────────────────────────────
    T* out = static_cast<T*>(p.out);
    const int64_t row_base = static_cast<int64_t>(b) * p.o_sb + static_cast<int64_t>(h) * p.o_sh;
    if (p.splits == 1) {
        if (has_rows && ok) {
            const float inv = (l_run > 0.f && m_ref != -INFINITY) ? 1.f / l_run : 0.f;
            T* dst = out + row_base + static_cast<int64_t>(q0 + row) * p.o_ss + 32 * grp;
#pragma unroll
            for (int c = 0; c < 32; c += 8) {
                uint4 u;
                u.x = HO::pack(o_row[c + 0] * inv, o_row[c + 1] * inv);
                u.y = HO::pack(o_row[c + 2] * inv, o_row[c + 3] * inv);
                u.z = HO::pack(o_row[c + 4] * inv, o_row[c + 5] * inv);
                u.w = HO::pack(o_row[c + 6] * inv, o_row[c + 7] * inv);
                *reinterpret_cast<uint4*>(dst + c) = u;
            }
        }
    } else {
        // Row r is owned by CTA r % C at slot r / C of source block `split`. The
        // merge buffer is dedicated (never a TMA target), so partials are pushed
        // as soon as they are ready; one cluster barrier publishes them.
        const int C = p.splits;
        const int slots = (rows + C - 1) / C;
        float* sO = reinterpret_cast<float*>(smem + kOffMerge);        // [C][slots][2][kOStride]
        float* sM = sO + C * slots * 2 * kOStride;                     // [C][slots]
        float* sL = sM + C * slots;                                    // [C][slots]
        cluster_wait();                  // every peer has started (arrived after its setup)
        if (has_rows) {
            const int owner = row % C, slot = row / C;
            const uint32_t dO = dsmem_map(smem_u32(sO + ((split * slots + slot) * 2 + grp) * kOStride), owner);
#pragma unroll
            for (int c = 0; c < 32; c += 4)
                dsmem_st_f32x4(dO + c * 4, make_float4(o_row[c], o_row[c + 1], o_row[c + 2], o_row[c + 3]));
            if (grp == 0) {
                dsmem_st_f32(dsmem_map(smem_u32(sM + split * slots + slot), owner), m_ref);
                dsmem_st_f32(dsmem_map(smem_u32(sL + split * slots + slot), owner), l_run);
            }
        }
        SFB_T(163);
        cluster_sync();
        SFB_T(164);
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
                    const float mk = sM[k * slots + slot];
                    if (mk == -INFINITY) continue;
                    const float w = ptx::ex2(mk - M);
                    L += w * sL[k * slots + slot];
                    const float4 o = *reinterpret_cast<const float4*>(
                        sO + ((k * slots + slot) * 2 + (c4 >> 5)) * kOStride + (c4 & 31));
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

    SFB_T(165);
#ifdef SFB_TRACE
    if (p.trace && tid == 0) {
        const int cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
        if (cta < 1024) {
            p.trace[1024 + 2 * cta] = cta_t0;
            p.trace[1025 + 2 * cta] = ptx::global_timer_ns();
        }
    }
#endif
    if (!ok) atomicExch(&g_sfb_device_error, SFB_ERR_DEVICE_TIMEOUT);
    tc_fence_before_sync();
    __syncthreads();
#ifdef SFB_TRACE
    tl_record(p.tl, p.tl_launch, 3, cta_t0, tl_t1);
#endif
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
extern "C" void sfb_debug_set_timeline(void* p) { tl_buf() = static_cast<unsigned long long*>(p); tl_count() = 0; }
static int g_attn_skip = 0;
static int g_attn_trace_launch = -1;
extern "C" void sfb_debug_set_attn_trace_launch(int i) { g_attn_trace_launch = i; }
extern "C" void sfb_debug_set_attn_skip(int s) { g_attn_skip = s; }
#endif

// Cluster size along Lk: as many splits as keep every CTA co-resident in one
// wave (one CTA per SM), at least two key tiles per split.
int choose_attn_splits(int units, int ntiles_max, int num_sms) {
    int s = std::max(1, num_sms / std::max(units, 1));
    s = std::min(s, 16);
    s = std::min(s, std::max(1, ntiles_max / 2));
    return s;
}

int attention_tc_launch(const sfb_attn_args& a, cudaStream_t stream, const AttnOpts& o) {
    const bool pdl = o.pdl, v_f16 = o.v_f16;
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
    if (v_f16 && a.dtype != SFB_BF16) return SFB_ERR_DTYPE;
    if ((rc = make_map_4d(&mv, a.v, v_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : dt, 64, a.seq_k, a.heads_kv, a.batch, a.v_stride[2], a.v_stride[1],
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
    p.v_f16 = v_f16 ? 1 : 0;
    p.qn_w = static_cast<const __nv_bfloat16*>(o.qn_w);
    p.kn_w = static_cast<const __nv_bfloat16*>(o.kn_w);
    p.norm_eps = o.norm_eps;
    p.kv_stream = o.v_f16 ? 1 : 0;   // the model's cross-attention cache
    p.amask = a.attn_mask;
    p.am_dt = a.attn_mask_dtype;
    p.am_sb = a.attn_mask_stride[0];
    p.am_ss = a.attn_mask_stride[1];
    p.inv_scale = 1.f / scale;
    if ((o.qn_w || o.kn_w) && (a.dtype != SFB_BF16 || a.head_dim != 64)) return SFB_ERR_DTYPE;
#ifdef SFB_TRACE
    p.tl = tl_buf();
    p.tl_launch = tl_next();
    p.trace = (g_attn_trace_launch < 0 || g_attn_trace_launch == p.tl_launch) ? g_trace_ptr : nullptr;
    p.dbg_skip = g_attn_skip;
#endif
    const int units = a.batch * a.heads * p.qtiles;
    const int ntiles_max = (a.seq_k + 127) / 128;
    p.splits = a.num_splits > 0 ? std::min(a.num_splits, 16)
                                : choose_attn_splits(units, ntiles_max, dev.num_sms);
    if (p.splits > std::max(1, ntiles_max)) p.splits = std::max(1, ntiles_max);
    if ((p.o_ss % 8) != 0 && p.splits == 1) return SFB_ERR_ALIGN;

    const bool am = a.attn_mask != nullptr;
    auto kern = a.dtype == SFB_BF16 ? (am ? attn_tc::attn_fwd_tc_kernel<__nv_bfloat16, true>
                                          : attn_tc::attn_fwd_tc_kernel<__nv_bfloat16, false>)
                                    : (am ? attn_tc::attn_fwd_tc_kernel<__half, true>
                                          : attn_tc::attn_fwd_tc_kernel<__half, false>);
    // kernel attributes, set once per variant and device (idempotent: a race only repeats them)
    static std::atomic<bool> attr_done[4][64];
    const int ki = (a.dtype == SFB_BF16 ? 0 : 1) + (am ? 2 : 0);
    if (!attr_done[ki][dev.ordinal & 63].load(std::memory_order_acquire)) {
        cudaError_t e1 = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              attn_tc::kSmemBytes);
        cudaError_t e2 = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e1 != cudaSuccess || e2 != cudaSuccess) {
            (void)cudaGetLastError();
            record_cuda_error(e1 != cudaSuccess ? e1 : e2, "attention kernel attributes");
            return SFB_ERR_CUDA;
        }
        attr_done[ki][dev.ordinal & 63].store(true, std::memory_order_release);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim  = dim3(p.splits, a.heads, a.batch * p.qtiles);
    cfg.blockDim = dim3(attn_tc::kThreads, 1, 1);
    cfg.dynamicSmemBytes = attn_tc::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = p.splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1 + pdl_attr(&attr[1], pdl);
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mq, mk, mv, p);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        record_cuda_error(e, "attention (tcgen05) launch");
        return SFB_ERR_LAUNCH;
    }
    return SFB_OK;
}

}  // namespace sfb
