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
// Work of a projection stage: output tiles of 64 weight rows; a 4-CTA
// thread-block cluster takes a tile and splits K four ways; clusters walk the
// tiles round-robin. Per CTA (11 warps):
//   warp 0      pulls every weight box of the launch into L2 at start, then
//               streams its int8 tiles [64 × 64] through an 8-slot ring,
//               running ahead across stages (weights depend on nothing);
//   warps 3..6  convert int8 → bf16 (exact) into an 8-slot SW128 ring, up to
//               a whole unit ahead of the MMAs;
//   warp 1      issues tcgen05.mma (M = 64 weight rows, N = 80 tokens, K = 16)
//               into one of two TMEM accumulators;
//   warp 2      waits for the previous stage's counter (acquire, bounded),
//               then loads the CTA's activation slice [80 × K/4] by TMA;
//   warps 7..10 run the epilogue.
// Split-K partials go from TMEM straight into the owning CTA's shared memory
// (st.async, counted by the owner's mbarrier transaction count; the owner of
// a channel row is the cluster rank that equals its TMEM lane window); owners
// sum the four partials, apply the epilogue and store coalesced 16-byte rows.
// Every CTA then bumps the stage's completion counter (release). No global
// scratch beyond the counters and the stage table.
//
// Attention stages run on the same warps: self-attention over the session's
// tokens (one head per CTA) and cross-attention against a per-tick K/V cache
// (one head per cluster, key tiles split over its four CTAs, partial rows
// merged in their owners' shared memory).
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
    CUtensorMap tmW;                 // int8 [N, K], box {64, TM}, no swizzle (cross-attention: K/V cache)
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
    const __nv_bfloat16* qn_w;       // self-attention stages: per-head RMSNorm weights [64] of Q
    const __nv_bfloat16* kn_w;       // and of K
    const int32_t* kv_len;           // cross-attention: valid keys (device, [1]) or null
    int32_t lk;                      // cross-attention: keys in the cache
    int64_t ldr, ldy, ldg;
    int32_t n_ss_in;
    int32_t N, K, TM, tiles, act, y_f32;
    int32_t kind;                    // kDenseGemm, kDenseSelfAttn or kDenseCrossAttn
    float eps;
    float sm_scale;                  // self-attention: softmax scale
};
constexpr int kDenseGemm = 0;
// Self-attention over the stage's token rows (M <= 80 queries and keys), one
// head per CTA: tmX maps the fused qkv activations [M, 3·N] with a 128-row box;
// y receives [M, N]; tiles = heads = N / 64.
constexpr int kDenseSelfAttn = 1;
// Cross-attention of the stage's query rows (M <= 80; Q = y-side input at
// tmX, [M, N], q-normed here) against a per-tick K (bf16, normed) / V (fp16)
// cache of lk keys (tmW: K in columns [0, N), V in [N, 2N)), first kv_len keys valid: one head per cluster,
// its key tiles split over the cluster's four CTAs, the partial (O, m, l) rows
// merged in their owners' shared memory. tiles = heads = N / 64.
constexpr int kDenseCrossAttn = 2;

// The scalar part of a stage, copied into shared memory at kernel start: the
// kernel's waits are asm statements that clobber memory, so every field read
// from the stage table itself would be re-read from global memory after each
// of them (and the acquire of a stage counter invalidates the L1).
struct StageInfo {
    const CUtensorMap* tmW;
    const CUtensorMap* tmX;
    const float* w_scale;
    const __nv_bfloat16* bias;
    const void* residual;
    void* y;
    const __nv_bfloat16* g_next;
    __nv_bfloat16* xg;
    float* ss_out;
    const float* ss_in;
    const uint8_t* l2_prefetch;
    uint64_t l2_bytes;
    const __nv_bfloat16* qn_w;
    const __nv_bfloat16* kn_w;
    const int32_t* kv_len;
    int64_t ldr, ldy, ldg;
    int32_t n_ss_in, N, K, TM, tiles, act, y_f32, kind, lk;
    float eps, sm_scale;
};
__device__ __forceinline__ StageInfo stage_info(const DenseStage& S) {
    StageInfo i;
    i.tmW = &S.tmW; i.tmX = &S.tmX;
    i.w_scale = S.w_scale; i.bias = S.bias; i.residual = S.residual; i.y = S.y; i.g_next = S.g_next;
    i.xg = S.xg; i.ss_out = S.ss_out; i.ss_in = S.ss_in; i.l2_prefetch = S.l2_prefetch; i.l2_bytes = S.l2_bytes;
    i.qn_w = S.qn_w; i.kn_w = S.kn_w; i.kv_len = S.kv_len; i.lk = S.lk;
    i.ldr = S.ldr; i.ldy = S.ldy; i.ldg = S.ldg;
    i.n_ss_in = S.n_ss_in; i.N = S.N; i.K = S.K; i.TM = S.TM; i.tiles = S.tiles; i.act = S.act; i.y_f32 = S.y_f32;
    i.kind = S.kind; i.eps = S.eps; i.sm_scale = S.sm_scale;
    return i;
}

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
constexpr int kTM = 64;                       // weight rows per output tile (MMA M)
constexpr int kNW = 8;                        // int8 weight ring slots (kTM × 64 B)
constexpr int kNB = 8;                        // converted bf16 weight slots (SW128, kTM × 128 B)
constexpr int kNX = 8;                        // activation chunks per CTA (K / 4 / 64 <= 8)
constexpr int kXBytes = kBN * 128;            // one activation chunk [80 × 64] bf16, SW128
constexpr int kXRows = kBN;                   // rows of an activation box (>= M)
constexpr uint32_t kXBoxBytes = kXRows * 128;
constexpr int kWBytes = kTM * 64;             // int8 slot
constexpr int kWBBytes = kTM * 128;           // bf16 slot
constexpr int kOffX = 0;
constexpr int kOffWB = kOffX + kNX * kXBytes;                 // 81920
constexpr int kOffW = kOffWB + kNB * kWBBytes;                // 147456
constexpr int kOffRcv = kOffW + kNW * kWBytes;                // 180224
constexpr int kRcvBytes = 24576;                              // [4 sources][16 rows][80] fp32; cross-attention rows
static_assert(kRcvBytes >= kSplit * (kTM / 4) * kBN * 4 && kRcvBytes >= kSplit * 20 * 68 * 4, "receive area");
constexpr int kOffRinv = kOffRcv + kRcvBytes;
constexpr int kOffRed = kOffRinv + kBN * 4;                   // [6 groups][80] partial row sums
constexpr int kOffSSt = kOffRed + 6 * kBN * 4;                 // [80] this CTA's quarter of the row sums
constexpr int kOffSSx = kOffSSt + kBN * 4;                    // [4 ranks][80] the cluster's quarters
constexpr int kOffBar = kOffSSx + kSplit * kBN * 4;
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
constexpr int kBarQK = kBarDrain + 1;                         // self-attention: Q, K normalised, V in fp16
constexpr int kBarS = kBarQK + 1;                             // S = Q·Kᵀ in TMEM
constexpr int kBarP = kBarS + 1;                              // P written to TMEM
constexpr int kBarO = kBarP + 1;                              // O = P·V in TMEM
constexpr int kBarKV = kBarO + 1;                             // cross-attention: [K0, V0, K1, V1] landed
constexpr int kBarKVFree = kBarKV + 4;                        // [2]: the stage's P·V is done
constexpr int kBarARcv = kBarKVFree + 2;                      // cross-attention: the sources' partial rows
constexpr int kBarCQ = kBarARcv + 1;                          // cross-attention: Q normalised
constexpr int kBarCS = kBarCQ + 1;                            // [2]: S of TMEM buffer b
constexpr int kBarCP = kBarCS + 2;                            // P written
constexpr int kBarCO = kBarCP + 1;                            // O += P·V done
constexpr int kBarDrain2 = kBarCO + 1;                        // the activation warp's MMAs after a failure
constexpr int kBarSS = kBarDrain2 + 1;                        // the cluster's RMS quarter sums landed
constexpr int kNumBars = kBarSS + 1;
// TMEM columns: projection accumulators [0, 256); self-attention S [256, 336),
// P (fp16 pairs) [336, 384), O [384, 448); cross-attention S buffers at 0
// and 128 (the accumulators' columns: no projection runs in that stage), P
// buffers at 256 and 320, O at 384
// shared memory of a cross-attention stage (the activation area): Q [128 × 64]
// at 0, then two K/V stages of [128 keys × 64] K (bf16) and V (fp16)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 256, kColP = 336, kColO = 384;
constexpr uint32_t kColCrossP = 256;
// A projection unit's MMAs are issued by kIssuers warps (the MMA warp and the
// activation warp, which is idle once its loads are out): warp w takes the
// K chunks c with c % kIssuers == w into its own TMEM accumulator (chain w).
// One thread's tcgen05.mma issue takes ~165 cycles whatever the shape, so a
// unit's 32 small MMAs (64 × 80 × 16) from one warp cost ~2.9 µs; issue from
// several warps overlaps. The epilogue adds the chains. Unit buffer b's chain
// w sits at TMEM column b · kAccBufCols + w · kBN.
constexpr int kIssuers = 2;
constexpr uint32_t kAccBufCols = 256;
static_assert(kIssuers * 80 <= static_cast<int>(kAccBufCols) && 2 * kAccBufCols <= 512, "accumulator columns");                          // cross-attention P buffers [256, 384)
constexpr int kQKVBytes = 128 * 128;                          // one [128 × 64] bf16 tile, SW128
constexpr int kOffKV = kOffX + kQKVBytes;                     // stage st: K at + st · 2 tiles, V after it
static_assert(kOffKV + 4 * kQKVBytes <= kOffWB, "cross-attention tiles fit the activation area");
constexpr int kOffTmem = kOffBar + 8 * kNumBars;
constexpr int kOffGen = kOffTmem + 8;
constexpr int kMaxStages = 48;                                // stages of one launch
constexpr int kOffInfo = (kOffGen + 8 + 15) & ~15;
constexpr int kSmemUsed = kOffInfo + kMaxStages * static_cast<int>(sizeof(StageInfo));
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
// Waits of the kernel: blocking try_wait with the kernel's limit. (Polling
// test_wait in any of the roles measured no faster.)
__device__ __forceinline__ bool cwait(uint64_t* bar, uint32_t parity, uint64_t ns) {
    return mbar_wait_cluster(bar, parity, ns);
}

// Pulls one box of a tensor map into L2 (no shared memory, no completion).
__device__ __forceinline__ void prefetch_l2_tile(const CUtensorMap* map, int32_t c0, int32_t c1) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1) : "memory");
}
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(p)), "r"(bytes)
                 : "memory");
}
// 16-byte global loads issued where they are written (volatile asm: the
// compiler neither sinks them to their first use nor merges them with later
// ones). ld_cg_*: data written earlier in this launch by other CTAs (the
// residual stream, the RMS partials), read at L2 (.cg: never a stale L1 line;
// the writers' stage completion has been acquired). ld_nc_*: constants
// (weights' scales, biases, norm weights) through the non-coherent path.
__device__ __forceinline__ float4 ld_cg_f4(const float* p) {
    float4 v;
    asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ld_cg_u4(const void* p) {
    uint4 v;
    asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ int32_t ld_nc_i32(const int32_t* p) {
    int32_t v;
    asm volatile("ld.global.nc.b32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ld_nc_u4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
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

// The CTA's share of a projection stage: tiles t = cluster, cluster + nclusters, ...
__device__ __forceinline__ int units_of(const StageInfo& S, int cl, int ncl) {
    if (S.kind != kDenseGemm) return 0;
    return cl < S.tiles ? (S.tiles - cl + ncl - 1) / ncl : 0;
}
// Whether this CTA works in a stage at all (a self-attention stage: head = CTA index).
__device__ __forceinline__ bool works_in(const StageInfo& S, int cl, int ncl) {
    if (S.kind == kDenseGemm) return units_of(S, cl, ncl) > 0;
    if (S.kind == kDenseCrossAttn) return cl < S.tiles;
    return static_cast<int>(blockIdx.x) < S.tiles;
}

// A cross-attention CTA's key tiles [t0, t0 + n) of 128 keys: this cluster
// rank's contiguous share of the valid keys (kv_len, read after the stage's
// dependency).
struct KeyRange { int t0, n, kend; };
__device__ __forceinline__ KeyRange key_range(const StageInfo& S, int rank) {
    int kend = S.lk;
    if (S.kv_len != nullptr) kend = min(kend, max(0, ld_nc_i32(S.kv_len)));
    const int nt = (kend + 127) / 128;
    const int base = nt / kSplit, rem = nt - base * kSplit;
    return {rank * base + min(rank, rem), base + (rank < rem ? 1 : 0), kend};
}

// The kernel body: `stages` in global memory (a model's stage table) or in
// the parameter space of a launch (dense_pair_kernel).
// The epilogue warps' part of a self-attention stage (warps 7..10, thread =
// query row = TMEM lane): wait for Q/K/V, RMS-normalise the Q and K rows in
// place (the qk-norm of dit_block.cu:185-196, same arithmetic and summation
// order as the attention kernel's), convert V to fp16 in place (exact for
// |v| <= 65504, else SFB_ERR_RANGE), then the softmax of S = Q·Kᵀ into fp16 P
// in TMEM, and finally out = O / l for this CTA's head.
__device__ __forceinline__ void self_attention_epilogue(const StageInfo& S, uint8_t* smem, uint64_t* bars,
                                                        uint32_t tmem, uint32_t xs, uint32_t xmask, uint32_t aq,
                                                        uint32_t ap, int M, bool& ok) {
    using namespace ptx;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int et = threadIdx.x - kWarpEpi0 * 32, q = warp & 3;
    auto wait = [&](int b, uint32_t parity) {
        if (!mbar_wait(&bars[b], parity, ok ? kWaitNs : 0ull)) ok = false;
    };
    uint8_t* sQ = smem + kOffX;
    uint8_t* sK = sQ + kQKVBytes;
    uint8_t* sV = sK + kQKVBytes;
    wait(kBarDep, xs & 1);
    for (int t = 0; t < 3; ++t) wait(kBarXFull + t, (xmask >> t) & 1u);
    for (int r = et; r < 2 * M; r += kEpiThreads) {
        if (r < M) attn_tc::norm_row_sw128(sQ, r, S.qn_w, S.eps);
        else attn_tc::norm_row_sw128(sK, r - M, S.kn_w, S.eps);
    }
    uint32_t bad = 0;
    uint4* v4 = reinterpret_cast<uint4*>(sV);
    for (int i = et; i < kBN * 8; i += kEpiThreads) {     // rows 0..79, 8 × 16 bytes each
        uint4 w = v4[i];
        uint32_t* u = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float lo = __uint_as_float(u[e] << 16), hi = __uint_as_float(u[e] & 0xffff0000u);
            bad |= (fabsf(lo) > 65504.f) | (fabsf(hi) > 65504.f);
            const __half2 hv = __floats2half2_rn(lo, hi);
            u[e] = *reinterpret_cast<const uint32_t*>(&hv);
        }
        v4[i] = w;
    }
    if (__any_sync(0xffffffffu, bad != 0) && lane == 0) atomicExch(&g_sfb_device_error, SFB_ERR_RANGE);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars[kBarQK]);
    // softmax over the M valid keys of this row
    wait(kBarS, ap & 1);
    tc_fence_after_sync();
    const uint32_t tq = tmem + (static_cast<uint32_t>(q * 32) << 16);
    float sv[kBN];
    tmem_ld32(tq + kColS, *reinterpret_cast<float(*)[32]>(sv));
    tmem_ld32(tq + kColS + 32, *reinterpret_cast<float(*)[32]>(sv + 32));
    {
        float tail[32];
        tmem_ld32(tq + kColS + 64, tail);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < kBN - 64; ++i) sv[64 + i] = tail[i];
    }
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < kBN; ++j) if (j < M) mx = fmaxf(mx, sv[j]);
    const float sl2 = S.sm_scale * 1.4426950408889634f;
    const float moff = mx * sl2;
    float l = 0.f;
    uint32_t pu[48];
#pragma unroll
    for (int i = 0; i < 48; ++i) {
        float p0 = 0.f, p1 = 0.f;
        if (2 * i < M && 2 * i < kBN) p0 = ex2(fmaf(sv[2 * i], sl2, -moff));
        if (2 * i + 1 < M && 2 * i + 1 < kBN) p1 = ex2(fmaf(sv[2 * i + 1], sl2, -moff));
        l += p0 + p1;
        const __half2 h2 = __floats2half2_rn(p0, p1);
        pu[i] = *reinterpret_cast<const uint32_t*>(&h2);
    }
    tmem_st32(tq + kColP, *reinterpret_cast<uint32_t(*)[32]>(pu));
    tmem_st16(tq + kColP + 32, *reinterpret_cast<uint32_t(*)[16]>(pu + 32));
    tmem_st_wait();
    tc_fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars[kBarP]);
    // out = O / l, this head's 64 columns of row r
    wait(kBarO, ap & 1);
    tc_fence_after_sync();
    float o[64];
    tmem_ld32(tq + kColO, *reinterpret_cast<float(*)[32]>(o));
    tmem_ld32(tq + kColO + 32, *reinterpret_cast<float(*)[32]>(o + 32));
    tmem_ld_wait();
    const int r = q * 32 + lane;
    if (r < M && ok) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(S.y) + r * S.ldy + static_cast<int64_t>(blockIdx.x) * 64;
#pragma unroll
        for (int c = 0; c < 64; c += 8) {
            uint4 w;
            __nv_bfloat162* w2 = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
            for (int k = 0; k < 4; ++k) w2[k] = __floats2bfloat162_rn(o[c + 2 * k] * inv, o[c + 2 * k + 1] * inv);
            *reinterpret_cast<uint4*>(dst + c) = w;
        }
    }
    tc_fence_before_sync();
}

// The epilogue warps' part of a cross-attention stage (thread = query row =
// TMEM lane): normalise the Q rows (q-norm), then per key tile the softmax of
// S = Q·Kᵀ into fp16 P in TMEM with a lazily rescaled running maximum (O is
// rescaled only when a tile raises the maximum by more than 2^8), and finally
// this split's (O, m, l) rows go to their owner CTAs, which merge the four
// splits and write out = O / l. `ct` (this CTA's count of cross-attention
// key tiles) advances by the tiles done; `cq` counts cross-attention stages.
__device__ __forceinline__ void cross_attention_epilogue(const StageInfo& S, uint8_t* smem, uint64_t* bars,
                                                         uint32_t tmem, float* rcv, uint32_t xs, uint32_t xmask,
                                                         uint32_t cq, uint32_t& ct, int M, int rank, bool& ok) {
    using namespace ptx;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int et = threadIdx.x - kWarpEpi0 * 32, q = warp & 3;
    auto wait = [&](int b, uint32_t parity) {
        if (!mbar_wait(&bars[b], parity, ok ? kWaitNs : 0ull)) ok = false;
    };
    constexpr int kOwnRows = (kBN + kSplit - 1) / kSplit;         // 20: rows per owner CTA
    constexpr int kRowF = 68;                                     // floats per sent row: O[64], m, l, pad
    uint8_t* sQ = smem + kOffX;
    wait(kBarDep, xs & 1);
    const KeyRange kr = key_range(S, rank);
    const int own0 = rank * kOwnRows, own_n = max(0, min(kOwnRows, M - own0));
    if (et == 0) mbar_arrive_expect_tx(&bars[kBarARcv], static_cast<uint32_t>(kSplit * own_n * kRowF * 4));
    wait(kBarXFull + 0, xmask & 1u);
    if (et < M) attn_tc::norm_row_sw128(sQ, et, S.qn_w, S.eps);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars[kBarCQ]);
    const uint32_t tq = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const float sl2 = S.sm_scale * 1.4426950408889634f;
    float m_ref = -INFINITY, l_run = 0.f;
    for (int i = 0; i < kr.n; ++i, ++ct) {
        const int key0 = (kr.t0 + i) * 128;
        const uint32_t tS = tq + (ct & 1u) * 128;          // this tile's S / P buffer
        wait(kBarCS + (ct & 1), (ct >> 1) & 1);
        tc_fence_after_sync();
        const bool full = key0 + 128 <= kr.kend;
        // One pass over S: p = 2^(s·scale·log2e − m_use) as fp16 pairs into the
        // tile's P buffer (TMEM columns 256 + 64·(tile & 1), apart from S, so that
        // a pass can be redone), the tile's row maximum (log2 units) and row sum.
        const uint32_t tP = tq + kColCrossP + (ct & 1u) * 64;
        auto exp_pass = [&](float m_use, float& mx, float& lsum) {
            mx = -INFINITY;
            lsum = 0.f;
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                float v[32];
                tmem_ld32(tS + 32 * c, v);
                tmem_ld_wait();
                uint32_t pk[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int k0 = key0 + 32 * c + 2 * j;
                    const bool v0 = full || k0 < kr.kend, v1 = full || k0 + 1 < kr.kend;
                    const float s0 = v[2 * j] * sl2, s1 = v[2 * j + 1] * sl2;
                    mx = fmaxf(mx, fmaxf(v0 ? s0 : -INFINITY, v1 ? s1 : -INFINITY));
                    const float p0 = v0 ? ex2(s0 - m_use) : 0.f;
                    const float p1 = v1 ? ex2(s1 - m_use) : 0.f;
                    lsum += p0 + p1;
                    const __half2 h2 = __floats2half2_rn(p0, p1);
                    pk[j] = *reinterpret_cast<const uint32_t*>(&h2);
                }
                tmem_st16(tP + 16 * c, pk);
            }
        };
        float mx = -INFINITY, lsum = 0.f;
        // after the first tile every row has a finite reference maximum: one pass,
        // redone (rarely) for a warp in which a row's maximum rose by more than 2^8
        if (i > 0) exp_pass(m_ref, mx, lsum);
        const bool raise = i == 0 || mx > m_ref + 8.f;
        if (__any_sync(0xffffffffu, raise)) {
            if (i == 0) {
                // the first tile: its row maximum first
#pragma unroll 1
                for (int c = 0; c < 4; ++c) {
                    float v[32];
                    tmem_ld32(tS + 32 * c, v);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (full || key0 + 32 * c + j < kr.kend) mx = fmaxf(mx, v[j] * sl2);
                }
            }
            const float m_new = raise ? mx : m_ref;
            const float alpha = (raise && m_ref != -INFINITY) ? ex2(m_ref - m_new) : 1.f;
            if (__any_sync(0xffffffffu, alpha != 1.f)) {
                // rescale O (warp-wide TMEM accesses; factor 1 for the other rows)
                wait(kBarCO, (ct - 1) & 1);            // the previous tile's P·V is in O
                tc_fence_after_sync();
#pragma unroll 1
                for (int c = 0; c < 2; ++c) {
                    float o[32];
                    tmem_ld32(tq + kColO + 32 * c, o);
                    tmem_ld_wait();
                    uint32_t ou[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) ou[j] = __float_as_uint(o[j] * alpha);
                    tmem_st32(tq + kColO + 32 * c, ou);
                }
                tmem_st_wait();
            }
            l_run *= alpha;
            m_ref = m_new;
            float mx2;
            exp_pass(m_ref == -INFINITY ? 0.f : m_ref, mx2, lsum);
        }
        l_run += lsum;
        tmem_st_wait();
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[kBarCP]);
    }
    // this split's rows to their owners: O (64), m (log2 units), l
    float o[64];
    if (kr.n > 0) {
        wait(kBarCO, (ct - 1) & 1);
        tc_fence_after_sync();
        tmem_ld32(tq + kColO, *reinterpret_cast<float(*)[32]>(o));
        tmem_ld32(tq + kColO + 32, *reinterpret_cast<float(*)[32]>(o + 32));
        tmem_ld_wait();
    } else {
#pragma unroll
        for (int j = 0; j < 64; ++j) o[j] = 0.f;
    }
    tc_fence_before_sync();
    const int row = q * 32 + lane;
    if (row < M) {
        const int owner = row / kOwnRows, slot = row - owner * kOwnRows;
        const uint32_t dst = dsmem_map(smem_u32(rcv + (rank * kOwnRows + slot) * kRowF), static_cast<uint32_t>(owner));
        const uint32_t rbar = dsmem_map(smem_u32(&bars[kBarARcv]), static_cast<uint32_t>(owner));
#pragma unroll
        for (int c = 0; c < 64; c += 4) st_async_v4(dst + c * 4, make_float4(o[c], o[c + 1], o[c + 2], o[c + 3]), rbar);
        st_async_v4(dst + 64 * 4, make_float4(m_ref, l_run, 0.f, 0.f), rbar);
    }
    // owner: merge the four splits of its rows
    if (!cwait(&bars[kBarARcv], cq & 1, ok ? kWaitNs : 0ull)) ok = false;
    const int h = static_cast<int>(blockIdx.x) / kSplit;
    for (int w = et; w < own_n * 16; w += kEpiThreads) {
        const int slot = w / 16, c4 = (w - slot * 16) * 4;
        float mk[kSplit], Mx = -INFINITY;
#pragma unroll
        for (int k = 0; k < kSplit; ++k) {
            mk[k] = rcv[(k * kOwnRows + slot) * kRowF + 64];
            Mx = fmaxf(Mx, mk[k]);
        }
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        float L = 0.f;
        if (Mx != -INFINITY) {
#pragma unroll
            for (int k = 0; k < kSplit; ++k) {
                if (mk[k] == -INFINITY) continue;
                const float wk = ex2(mk[k] - Mx);
                const float* src = rcv + (k * kOwnRows + slot) * kRowF;
                L += wk * src[65];
                acc.x += wk * src[c4]; acc.y += wk * src[c4 + 1]; acc.z += wk * src[c4 + 2]; acc.w += wk * src[c4 + 3];
            }
        }
        const float inv = L > 0.f ? 1.f / L : 0.f;
        if (ok) {
            __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(S.y) + (own0 + slot) * S.ldy + h * 64 + c4;
            __nv_bfloat162 a = __floats2bfloat162_rn(acc.x * inv, acc.y * inv);
            __nv_bfloat162 b = __floats2bfloat162_rn(acc.z * inv, acc.w * inv);
            uint2 u;
            u.x = *reinterpret_cast<uint32_t*>(&a);
            u.y = *reinterpret_cast<uint32_t*>(&b);
            *reinterpret_cast<uint2*>(dst) = u;
        }
    }
}

#ifdef SFB_TRACE
// per launch slot: [CTA < 160][stage < 16, then 16 = setup][8] global-timer stamps
constexpr int kTrStages = kMaxStages + 1;                     // + the launch slot
#define DN_T(st, k) do { if (trace != nullptr && blockIdx.x < 160 && (st) < kTrStages) \
        trace[(blockIdx.x * kTrStages + (st)) * 40 + (k)] = ptx::global_timer_ns(); } while (0)
#define DN_C(st, k) do { if (trace != nullptr && blockIdx.x < 160 && (st) < kTrStages) \
        trace[(blockIdx.x * kTrStages + (st)) * 40 + (k)] = clock64(); } while (0)
#else
#define DN_T(st, k) do { } while (0)
#define DN_C(st, k) do { } while (0)
#endif

__device__ __forceinline__ void dense_run(const DenseStage* __restrict__ stages, int nst,
                                          unsigned long long* __restrict__ ctr, int M
#ifdef SFB_TRACE
                                          , unsigned long long* trace
#endif
                                          ) {
    using namespace ptx;
    if (threadIdx.x == 0) DN_T(kMaxStages, 0);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kOffTmem);
    uint64_t* gen_slot = reinterpret_cast<uint64_t*>(smem + kOffGen);
    float* rcv = reinterpret_cast<float*>(smem + kOffRcv);
    float* rinv = reinterpret_cast<float*>(smem + kOffRinv);
    float* red = reinterpret_cast<float*>(smem + kOffRed);
    float* sst = reinterpret_cast<float*>(smem + kOffSSt);
    float* ssx = reinterpret_cast<float*>(smem + kOffSSx);
    StageInfo* sinfo = reinterpret_cast<StageInfo*>(smem + kOffInfo);
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
        for (int i = 0; i < 2; ++i) { mbar_init(&bars[kBarAccFull + i], kIssuers); mbar_init(&bars[kBarAccFree + i], 4); }
        mbar_init(&bars[kBarRcv], 1);                       // armed by the owner (expect_tx), filled by st.async
        for (int i = 0; i < kSplit; ++i) mbar_init(&bars[kBarRcvFree + i], 4);   // the owner's 4 warps
        mbar_init(&bars[kBarDrain], 1);
        mbar_init(&bars[kBarDrain2], 1);
        mbar_init(&bars[kBarSS], 1);                        // armed by this CTA (expect_tx), filled by st.async
        mbar_init(&bars[kBarQK], 4);
        mbar_init(&bars[kBarS], 1);
        mbar_init(&bars[kBarP], 4);
        mbar_init(&bars[kBarO], 1);
        for (int i = 0; i < 4; ++i) mbar_init(&bars[kBarKV + i], 1);
        for (int i = 0; i < 2; ++i) mbar_init(&bars[kBarKVFree + i], 1);
        mbar_init(&bars[kBarARcv], 1);                      // armed by the owner (expect_tx)
        mbar_init(&bars[kBarCQ], 4);
        for (int i = 0; i < 2; ++i) mbar_init(&bars[kBarCS + i], 1);
        mbar_init(&bars[kBarCP], 4);
        mbar_init(&bars[kBarCO], 1);
        fence_mbarrier_init();
    }
    for (int i = tid; i < nst && i < kMaxStages; i += blockDim.x) sinfo[i] = stage_info(stages[i]);
    if (tid == 0) {
        // this launch's generation: every CTA adds 1 to the start counter; a
        // launch adds exactly gridDim.x, so old / gridDim.x names the launch
        const unsigned long long old = atomicAdd(&ctr[0], 1ull);
        *gen_slot = old / ncta;
    }
    if (warp == 0) {
        tmem_alloc(tmem_holder, kTmemCols);
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
    if (tid == 0) DN_T(kMaxStages, 1);

    bool ok = true;
    auto wait = [&](int b, uint32_t parity) {
        if (!mbar_wait(&bars[b], parity, ok ? kWaitNs : 0ull)) ok = false;
    };

    // Issuer w's share of projection unit j of stage s (see kIssuers): its K
    // chunks into chain w of accumulator buffer um & 1, each chunk's weight
    // slot released when its MMAs complete, the buffer's full barrier
    // committed after the last (or at once when the unit has no chunk for w).
    auto issue_unit = [&](const StageInfo& S, int s, int j, int nk, uint32_t um, uint32_t gm, uint32_t xm, int w) {
        const int buf = um & 1;
        if (um >= 2) wait(kBarAccFree + buf, ((um >> 1) - 1) & 1);
        const uint32_t tacc = tmem + buf * kAccBufCols + static_cast<uint32_t>(w) * kBN;
        const uint32_t idesc = idesc_f16(static_cast<uint32_t>(S.TM), kBN, 1, 0, 0);
        int last = -1;
        for (int c = w; c < nk; c += kIssuers) last = c;
        for (int c = w; c < nk && ok; c += kIssuers) {
            const uint32_t g = gm + static_cast<uint32_t>(c);
            const int bs = g % kNB;
            wait(kBarBFull + bs, (g / kNB) & 1);
            wait(kBarXFull + c, (xm >> c) & 1u);
            if (!ok) break;
            tc_fence_after_sync();
            if (w == 0 && j == 0 && (c == 0 || c == last) && lane == 0) DN_T(s, c == 0 ? 8 : 9);
            const uint32_t aw = smem_u32(sWB(bs)), ax = smem_u32(sX(c));
            if (elect_one()) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    mma_f16_ss(tacc, smem_desc_sw128(aw + kk * 32, 16, 1024), smem_desc_sw128(ax + kk * 32, 16, 1024),
                               idesc, (c > w || kk > 0) ? 1u : 0u);
                mma_commit(&bars[kBarBFree + bs]);
                if (c == last) mma_commit(&bars[kBarAccFull + buf]);
            }
            __syncwarp();
        }
        if (last < 0) {
            if (elect_one()) mma_commit(&bars[kBarAccFull + buf]);
            __syncwarp();
        }
    };

    if (warp == kWarpW) {
        // ── int8 weight stream, running ahead across stages ────────────────
        // The weight boxes this CTA will load are pulled into L2 kPrefetch
        // stages ahead of the ring (weights depend on nothing: HBM streams them
        // while the stages wait on each other), so the ring refills from L2
        // without holding a whole launch's weights there.
        constexpr int kPrefetch = 3;
        auto prefetch_stage = [&](int s) {
            if (s >= nst) return;
            const StageInfo& S = sinfo[s];
            const int nu = units_of(S, cl, ncl), nk = S.K / 64 / kSplit;
            for (int j = 0; j < nu; ++j)
                for (int c = 0; c < nk; ++c)
                    prefetch_l2_tile(S.tmW, (rank * nk + c) * 64, (cl + j * ncl) * S.TM);
        };
        if (lane == 0)
            for (int s = 1; s <= kPrefetch; ++s) prefetch_stage(s);
        __syncwarp();
        uint32_t gw = 0;
        const uint64_t pol = l2_evict_first_policy();
        for (int s = 0; s < nst && ok; ++s) {
            const StageInfo& S = sinfo[s];
            if (lane == 0) prefetch_stage(s + 1 + kPrefetch);
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
                        tma_load_2d_hint(sW(slot), S.tmW, &bars[kBarWFull + slot], (rank * nk + c) * 64, n0, pol);
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
        uint32_t xmask = 0, last_mask = 0, gkv = 0;        // gkv: cross-attention key tiles issued
        uint32_t um2 = 0, gm2 = 0;                         // projection units / chunks, as the MMA warp's
        int loaded = 0;                                    // chunks of the last load issued
        pdl_wait();                                        // everything earlier kernels wrote
        for (int s = 0; s < nst; ++s) {
            const StageInfo& S = sinfo[s];
            if (!works_in(S, cl, ncl)) continue;
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
            if (S.kind == kDenseCrossAttn) {
                // this cluster's head: Q [128 × 64] (rows past M zero-filled), then
                // this rank's key tiles, K and V [128 × 64] each, through two stages
                if (!ok) continue;
                const int h = cl, d = S.N;
                if (elect_one()) {
                    mbar_arrive_expect_tx(&bars[kBarXFull + 0], kQKVBytes);
                    tma_load_2d(smem + kOffX, S.tmX, &bars[kBarXFull + 0], h * 64, 0);
                }
                __syncwarp();
                last_mask = xmask;
                loaded = 1;
                xmask ^= 1u;
                const KeyRange kr = key_range(S, rank);
                for (int i = 0; i < kr.n && ok; ++i, ++gkv) {
                    const int st = gkv & 1;
                    if (gkv >= 2) wait(kBarKVFree + st, ((gkv >> 1) - 1) & 1);
                    if (!ok) break;
                    if (elect_one()) {
                        const int key0 = (kr.t0 + i) * 128;
                        uint8_t* kt = smem + kOffKV + st * 2 * kQKVBytes;
                        mbar_arrive_expect_tx(&bars[kBarKV + 2 * st], kQKVBytes);
                        tma_load_2d(kt, S.tmW, &bars[kBarKV + 2 * st], h * 64, key0);
                        mbar_arrive_expect_tx(&bars[kBarKV + 2 * st + 1], kQKVBytes);
                        tma_load_2d(kt + kQKVBytes, S.tmW, &bars[kBarKV + 2 * st + 1], d + h * 64, key0);
                    }
                    __syncwarp();
                }
                continue;
            }
            if (S.kind == kDenseSelfAttn) {
                // this CTA's head: Q, K and V tiles [128 × 64] (rows past M zero-filled)
                if (ok) {
                    if (elect_one()) {
                        const int h = static_cast<int>(blockIdx.x);
                        for (int t = 0; t < 3; ++t) {
                            mbar_arrive_expect_tx(&bars[kBarXFull + t], kQKVBytes);
                            tma_load_2d(smem + kOffX + t * kQKVBytes, S.tmX, &bars[kBarXFull + t], t * S.N + h * 64, 0);
                        }
                    }
                    __syncwarp();
                    last_mask = xmask;
                    loaded = 3;
                    xmask ^= 7u;
                }
                continue;
            }
            const int nk = S.K / 64 / kSplit;
            if (ok) {
                if (elect_one()) {
                    for (int c = 0; c < nk; ++c) {
                        mbar_arrive_expect_tx(&bars[kBarXFull + c], kXBoxBytes);
                        tma_load_2d(sX(c), S.tmX, &bars[kBarXFull + c], (rank * nk + c) * 64, 0);
                    }
                }
                __syncwarp();
                if (lane == 0) DN_T(s, 12);
                last_mask = xmask;
                loaded = nk;
                xmask ^= (nk >= 32 ? 0xffffffffu : ((1u << nk) - 1u));
                // then this warp's share of the stage's MMAs
                const int nu = units_of(S, cl, ncl);
                for (int j = 0; j < nu && ok; ++j, ++um2, gm2 += nk) issue_unit(S, s, j, nk, um2, gm2, last_mask, 1);
            }
        }
        // the last loads land before the CTA leaves (bounded; immediate on the normal path)
        for (int c = 0; c < loaded; ++c)
            if (!mbar_wait(&bars[kBarXFull + c], (last_mask >> c) & 1u, kDrainNs)) ok = false;
        for (uint32_t g = gkv > 2 ? gkv - 2 : 0; g < gkv; ++g)
            for (int t = 0; t < 2; ++t)
                if (!mbar_wait(&bars[kBarKV + 2 * (g & 1) + t], (g >> 1) & 1, kDrainNs)) ok = false;
        if (!ok) {
            // this warp's MMAs in flight complete before the TMEM is freed
            if (elect_one()) mma_commit(&bars[kBarDrain2]);
            __syncwarp();
            mbar_wait(&bars[kBarDrain2], 0, kDrainNs);
        }
    } else if (warp == kWarpMma) {
        // ── MMA issuer ──────────────────────────────────────────────────────
        uint32_t gm = 0, um = 0, xmask = 0, au = 0;        // xmask as the activation loader's
        uint32_t cq = 0, ct = 0;                           // cross-attention stages / key tiles
        for (int s = 0; s < nst && ok; ++s) {
            const StageInfo& S = sinfo[s];
            if (S.kind == kDenseCrossAttn) {
                if (!works_in(S, cl, ncl)) continue;
                xmask ^= 1u;
                // S_i = Q·K_iᵀ (128 queries × 128 keys, bf16) into TMEM buffer i & 1,
                // issued one tile ahead of the softmax; O += P_i·V_i with P (fp16)
                // read from that buffer
                wait(kBarCQ, cq & 1);
                ++cq;
                if (!ok) break;
                const KeyRange kr = key_range(S, rank);    // after the stage's dependency
                tc_fence_after_sync();
                const uint32_t aq = smem_u32(smem + kOffX);
                constexpr uint32_t idS = idesc_f16(128, 128, 1, 0, 0);
                constexpr uint32_t idPV = idesc_f16(128, 64, 0, 0, 1);
                auto issue_s = [&](uint32_t g) {
                    const uint32_t st = g & 1u;
                    wait(kBarKV + 2 * st, (g >> 1) & 1);
                    if (!ok) return;
                    tc_fence_after_sync();
                    const uint32_t ak = smem_u32(smem + kOffKV + st * 2 * kQKVBytes);
                    if (elect_one()) {
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            mma_f16_ss(tmem + (g & 1u) * 128, smem_desc_sw128(aq + kk * 32, 16, 1024),
                                       smem_desc_sw128(ak + kk * 32, 16, 1024), idS, kk > 0 ? 1u : 0u);
                        mma_commit(&bars[kBarCS + (g & 1u)]);
                    }
                    __syncwarp();
                };
                if (kr.n > 0) issue_s(ct);
                for (int i = 0; i < kr.n && ok; ++i, ++ct) {
                    if (i + 1 < kr.n) {
                        // buffer (ct + 1) & 1 was read by the previous tile's P·V
                        if (i >= 1) wait(kBarCO, (ct - 1) & 1);
                        issue_s(ct + 1);
                    }
                    const uint32_t st = ct & 1u;
                    wait(kBarCP, ct & 1);
                    wait(kBarKV + 2 * st + 1, (ct >> 1) & 1);
                    if (!ok) break;
                    tc_fence_after_sync();
                    const uint32_t av = smem_u32(smem + kOffKV + st * 2 * kQKVBytes + kQKVBytes);
                    if (elect_one()) {
#pragma unroll
                        for (int k = 0; k < 8; ++k)                // 16 keys per MMA
                            mma_f16_ts(tmem + kColO, tmem + kColCrossP + (ct & 1u) * 64 + 8 * k,
                                       smem_desc_sw128(av + k * 2048, 8192, 1024), idPV,
                                       (i > 0 || k > 0) ? 1u : 0u);
                        mma_commit(&bars[kBarKVFree + st]);
                        mma_commit(&bars[kBarCO]);
                    }
                    __syncwarp();
                }
                continue;
            }
            if (S.kind == kDenseSelfAttn) {
                if (!works_in(S, cl, ncl)) continue;
                // S = Q·Kᵀ (M 128 queries, N 80 keys, K 64), bf16 operands from the
                // TMA tiles, once the epilogue warps have normalised Q/K and
                // converted V; then O = P·V with P (fp16) from TMEM
                wait(kBarQK, au & 1);
                if (!ok) break;
                tc_fence_after_sync();
                const uint32_t aq = smem_u32(smem + kOffX), ak = aq + kQKVBytes, av = ak + kQKVBytes;
                constexpr uint32_t idS = idesc_f16(128, kBN, 1, 0, 0);
                constexpr uint32_t idPV = idesc_f16(128, 64, 0, 0, 1);
                if (elect_one()) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_f16_ss(tmem + kColS, smem_desc_sw128(aq + kk * 32, 16, 1024),
                                   smem_desc_sw128(ak + kk * 32, 16, 1024), idS, kk > 0 ? 1u : 0u);
                    mma_commit(&bars[kBarS]);
                }
                __syncwarp();
                wait(kBarP, au & 1);
                if (!ok) break;
                tc_fence_after_sync();
                if (elect_one()) {
#pragma unroll
                    for (int k = 0; k < kBN / 16; ++k)              // 16 keys per MMA
                        mma_f16_ts(tmem + kColO, tmem + kColP + 8 * k, smem_desc_sw128(av + k * 2048, 8192, 1024),
                                   idPV, k > 0 ? 1u : 0u);
                    mma_commit(&bars[kBarO]);
                }
                __syncwarp();
                ++au;
                xmask ^= 7u;
                continue;
            }
            const int nu = units_of(S, cl, ncl);
            if (nu == 0) continue;
            const int nk = S.K / 64 / kSplit;
            for (int j = 0; j < nu && ok; ++j, ++um, gm += nk) issue_unit(S, s, j, nk, um, gm, xmask, 0);
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
            const StageInfo& S = sinfo[s];
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
                    if (ct == 0 && j == 0 && c == nk - 1) DN_T(s, 11);
                    if (lane == 0 && j == 0 && c < 8) DN_T(s, 32 + c);
                }
            }
        }
    } else {
        // ── epilogue (warps 7..10; TMEM quadrant q = warp % 4 = owner rank) ──
        const int et = tid - kWarpEpi0 * 32;               // 0..127
        const int q = warp & 3;
        constexpr int kMaxIt = 2;                          // owner units (<= 80 · 16 / 8) / 128 threads
        uint32_t ue = 0, xs = 0, au = 0, xmask = 0;        // xmask as the activation loader's
        uint32_t ssn = 0;                                  // stages whose RMS sums this CTA exchanged
        uint32_t cq = 0, ct = 0;                           // cross-attention stages / key tiles
        const int mvalid = min(M, kBN);
        for (int s = 0; s < nst; ++s) {
            const StageInfo& S = sinfo[s];
            if (S.kind == kDenseCrossAttn) {
                if (works_in(S, cl, ncl)) {
                    cross_attention_epilogue(S, smem, bars, tmem, rcv, xs, xmask, cq, ct, mvalid, rank, ok);
                    ++xs; ++cq;
                    xmask ^= 1u;
                }
                named_bar_sync(1, kEpiThreads);
                if (et == 0) {
                    DN_T(s, 2);
                    red_release_gpu_add(&ctr[1 + s], 1ull);
                    DN_T(s, 3);
                }
                continue;
            }
            if (S.kind == kDenseSelfAttn) {
                if (works_in(S, cl, ncl)) {
                    self_attention_epilogue(S, smem, bars, tmem, xs, xmask, au, au, mvalid, ok);
                    ++xs; ++au;
                    xmask ^= 7u;
                }
                named_bar_sync(1, kEpiThreads);
                if (et == 0) {
                    DN_T(s, 2);
                    red_release_gpu_add(&ctr[1 + s], 1ull);
                    DN_T(s, 3);
                }
                continue;
            }
            const int nu = units_of(S, cl, ncl);
            if (nu > 0) {
                const int nk0 = S.K / 64 / kSplit;
                xmask ^= (nk0 >= 32 ? 0xffffffffu : ((1u << nk0) - 1u));
            }
            const int TM = S.TM, RPW = TM / 4;             // rows per TMEM quadrant = rows per owner
            const int segs = RPW / 8;                      // 8-channel segments per owned row
            const int units = mvalid * segs;
            for (int j = 0; j < nu; ++j, ++ue) {
                const int n0 = (cl + j * ncl) * TM;
                const int nb = n0 + rank * RPW;            // first channel this CTA owns
                // (0) the unit's constants (weights' scales, bias, next norm's weight):
                // independent of the stage's dependency, so loaded before waiting for it.
                // Every global load below lands in the register it is used from, raw,
                // so that nothing waits for it before its first use.
                const bool lane_ok = lane < RPW;
                const int trow = q * RPW + lane;               // tile row (owner q, slot lane)
                float sc = 0.f;
                if (lane_ok && n0 + trow < S.N)
                    asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(sc) : "l"(S.w_scale + n0 + trow));
                uint4 rbias[kMaxIt], rg[kMaxIt], rr[kMaxIt][2];
#pragma unroll
                for (int it = 0; it < kMaxIt; ++it) {
                    const int u = et + it * kEpiThreads;
                    const int m = u < units ? u / segs : 0, n = nb + (u < units ? (u - m * segs) * 8 : 0);
                    const bool use = u < units && n < S.N;
                    rbias[it] = make_uint4(0u, 0u, 0u, 0u);
                    rg[it] = make_uint4(0u, 0u, 0u, 0u);
                    if (use && S.bias != nullptr) rbias[it] = ld_nc_u4(S.bias + n);
                    if (use && S.g_next != nullptr) rg[it] = ld_nc_u4(S.g_next + n);
                }
                // (1) the stage's dependency (once per stage)
                if (j == 0) {
                    wait(kBarDep, xs & 1);
                    if (et == 0) { DN_T(s, 16); DN_C(s, 20); }
                }
                // (2) the residual rows this thread's owner pass adds (written by earlier stages)
#pragma unroll
                for (int it = 0; it < kMaxIt; ++it) {
                    const int u = et + it * kEpiThreads;
                    const int m = u < units ? u / segs : 0, n = nb + (u < units ? (u - m * segs) * 8 : 0);
                    const bool use = u < units && n < S.N;
                    rr[it][0] = make_uint4(0u, 0u, 0u, 0u);
                    rr[it][1] = make_uint4(0u, 0u, 0u, 0u);
                    if (use && S.residual != nullptr) {
                        if (S.y_f32) {
                            const float* rp = static_cast<const float*>(S.residual) + m * S.ldr + n;
                            rr[it][0] = ld_cg_u4(rp);
                            rr[it][1] = ld_cg_u4(rp + 4);
                        } else {
                            rr[it][0] = ld_cg_u4(static_cast<const __nv_bfloat16*>(S.residual) + m * S.ldr + n);
                        }
                    }
                }
                // (1b) rows' RMS factors from the producing stage's partial sums (once per stage)
                if (j == 0) {
                    if (S.ss_in != nullptr) {
                        // The cluster's four CTAs each read a quarter of the
                        // partials (one read of every partial per cluster instead of
                        // per CTA: 132 CTAs would all hit the same lines) and
                        // exchange their 80 quarter sums through shared memory.
                        // Thread t < 120 sums the float4 column t % 20 (token rows
                        // 4·(t % 20) .. +3) over partials group t / 20 (six groups of
                        // consecutive partials of the quarter), all its loads in
                        // flight at once; the group sums, then the quarters, are
                        // added in a fixed order.
                        constexpr int kCols = kBN / 4, kGroups = kEpiThreads / kCols;   // 20, 6
                        constexpr int kBatch = 8;           // loads in flight: a group's share of a quarter
                        const int np = S.n_ss_in;
                        const int q0p = rank * np / kSplit, q1p = (rank + 1) * np / kSplit;
                        const int col = et % kCols, grpi = et / kCols;
                        const int per = (q1p - q0p + kGroups - 1) / kGroups;
                        const int p0 = q0p + grpi * per, p1 = min(q1p, p0 + per);
                        if (et == 0) mbar_arrive_expect_tx(&bars[kBarSS], static_cast<uint32_t>(kSplit * kBN * 4));
                        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                        if (grpi < kGroups) {
                            for (int pb = p0; pb < p1; pb += kBatch) {
                                float4 t[kBatch];
#pragma unroll
                                for (int i = 0; i < kBatch; ++i)
                                    t[i] = pb + i < p1 ? ld_cg_f4(S.ss_in + (pb + i) * kBN + 4 * col)
                                                       : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                                for (int i = 0; i < kBatch; ++i) {
                                    acc.x += t[i].x; acc.y += t[i].y; acc.z += t[i].z; acc.w += t[i].w;
                                }
                            }
                            *reinterpret_cast<float4*>(red + grpi * kBN + 4 * col) = acc;
                        }
                        named_bar_sync(1, kEpiThreads);
                        if (et < kBN) {
                            float tot = 0.f;
#pragma unroll
                            for (int g = 0; g < kGroups; ++g) tot += red[g * kBN + et];
                            sst[et] = tot;
                        }
                        named_bar_sync(1, kEpiThreads);
                        if (et < kSplit * kCols) {
                            // thread t: float4 column t % 20 of this quarter to rank t / 20
                            const uint32_t dst_rank = static_cast<uint32_t>(et / kCols), c4 = et % kCols;
                            const uint32_t dst = dsmem_map(smem_u32(ssx + rank * kBN + 4 * c4), dst_rank);
                            const uint32_t rb = dsmem_map(smem_u32(&bars[kBarSS]), dst_rank);
                            st_async_v4(dst, *reinterpret_cast<const float4*>(sst + 4 * c4), rb);
                        }
                        if (!cwait(&bars[kBarSS], ssn & 1, ok ? kWaitNs : 0ull)) ok = false;
                        ++ssn;
                        if (et < mvalid) {
                            const float tot = (ssx[et] + ssx[kBN + et]) + (ssx[2 * kBN + et] + ssx[3 * kBN + et]);
                            rinv[et] = 1.f / sqrtf(tot / static_cast<float>(S.K) + S.eps);
                        }
                    }
                    named_bar_sync(1, kEpiThreads);
                }
                if (et == 0 && j == 0) { DN_T(s, 17); DN_C(s, 21); }
                if (et == 0 && j == 0) DN_T(s, 18);
                // (3) accumulator → scaled partials into the owner's receive area
                static_assert(kIssuers == 2, "the epilogue adds two chains");
                const int nk_unit = S.K / 64 / kSplit;
                const int buf = ue & 1;
                // arm this CTA's receive barrier for the unit: the four sources' partials
                // of its RPW rows (this thread has passed the previous unit's phase)
                if (et == 0)
                    mbar_arrive_expect_tx(&bars[kBarRcv], static_cast<uint32_t>(kSplit * RPW * kBN * 4));
                if (ue >= 1) {
                    // the owner has read this area's previous contents
                    if (!cwait(&bars[kBarRcvFree + q], (ue - 1) & 1, ok ? kWaitNs : 0ull)) ok = false;
                }
                if (et == 0 && j == 0) DN_T(s, 10);
                wait(kBarAccFull + buf, (ue >> 1) & 1);
                if (et == 0 && j == 0) { DN_T(s, 1); DN_C(s, 22); }
                tc_fence_after_sync();
                const uint32_t tq = tmem + buf * kAccBufCols + (static_cast<uint32_t>(q * 32) << 16);
                const uint32_t base = dsmem_map(smem_u32(rcv + (rank * RPW + (lane_ok ? lane : 0)) * kBN),
                                                static_cast<uint32_t>(q));
                const uint32_t rbar = dsmem_map(smem_u32(&bars[kBarRcv]), static_cast<uint32_t>(q));
#pragma unroll 1
                for (int blk = 0; blk < 3; ++blk) {                 // 32 token columns at a time
                    float v[32];
                    tmem_ld32(tq + 32 * blk, v);
                    if (nk_unit > 1) {                     // chain 1 (kIssuers == 2)
                        float w[32];
                        tmem_ld32(tq + kBN + 32 * blk, w);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] += w[i];
                    }
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
                if (et == 0 && j == nu - 1) { DN_T(s, 4); DN_C(s, 23); }
                // (4) owner pass: rows [nb, nb + RPW) of the tile, every token
                if (!cwait(&bars[kBarRcv], ue & 1, ok ? kWaitNs : 0ull)) ok = false;
                if (et == 0 && j == nu - 1) { DN_T(s, 5); DN_C(s, 24); }
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
                if (et == 0 && j == nu - 1) { DN_T(s, 13); DN_C(s, 25); }
                __syncwarp();
                if (lane < kSplit) mbar_arrive_remote(&bars[kBarRcvFree + rank], static_cast<uint32_t>(lane));
                if (et == 0 && j == nu - 1) { DN_T(s, 6); DN_C(s, 26); }
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
                        float rres[8];
                        if (S.y_f32) {
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                rres[k] = __uint_as_float((&rr[it][0].x)[k]);
                                rres[4 + k] = __uint_as_float((&rr[it][1].x)[k]);
                            }
                        } else {
                            const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rr[it][0]);
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                const float2 f = __bfloat1622float2(r2[k]);
                                rres[2 * k] = f.x; rres[2 * k + 1] = f.y;
                            }
                        }
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
                                outv[2 * k + h] = t + rres[2 * k + h];
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
            if (et == 0) { DN_T(s, 7); DN_C(s, 27); }
            // (5) this CTA is done with stage s: publish its writes, bump the counter
            named_bar_sync(1, kEpiThreads);
            if (et == 0) {
                // release at GPU scope: covers every epilogue thread's stores, which the
                // named barrier ordered before it; readers acquire and fence the
                // async proxy before their TMA loads
                { DN_T(s, 2); DN_C(s, 28); }
                red_release_gpu_add(&ctr[1 + s], 1ull);
                { DN_T(s, 3); DN_C(s, 29); }
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
        tmem_dealloc(tmem, kTmemCols);
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
    if (M < 1 || M > dense::kXRows) return SFB_ERR_SHAPE;
    if (TM != dense::kTM || N % TM != 0 || K % (64 * dense::kSplit) != 0 ||
        K / 64 / dense::kSplit > dense::kNX)
        return SFB_ERR_SHAPE;
    S.N = N; S.K = K; S.TM = TM; S.tiles = N / TM;
    {
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
        cuuint64_t str[1] = {(cuuint64_t)(ldx * 2)};
        cuuint32_t box[2] = {64, (cuuint32_t)dense::kXRows};
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

// A self-attention stage over the fused qkv activations [M, 3·D] (row stride
// ldqkv): Q, K, V of head h at columns h·64, D + h·64, 2·D + h·64; out: [M, D].
int dense_attn_stage_init(DenseStage& S, const void* qkv, int64_t ldqkv, int M, int D, void* out, int64_t ldo,
                          const __nv_bfloat16* qn_w, const __nv_bfloat16* kn_w, float eps, float scale) {
    if (M < 1 || M > dense::kBN || D % 64 != 0 || qn_w == nullptr || kn_w == nullptr) return SFB_ERR_SHAPE;
    if (D / 64 > dense::kSplit * dense_clusters(device_info())) return SFB_ERR_SHAPE;   // one CTA per head
    cuuint64_t dims[2] = {(cuuint64_t)(3 * D), (cuuint64_t)M};
    cuuint64_t str[1] = {(cuuint64_t)(ldqkv * 2)};
    cuuint32_t box[2] = {64, 128};
    cuuint32_t es[2] = {1, 1};
    SFB_TRY(encode_tensor_map(&S.tmX, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(qkv), dims, str, box,
                              es, CU_TENSOR_MAP_SWIZZLE_128B));
    S.kind = kDenseSelfAttn;
    S.N = D; S.tiles = D / 64;
    S.y = out; S.ldy = ldo;
    S.qn_w = qn_w; S.kn_w = kn_w;
    S.eps = eps; S.sm_scale = scale;
    return SFB_OK;
}

// A cross-attention stage: queries q [M, D] (row stride ldq) against the
// cache kv [Lk, ldkv] whose row holds K (bf16, k-normed) in columns [0, D)
// and V (fp16) in [D, 2D); the first *kv_len keys are valid (all when
// kv_len is null). out [M, D] (ldo) gets softmax(qnorm(q)·Kᵀ·scale)·V per
// head of 64. Needs one cluster per head.
int dense_cross_stage_init(DenseStage& S, const void* q, int64_t ldq, int M, int D, const void* kv, int64_t ldkv,
                           int Lk, const int32_t* kv_len, void* out, int64_t ldo, const __nv_bfloat16* qn_w,
                           float eps, float scale) {
    if (M < 1 || M > dense::kBN || D % 64 != 0 || Lk < 1 || ldkv < 2 * D || qn_w == nullptr) return SFB_ERR_SHAPE;
    if (D / 64 > dense_clusters(device_info())) return SFB_ERR_SHAPE;
    cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)M};
    cuuint64_t str[1] = {(cuuint64_t)(ldq * 2)};
    cuuint32_t box[2] = {64, 128};
    cuuint32_t es[2] = {1, 1};
    SFB_TRY(encode_tensor_map(&S.tmX, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(q), dims, str, box,
                              es, CU_TENSOR_MAP_SWIZZLE_128B));
    // K and V through one map (both 2-byte elements; zero fill past Lk)
    cuuint64_t kdims[2] = {(cuuint64_t)(2 * D), (cuuint64_t)Lk};
    cuuint64_t kstr[1] = {(cuuint64_t)(ldkv * 2)};
    SFB_TRY(encode_tensor_map(&S.tmW, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(kv), kdims, kstr, box,
                              es, CU_TENSOR_MAP_SWIZZLE_128B));
    S.kind = kDenseCrossAttn;
    S.N = D; S.K = D; S.tiles = D / 64;
    S.lk = Lk; S.kv_len = kv_len;
    S.y = out; S.ldy = ldo;
    S.qn_w = qn_w;
    S.eps = eps; S.sm_scale = scale;
    return SFB_OK;
}

// One launch over stages[0, nst) (device memory); ctr: nst + 1 counters of
// this launch slot (zero at allocation, never reset).
#ifdef SFB_TRACE
static unsigned long long* g_dense_trace = nullptr;
extern "C" void sfb_debug_set_dense_trace(void* p) { g_dense_trace = static_cast<unsigned long long*>(p); }
#endif

int dense_launch(const DenseStage* stages, int nst, unsigned long long* ctr, int M, cudaStream_t stream, bool pdl,
                 int trace_slot) {
    if (nst < 1 || nst > dense::kMaxStages || M < 1 || M > dense::kBN) return SFB_ERR_SHAPE;
    const DeviceInfo& dev = device_info();
    const int ncl = dense_clusters(dev);
    if (ncl <= 0) { record_cuda_error(cudaErrorInvalidConfiguration, "dense kernel clusters"); return SFB_ERR_LAUNCH; }
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = dense_config(ncl, stream, attr, pdl);
#ifdef SFB_TRACE
    unsigned long long* tr = (g_dense_trace != nullptr && trace_slot >= 0)
                                 ? g_dense_trace + static_cast<size_t>(trace_slot) * 160 * dense::kTrStages * 40 : nullptr;
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
