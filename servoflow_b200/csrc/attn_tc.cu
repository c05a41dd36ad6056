// attn_tc.cu — tensor-core attention forward for sm_100a (head_dim 64,
// fp16/bf16 in, fp32 softmax/accumulate).
//
// Replaces the reference's FlashAttention-2 SM80 forward
// (src/backend/cuda/flash_attn/flash_fwd_kernel.h:52-497, reached through
// src/backend/cuda/ops/attention.cu:29-80) with a Blackwell design built for
// RDT-1B's shapes: Lq = 67 action tokens against Lk ∈ {67, 1024 (masked
// language), 4374 (image)}.
//
// One CTA = 128 query rows × a contiguous range of 128-key tiles, 4 warps.
//   * TMA (SWIZZLE_128B) stages Q once and K/V tiles through a 2-deep ring.
//   * tcgen05.mma computes S = Q·Kᵀ (M=128, N=128, K=64) into TMEM; thread t
//     owns query row t (TMEM lane t), so the row max / row sum of the online
//     softmax are thread-local — no shuffles and no shared-memory reductions.
//   * P (bf16/fp16) is written to shared memory in the UMMA K-major SW128
//     layout — keys 0..63 into a dedicated buffer, keys 64..127 over the
//     K tile of the same stage (free once S is computed) — and
//     O_tile = P·V (M=128, N=64, K=128) runs on tcgen05 with V read MN-major
//     straight from its TMA tile. The fp32 running O lives in registers.
//   * The next tile's S MMA is issued right behind the current P·V, so the
//     tensor pipe, the softmax and the TMA refill overlap; two CTAs share an
//     SM (≈97 KB smem, 256 TMEM columns each).
//   * Split-K over Lk: the CTAs of one (batch, head, q-tile) form a thread-
//     block cluster; each keeps (m, l, O) for its key range, and the partials
//     are merged through distributed shared memory at the end. No global
//     scratch, no atomics, no inter-CTA spin waits (cluster barriers are
//     hardware barriers).
//
// Every mbarrier wait is bounded (1 s); on expiry the CTA finishes its
// control flow without further waiting, skips its output and records
// SFB_ERR_DEVICE_TIMEOUT in g_sfb_device_error.
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
};

namespace attn_tc {

constexpr int kThreads   = 128;
constexpr int kTileKeys  = 128;
constexpr int kTileBytes = 128 * 128;     // 128 rows × 64 halves
constexpr int kOffQ      = 0;
constexpr int kOffP      = kOffQ + kTileBytes;
constexpr int kOffStage  = kOffP + kTileBytes;           // [2] × (K, V)
constexpr int kOffBar    = kOffStage + 4 * kTileBytes;    // 98304
constexpr int kOffTmem   = kOffBar + 64;
constexpr int kOffMask   = kOffTmem + 16;
constexpr int kSmemUsed  = kOffMask + 128;
constexpr int kSmemBytes = kSmemUsed + 1024;              // + alignment slack
constexpr int kTmemCols  = 256;                           // S: 0..127, O tile: 128..191
// Split-K merge buffers reuse the stage region once the main loop is done.
constexpr int kOStride   = 68;                            // floats per row (16-B aligned, skewed)
constexpr int kOffCombO  = kOffStage;
constexpr int kOffCombM  = kOffCombO + 128 * kOStride * 4;
constexpr int kOffCombL  = kOffCombM + 128 * 4;
static_assert(kOffCombL + 128 * 4 <= kOffBar, "merge buffers must fit in the stage region");

enum Bar { kBarQ = 0, kBarK0 = 1, kBarK1 = 2, kBarV0 = 3, kBarV1 = 4, kBarS = 5, kBarO = 6 };

template <typename T> struct Pack2;
template <> struct Pack2<__nv_bfloat16> {
    static __device__ __forceinline__ uint32_t pack(float a, float b, float& ra, float& rb) {
        __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
        float2 f = __bfloat1622float2(v);
        ra = f.x; rb = f.y;
        return *reinterpret_cast<uint32_t*>(&v);
    }
};
template <> struct Pack2<__half> {
    static __device__ __forceinline__ uint32_t pack(float a, float b, float& ra, float& rb) {
        __half2 v = __floats2half2_rn(a, b);
        float2 f = __half22float2(v);
        ra = f.x; rb = f.y;
        return *reinterpret_cast<uint32_t*>(&v);
    }
};

template <typename T>
__device__ __forceinline__ void store_row8(T* dst, const float* v) {
    float d0, d1;
    uint4 u;
    u.x = Pack2<T>::pack(v[0], v[1], d0, d1);
    u.y = Pack2<T>::pack(v[2], v[3], d0, d1);
    u.z = Pack2<T>::pack(v[4], v[5], d0, d1);
    u.w = Pack2<T>::pack(v[6], v[7], d0, d1);
    *reinterpret_cast<uint4*>(dst) = u;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 2)
attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                   const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV,
                   const AttnTcParams p) {
    using namespace ptx;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t*  sQ    = smem + kOffQ;
    uint8_t*  sP    = smem + kOffP;
    uint64_t* bars  = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kOffTmem);
    uint8_t*  sMask = smem + kOffMask;
    auto sK = [&](int s) { return smem + kOffStage + (2 * s) * kTileBytes; };
    auto sV = [&](int s) { return smem + kOffStage + (2 * s + 1) * kTileBytes; };

    const int tid  = threadIdx.x;
    const int warp = tid >> 5;
    const int split = blockIdx.x;
    const int h     = blockIdx.y;
    const int b     = blockIdx.z / p.qtiles;
    const int qt    = blockIdx.z - b * p.qtiles;
    const int hk    = h / (p.H / p.Hkv);
    const int q0    = qt * 128;
    const int rows  = min(128, p.Lq - q0);

    // Key range of this (batch, q-tile), then this CTA's share of its tiles.
    int kend = p.Lk;
    if (p.kv_len != nullptr) kend = min(kend, max(0, p.kv_len[b]));
    if (p.causal) kend = min(kend, q0 + rows);
    const int ntiles  = (kend + kTileKeys - 1) / kTileKeys;
    const int tbase   = ntiles / p.splits;
    const int trem    = ntiles - tbase * p.splits;
    const int t_begin = split * tbase + min(split, trem);
    const int ntl     = tbase + (split < trem ? 1 : 0);

    if (tid == 0) {
        for (int i = 0; i < 7; ++i) mbar_init(&bars[i], 1);
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
    const uint32_t tmem     = *tmem_holder;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t tS = tmem, tO = tmem + 128;

    constexpr uint32_t kBF = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
    constexpr uint32_t idS  = idesc_f16(128, 128, kBF, 0, 0);   // Q (K-major) · K (K-major)
    constexpr uint32_t idPV = idesc_f16(128, 64, kBF, 0, 1);    // P (K-major) · V (MN-major)

    bool ok = true;
    auto wait = [&](int bar, uint32_t parity) {
        if (!mbar_wait(&bars[bar], parity, ok ? 1000000000ull : 0ull)) ok = false;
    };
    auto issue_kv = [&](int stage, int tile) {
        const int key0 = tile * kTileKeys;
        mbar_arrive_expect_tx(&bars[kBarK0 + stage], kTileBytes);
        tma_load_4d(sK(stage), &tmK, &bars[kBarK0 + stage], 0, key0, hk, b);
        mbar_arrive_expect_tx(&bars[kBarV0 + stage], kTileBytes);
        tma_load_4d(sV(stage), &tmV, &bars[kBarV0 + stage], 0, key0, hk, b);
    };
    auto issue_s = [&](int stage) {
        const uint32_t aq = smem_u32(sQ), ak = smem_u32(sK(stage));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
            mma_f16_ss(tS, smem_desc_sw128(aq + kk * 32, 16, 1024),
                       smem_desc_sw128(ak + kk * 32, 16, 1024), idS, kk > 0 ? 1u : 0u);
        mma_commit(&bars[kBarS]);
    };

    if (tid == 0 && ntl > 0) {
        mbar_arrive_expect_tx(&bars[kBarQ], kTileBytes);
        tma_load_4d(sQ, &tmQ, &bars[kBarQ], 0, q0, h, b);
        issue_kv(0, t_begin);
        if (ntl > 1) issue_kv(1, t_begin + 1);
        wait(kBarQ, 0);
        wait(kBarK0, 0);
        tc_fence_after_sync();
        issue_s(0);
    }

    float o_acc[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) o_acc[i] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;
    const int  qi          = q0 + tid;
    const bool warp_active = warp * 32 < rows;
    const bool use_mask    = p.key_mask != nullptr;
    const float sl2        = p.sl2;

    for (int j = 0; j < ntl; ++j) {
        const int s    = j & 1;
        const int key0 = (t_begin + j) * kTileKeys;
        if (use_mask) {
            const int key = key0 + tid;
            sMask[tid] = key < kend ? p.key_mask[static_cast<int64_t>(b) * p.mask_sb + key] : 0;
        }
        wait(kBarS, j & 1);
        tc_fence_after_sync();
        __syncthreads();   // sMask visible; previous tile fully consumed

        float alpha = 1.f;
        uint8_t* sPhi = sK(s);
        if (warp_active) {
            const bool full_tile = (key0 + kTileKeys <= kend) && !use_mask && !p.causal;
            auto valid = [&](int c) {
                const int key = key0 + c;
                bool v = key < kend;
                if (use_mask) v = v && sMask[c] != 0;
                if (p.causal) v = v && key <= qi;
                return v;
            };
            // pass 1: row max of the scaled logits (log2 domain)
            float mx = m_run;
            float sc[32];
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
                tmem_ld32(tS + lane_off + ch * 32, sc);
                tmem_ld_wait();
                if (full_tile) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) mx = fmaxf(mx, sc[i] * sl2);
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (valid(ch * 32 + i)) mx = fmaxf(mx, sc[i] * sl2);
                }
            }
            const float m_use = (mx == -INFINITY) ? 0.f : mx;
            alpha = ptx::ex2(m_run - m_use);
            // pass 2: P = exp2(s - m), rounded to the operand type, into smem
            float lsum = 0.f;
            const int r7 = tid & 7;
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
                tmem_ld32(tS + lane_off + ch * 32, sc);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const bool v = full_tile || valid(ch * 32 + i);
                    sc[i] = v ? ptx::ex2(sc[i] * sl2 - m_use) : 0.f;
                }
                uint8_t* base = (ch < 2 ? sP : sPhi) + tid * 128;
#pragma unroll
                for (int g = 0; g < 4; ++g) {          // 4 chunks of 8 keys
                    const int chunk = (ch & 1) * 4 + g;
                    float r0, r1;
                    uint4 u;
                    u.x = Pack2<T>::pack(sc[g * 8 + 0], sc[g * 8 + 1], r0, r1); lsum += r0 + r1;
                    u.y = Pack2<T>::pack(sc[g * 8 + 2], sc[g * 8 + 3], r0, r1); lsum += r0 + r1;
                    u.z = Pack2<T>::pack(sc[g * 8 + 4], sc[g * 8 + 5], r0, r1); lsum += r0 + r1;
                    u.w = Pack2<T>::pack(sc[g * 8 + 6], sc[g * 8 + 7], r0, r1); lsum += r0 + r1;
                    *reinterpret_cast<uint4*>(base + ((chunk ^ r7) << 4)) = u;
                }
            }
            l_run = l_run * alpha + lsum;
            m_run = mx;
        }
        fence_proxy_async_smem();
        tc_fence_before_sync();
        __syncthreads();   // P complete; S consumed

        if (tid == 0) {
            tc_fence_after_sync();
            wait(kBarV0 + s, (j >> 1) & 1);
            const uint32_t ap = smem_u32(sP), aph = smem_u32(sPhi), av = smem_u32(sV(s));
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t a = (k < 4 ? ap : aph) + (k & 3) * 32;
                mma_f16_ss(tO, smem_desc_sw128(a, 16, 1024),
                           smem_desc_sw128(av + k * 2048, 8192, 1024), idPV, k > 0 ? 1u : 0u);
            }
            mma_commit(&bars[kBarO]);
            if (j + 1 < ntl) {
                wait(kBarK0 + (s ^ 1), ((j + 1) >> 1) & 1);
                tc_fence_after_sync();
                issue_s(s ^ 1);
            }
        }
        wait(kBarO, j & 1);
        tc_fence_after_sync();
        if (warp_active) {
            float ot[32];
#pragma unroll
            for (int ch = 0; ch < 2; ++ch) {
                tmem_ld32(tO + lane_off + ch * 32, ot);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; ++i) o_acc[ch * 32 + i] = o_acc[ch * 32 + i] * alpha + ot[i];
            }
        }
        if (tid == 0 && j + 2 < ntl) issue_kv(s, t_begin + j + 2);
    }

    // ── epilogue ────────────────────────────────────────────────────────────
    T* out = static_cast<T*>(p.out);
    const int64_t row_base = static_cast<int64_t>(b) * p.o_sb + static_cast<int64_t>(h) * p.o_sh;
    if (p.splits == 1) {
        if (tid < rows && ok) {
            const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
            T* dst = out + row_base + static_cast<int64_t>(q0 + tid) * p.o_ss;
#pragma unroll
            for (int c = 0; c < 64; c += 8) {
                float v[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = o_acc[c + i] * inv;
                store_row8<T>(dst + c, v);
            }
        }
    } else {
        float* sO = reinterpret_cast<float*>(smem + kOffCombO);
        float* sM = reinterpret_cast<float*>(smem + kOffCombM);
        float* sL = reinterpret_cast<float*>(smem + kOffCombL);
        if (tid < rows) {
#pragma unroll
            for (int c = 0; c < 64; c += 4)
                *reinterpret_cast<float4*>(sO + tid * kOStride + c) =
                    make_float4(o_acc[c], o_acc[c + 1], o_acc[c + 2], o_acc[c + 3]);
            sM[tid] = m_run;
            sL[tid] = l_run;
        }
        cluster_sync();
        // CTA `split` merges rows split, split+C, ...; 16 threads per row, 4 columns each.
        const int C   = p.splits;
        const int sub = tid >> 4, c4 = (tid & 15) * 4;
        const uint32_t aO = smem_u32(sO), aM = smem_u32(sM), aL = smem_u32(sL);
        for (int row = split + sub * C; row < rows; row += 8 * C) {
            float M = -INFINITY;
            for (int r = 0; r < C; ++r) M = fmaxf(M, dsmem_ld_f32(dsmem_map(aM + row * 4, r)));
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            float L = 0.f;
            if (M != -INFINITY) {
                for (int r = 0; r < C; ++r) {
                    const float mr = dsmem_ld_f32(dsmem_map(aM + row * 4, r));
                    const float w  = ptx::ex2(mr - M);
                    L += w * dsmem_ld_f32(dsmem_map(aL + row * 4, r));
                    const float4 o = dsmem_ld_f32x4(dsmem_map(aO + (row * kOStride + c4) * 4, r));
                    acc.x += w * o.x; acc.y += w * o.y; acc.z += w * o.z; acc.w += w * o.w;
                }
            }
            const float inv = L > 0.f ? 1.f / L : 0.f;
            if (ok) {
                T* dst = out + row_base + static_cast<int64_t>(q0 + row) * p.o_ss + c4;
                float d0, d1;
                uint2 u;
                u.x = Pack2<T>::pack(acc.x * inv, acc.y * inv, d0, d1);
                u.y = Pack2<T>::pack(acc.z * inv, acc.w * inv, d0, d1);
                *reinterpret_cast<uint2*>(dst) = u;
            }
        }
        cluster_sync();   // keep this CTA's smem alive until every peer has read it
    }

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

int choose_attn_splits(int units, int ntiles_max, int num_sms) {
    const int target = 2 * num_sms;   // two resident CTAs per SM
    int s = (target + units - 1) / units;
    s = std::min(s, 16);
    s = std::min(s, std::max(1, ntiles_max / 2));  // keep >= 2 tiles per split
    return std::max(1, s);
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
