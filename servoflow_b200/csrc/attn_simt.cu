// attn_simt.cu — CUDA-core attention forward: the fp32 path (RDT-1B action
// self-attention at fp32, which must agree with the reference's fp32 kernel
// to 1e-5) and every head_dim other than 64.
//
// Same semantics as the reference's fp32 kernel (src/backend/cuda/ops/
// attention.cu:90-139: fp32 online softmax, causal cut at key > query),
// different parallelisation: the reference runs one thread per query row
// serially over all keys; here a warp owns 4 query rows, its 32 lanes score
// 32 keys of a shared-memory K/V tile in parallel, the tile max and the P
// broadcast go through warp shuffles, and lane l owns output columns
// l, l+32, ... of the running O.
#include "common.cuh"

#include <type_traits>

namespace sfb {

struct AttnSimtParams {
    const void* q; const void* k; const void* v; void* out;
    int64_t q_sb, q_sh, q_ss, k_sb, k_sh, k_ss, v_sb, v_sh, v_ss, o_sb, o_sh, o_ss;
    int32_t B, H, Hkv, Lq, Lk, D;
    int32_t causal;
    float   scale;
    const int32_t* kv_len;
    const uint8_t* key_mask;
    int64_t mask_sb;
    const void* amask;               // additive mask (element strides am_sb, am_ss; keys contiguous)
    int32_t am_dt;
    int64_t am_sb, am_ss;
};

namespace attn_simt {

constexpr int kWarps   = 4;
constexpr int kRowsPW  = 4;                   // query rows per warp
constexpr int kRowsCTA = kWarps * kRowsPW;    // 16
constexpr int kKeys    = 32;                  // keys per tile

template <typename T> __device__ __forceinline__ float ld(const T* p) { return static_cast<float>(*p); }
template <> __device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <> __device__ __forceinline__ float ld<__half>(const __half* p) { return __half2float(*p); }
template <typename T> __device__ __forceinline__ T cvt(float x) { return static_cast<T>(x); }
template <> __device__ __forceinline__ __nv_bfloat16 cvt<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half cvt<__half>(float x) { return __float2half_rn(x); }

template <typename T, int DP>
__global__ void __launch_bounds__(kWarps * 32)
attn_fwd_simt_kernel(const AttnSimtParams p) {
    constexpr int NC = DP / 32;                  // output columns per lane
    __shared__ float sQ[kRowsCTA][DP];
    __shared__ float sK[kKeys][DP + 1];
    __shared__ float sV[kKeys][DP];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.z, h = blockIdx.y;
    const int hk = h / (p.H / p.Hkv);
    const int q0 = blockIdx.x * kRowsCTA;
    const T* Q = static_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh;
    const T* K = static_cast<const T*>(p.k) + b * p.k_sb + hk * p.k_sh;
    const T* V = static_cast<const T*>(p.v) + b * p.v_sb + hk * p.v_sh;

    for (int i = tid; i < kRowsCTA * DP; i += blockDim.x) {
        const int r = i / DP, d = i % DP;
        const int qi = q0 + r;
        sQ[r][d] = (qi < p.Lq && d < p.D) ? ld<T>(Q + qi * p.q_ss + d) : 0.f;
    }

    int kend = p.Lk;
    if (p.kv_len != nullptr) kend = min(kend, max(0, p.kv_len[b]));
    if (p.causal) kend = min(kend, min(p.Lq, q0 + kRowsCTA));

    float m[kRowsPW], l[kRowsPW], o[kRowsPW][NC];
#pragma unroll
    for (int r = 0; r < kRowsPW; ++r) {
        m[r] = -INFINITY; l[r] = 0.f;
#pragma unroll
        for (int c = 0; c < NC; ++c) o[r][c] = 0.f;
    }

    for (int k0 = 0; k0 < kend; k0 += kKeys) {
        __syncthreads();
        for (int i = tid; i < kKeys * DP; i += blockDim.x) {
            const int r = i / DP, d = i % DP;
            const int kj = k0 + r;
            const bool in = kj < kend && d < p.D;
            sK[r][d] = in ? ld<T>(K + kj * p.k_ss + d) : 0.f;
            sV[r][d] = in ? ld<T>(V + kj * p.v_ss + d) : 0.f;
        }
        __syncthreads();

        const int kj = k0 + lane;
        bool kvalid = kj < kend;
        if (kvalid && p.key_mask != nullptr) kvalid = p.key_mask[b * p.mask_sb + kj] != 0;
#pragma unroll
        for (int r = 0; r < kRowsPW; ++r) {
            const int row = warp * kRowsPW + r;
            const int qi = q0 + row;
            float s = 0.f;
#pragma unroll 8
            for (int d = 0; d < DP; ++d) s = fmaf(sQ[row][d], sK[lane][d], s);
            s *= p.scale;
            const bool valid = kvalid && (!p.causal || kj <= qi);
            if (valid && p.amask != nullptr && qi < p.Lq)
                s += attn_mask_at(p.amask, p.am_dt, b * p.am_sb + qi * p.am_ss + kj);
            if (!valid) s = -INFINITY;
            float tmax = s;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
            const float mnew = fmaxf(m[r], tmax);
            const float muse = mnew == -INFINITY ? 0.f : mnew;
            const float alpha = expf(m[r] - muse);
            const float pk = valid ? expf(s - muse) : 0.f;
            l[r] = l[r] * alpha + pk;         // per-lane partial, reduced at the end
            m[r] = mnew;
#pragma unroll
            for (int c = 0; c < NC; ++c) o[r][c] *= alpha;
#pragma unroll 4
            for (int kk = 0; kk < kKeys; ++kk) {
                const float pb = __shfl_sync(0xffffffffu, pk, kk);
#pragma unroll
                for (int c = 0; c < NC; ++c) o[r][c] = fmaf(pb, sV[kk][lane + 32 * c], o[r][c]);
            }
        }
    }

    T* O = static_cast<T*>(p.out) + b * p.o_sb + h * p.o_sh;
#pragma unroll
    for (int r = 0; r < kRowsPW; ++r) {
        float lt = l[r];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) lt += __shfl_xor_sync(0xffffffffu, lt, off);
        const int qi = q0 + warp * kRowsPW + r;
        if (qi >= p.Lq) continue;
        const float inv = lt > 0.f ? 1.f / lt : 0.f;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const int d = lane + 32 * c;
            if (d < p.D) O[qi * p.o_ss + d] = cvt<T>(o[r][c] * inv);
        }
    }
}

// Short key ranges (Lk <= kResKeys, the action self-attention's 67 keys):
// the whole K and V of the head are loaded into shared memory at once, every
// load in flight together, instead of one 32-key tile per round trip. Eight
// warps of two query rows each then compute every score of their rows (one
// key per lane and tile, independent FMA chains), the exact row maximum, the
// exponentials and P·V; with the keys resident no online rescaling is needed.
// (16 warps of one row measured slower: more shared-memory loads.)
constexpr int kResKeys  = 128;
constexpr int kResWarps = 8;
constexpr int kResRowsPW = 2;
constexpr int kResRows  = kResWarps * kResRowsPW;   // 16, as kRowsCTA

// K rows padded to dp + 4 floats: 16-byte aligned, and a warp's float4 loads
// of 32 consecutive rows hit distinct bank groups
__host__ __device__ constexpr int res_k_stride(int dp) { return dp + 4; }
__host__ __device__ constexpr int res_smem_floats(int dp, int lkp) {
    return kResRows * dp + lkp * res_k_stride(dp) + lkp * dp;
}

template <typename T, int DP>
__global__ void __launch_bounds__(kResWarps * 32)
attn_fwd_simt_res_kernel(const AttnSimtParams p, int lkp) {
    constexpr int NC = DP / 32;
    extern __shared__ float sres[];
    float* sQ = sres;                                  // [16][DP]
    constexpr int KS = res_k_stride(DP);
    float* sK = sQ + kResRows * DP;                    // [lkp][KS]
    float* sV = sK + lkp * KS;                         // [lkp][DP]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.z, h = blockIdx.y;
    const int hk = h / (p.H / p.Hkv);
    const int q0 = blockIdx.x * kResRows;
    const T* Q = static_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh;
    const T* K = static_cast<const T*>(p.k) + b * p.k_sb + hk * p.k_sh;
    const T* V = static_cast<const T*>(p.v) + b * p.v_sb + hk * p.v_sh;

    int kend = p.Lk;
    if (p.kv_len != nullptr) kend = min(kend, max(0, p.kv_len[b]));
    if (p.causal) kend = min(kend, min(p.Lq, q0 + kResRows));
    const int ntile = (kend + kKeys - 1) / kKeys;
    const int nkeys = ntile * kKeys;                   // <= lkp

    // Q, K and V of the head: fp32 rows of exactly DP contiguous, 16-byte
    // aligned values go as float4 loads, all issued before the first store
    // (one memory latency); anything else element-wise.
    bool vec = false;
    if constexpr (std::is_same<T, float>::value && DP == 64) {
        vec = p.D == DP && ((p.q_ss | p.k_ss | p.v_ss) & 3) == 0 &&
              ((reinterpret_cast<uintptr_t>(Q) | reinterpret_cast<uintptr_t>(K) |
                reinterpret_cast<uintptr_t>(V)) & 15) == 0;
    }
    if (vec) {
        if constexpr (std::is_same<T, float>::value && DP == 64) {
            constexpr int kV = DP / 4;                             // float4 per row
            constexpr int kMax = ((kResRows + 2 * kResKeys) * kV + kResWarps * 32 - 1) / (kResWarps * 32);
            const int nq = kResRows * kV, nk = nkeys * kV, total = nq + 2 * nk;
            float4 buf[kMax];
#pragma unroll
            for (int it = 0; it < kMax; ++it) {
                const int i = tid + it * kResWarps * 32;
                float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
                if (i < nq) {
                    const int r = i / kV, c = i % kV;
                    if (q0 + r < p.Lq) x = *reinterpret_cast<const float4*>(Q + (q0 + r) * p.q_ss + 4 * c);
                } else if (i < total) {
                    const int j = i - nq, isv = j >= nk, jj = isv ? j - nk : j;
                    const int r = jj / kV, c = jj % kV;
                    if (r < kend)
                        x = *reinterpret_cast<const float4*>((isv ? V + r * p.v_ss : K + r * p.k_ss) + 4 * c);
                }
                buf[it] = x;
            }
#pragma unroll
            for (int it = 0; it < kMax; ++it) {
                const int i = tid + it * kResWarps * 32;
                const float4 x = buf[it];
                if (i < nq) {
                    *reinterpret_cast<float4*>(sQ + i * 4) = x;
                } else if (i < total) {
                    const int j = i - nq, isv = j >= nk, jj = isv ? j - nk : j;
                    const int r = jj / kV, c = jj % kV;
                    if (isv) {
                        *reinterpret_cast<float4*>(sV + r * DP + 4 * c) = x;
                    } else {
                        *reinterpret_cast<float4*>(sK + r * KS + 4 * c) = x;
                    }
                }
            }
        }
    } else {
#pragma unroll 4
    for (int i = tid; i < kResRows * DP; i += blockDim.x) {
        const int r = i / DP, d = i % DP;
        const int qi = q0 + r;
        sQ[r * DP + d] = (qi < p.Lq && d < p.D) ? ld<T>(Q + qi * p.q_ss + d) : 0.f;
    }
#pragma unroll 4
    for (int i = tid; i < nkeys * DP; i += blockDim.x) {
        const int r = i / DP, d = i % DP;
        const bool in = r < kend && d < p.D;
        sK[r * KS + d] = in ? ld<T>(K + r * p.k_ss + d) : 0.f;
        sV[r * DP + d] = in ? ld<T>(V + r * p.v_ss + d) : 0.f;
    }
    }
    __syncthreads();

    // Every score of the warp's two rows first (one key per lane and tile:
    // up to 4 tiles x 2 rows of independent FMA chains), then the exact row
    // maximum, the exponentials and P·V: the key range is resident, so no
    // online rescaling is needed.
    constexpr int kT = kResKeys / kKeys;               // 4
    float sc[kResRowsPW][kT];
#pragma unroll
    for (int r = 0; r < kResRowsPW; ++r)
#pragma unroll
        for (int t = 0; t < kT; ++t) sc[r][t] = 0.f;
#pragma unroll 2
    for (int d4 = 0; d4 < DP / 4; ++d4) {
        float4 qv[kResRowsPW];
#pragma unroll
        for (int r = 0; r < kResRowsPW; ++r)
            qv[r] = reinterpret_cast<const float4*>(sQ + (warp * kResRowsPW + r) * DP)[d4];
#pragma unroll
        for (int t = 0; t < kT; ++t) {
            if (t >= ntile) break;
            const float4 kv = reinterpret_cast<const float4*>(sK + (t * kKeys + lane) * KS)[d4];
#pragma unroll
            for (int r = 0; r < kResRowsPW; ++r) {
                sc[r][t] = fmaf(qv[r].x, kv.x, sc[r][t]); sc[r][t] = fmaf(qv[r].y, kv.y, sc[r][t]);
                sc[r][t] = fmaf(qv[r].z, kv.z, sc[r][t]); sc[r][t] = fmaf(qv[r].w, kv.w, sc[r][t]);
            }
        }
    }
    float l[kResRowsPW], o[kResRowsPW][NC];
    float pk[kResRowsPW][kT];
#pragma unroll
    for (int r = 0; r < kResRowsPW; ++r) {
        const int qi = q0 + warp * kResRowsPW + r;
        float mx = -INFINITY;
#pragma unroll
        for (int t = 0; t < kT; ++t) {
            float s = -INFINITY;
            if (t < ntile) {
                const int kj = t * kKeys + lane;
                bool valid = kj < kend && (!p.causal || kj <= qi);
                if (valid && p.key_mask != nullptr) valid = p.key_mask[b * p.mask_sb + kj] != 0;
                if (valid) {
                    s = sc[r][t] * p.scale;
                    if (p.amask != nullptr && qi < p.Lq)
                        s += attn_mask_at(p.amask, p.am_dt, b * p.am_sb + qi * p.am_ss + kj);
                }
            }
            sc[r][t] = s;
            mx = fmaxf(mx, s);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        const float muse = mx == -INFINITY ? 0.f : mx;
        l[r] = 0.f;
#pragma unroll
        for (int t = 0; t < kT; ++t) {
            pk[r][t] = sc[r][t] == -INFINITY ? 0.f : expf(sc[r][t] - muse);
            l[r] += pk[r][t];
        }
#pragma unroll
        for (int c = 0; c < NC; ++c) o[r][c] = 0.f;
    }
#pragma unroll
    for (int t = 0; t < kT; ++t) {
        if (t >= ntile) break;
        const float* vt = sV + t * kKeys * DP;
#pragma unroll 4
        for (int kk = 0; kk < kKeys; ++kk) {
            float pb[kResRowsPW];
#pragma unroll
            for (int r = 0; r < kResRowsPW; ++r) pb[r] = __shfl_sync(0xffffffffu, pk[r][t], kk);
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const float vv = vt[kk * DP + lane + 32 * c];
#pragma unroll
                for (int r = 0; r < kResRowsPW; ++r) o[r][c] = fmaf(pb[r], vv, o[r][c]);
            }
        }
    }

    T* O = static_cast<T*>(p.out) + b * p.o_sb + h * p.o_sh;
#pragma unroll
    for (int r = 0; r < kResRowsPW; ++r) {
        float lt = l[r];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) lt += __shfl_xor_sync(0xffffffffu, lt, off);
        const int qi = q0 + warp * kResRowsPW + r;
        if (qi >= p.Lq) continue;
        const float inv = lt > 0.f ? 1.f / lt : 0.f;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const int d = lane + 32 * c;
            if (d < p.D) O[qi * p.o_ss + d] = cvt<T>(o[r][c] * inv);
        }
    }
}

}  // namespace attn_simt

template <typename T, int DP>
static int launch_simt_res(const AttnSimtParams& p, cudaStream_t stream) {
    using namespace attn_simt;
    const int lkp = (p.Lk + kKeys - 1) / kKeys * kKeys;
    const size_t smem = static_cast<size_t>(res_smem_floats(DP, lkp)) * 4;
    static bool attr_set[64] = {};                     // per device: the maximum is constant
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        const cudaError_t e = cudaFuncSetAttribute(attn_fwd_simt_res_kernel<T, DP>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   res_smem_floats(DP, kResKeys) * 4);
        if (e != cudaSuccess) { record_cuda_error(e, "attention smem attribute"); return SFB_ERR_CUDA; }
        attr_set[dev & 63] = true;
    }
    dim3 grid((p.Lq + kResRows - 1) / kResRows, p.H, p.B);
    attn_fwd_simt_res_kernel<T, DP><<<grid, kResWarps * 32, smem, stream>>>(p, lkp);
    return launch_status();
}

template <typename T>
static int launch_simt_t(const AttnSimtParams& p, cudaStream_t stream) {
    if (p.Lk <= attn_simt::kResKeys) {
        if (p.D <= 32) return launch_simt_res<T, 32>(p, stream);
        if (p.D <= 64) return launch_simt_res<T, 64>(p, stream);
        return launch_simt_res<T, 128>(p, stream);
    }
    dim3 grid((p.Lq + attn_simt::kRowsCTA - 1) / attn_simt::kRowsCTA, p.H, p.B);
    dim3 block(attn_simt::kWarps * 32);
    if (p.D <= 32)
        attn_simt::attn_fwd_simt_kernel<T, 32><<<grid, block, 0, stream>>>(p);
    else if (p.D <= 64)
        attn_simt::attn_fwd_simt_kernel<T, 64><<<grid, block, 0, stream>>>(p);
    else
        attn_simt::attn_fwd_simt_kernel<T, 128><<<grid, block, 0, stream>>>(p);
    return launch_status();
}

int attention_simt_launch(const sfb_attn_args& a, cudaStream_t stream) {
    if (a.head_dim > 128) return SFB_ERR_SHAPE;
    AttnSimtParams p{};
    p.q = a.q; p.k = a.k; p.v = a.v; p.out = a.out;
    p.q_sb = a.q_stride[0]; p.q_sh = a.q_stride[1]; p.q_ss = a.q_stride[2];
    p.k_sb = a.k_stride[0]; p.k_sh = a.k_stride[1]; p.k_ss = a.k_stride[2];
    p.v_sb = a.v_stride[0]; p.v_sh = a.v_stride[1]; p.v_ss = a.v_stride[2];
    p.o_sb = a.out_stride[0]; p.o_sh = a.out_stride[1]; p.o_ss = a.out_stride[2];
    p.B = a.batch; p.H = a.heads; p.Hkv = a.heads_kv; p.Lq = a.seq_q; p.Lk = a.seq_k; p.D = a.head_dim;
    p.causal = a.is_causal ? 1 : 0;
    p.scale = a.scale == 0.f ? 1.f / sqrtf(static_cast<float>(a.head_dim)) : a.scale;
    p.kv_len = a.kv_len; p.key_mask = a.key_mask; p.mask_sb = a.key_mask_stride_b;
    p.amask = a.attn_mask; p.am_dt = a.attn_mask_dtype;
    p.am_sb = a.attn_mask_stride[0]; p.am_ss = a.attn_mask_stride[1];
    switch (a.dtype) {
        case SFB_F32:  return launch_simt_t<float>(p, stream);
        case SFB_F16:  return launch_simt_t<__half>(p, stream);
        case SFB_BF16: return launch_simt_t<__nv_bfloat16>(p, stream);
        default:       return SFB_ERR_DTYPE;
    }
}

}  // namespace sfb
