/*
 * sfo_oracle.c — CPU restatement of the reference's hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker for the CUDA kernels in
 * servoflow_b200/csrc and the timed CPU baseline of bench.py; the product
 * path never links, loads or calls it. Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / --impl reference legs may use it.
 *
 * Pinning: the attention restatement is checked against golden vectors made
 * with the reference's own Python oracle (torch scaled_dot_product_attention
 * in math mode, tests/alignment/test_rdt1b_alignment.py:133-134,148-149) and
 * against the reference's fp32 CUDA kernel itself on the GPU box
 * (oracle/_ref); the dequant restatement against the known answers of
 * tests/unit/test_quantization.cpp:9-94.
 *
 * Build: oracle/Makefile → oracle/libsfo_oracle.so (gcc -O2 -fopenmp).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ── attention ───────────────────────────────────────────────────────────────
 * Follows the reference's fp32 kernel (src/backend/cuda/ops/attention.cu:
 * 90-139): per query row, an online softmax over the keys in order
 * (m, sum, acc recurrence of :111-134), then acc / sum (:136-138); scale 0
 * means 1/sqrt(D) (:150); causal stops at key > query (:117). Differences,
 * all deliberate: the recurrence runs in double; the key-padding mask and
 * kv_len (which the reference drops, attention.cu:30) are applied as −inf
 * logits, the torch SDPA boolean-mask convention of the reference's Python
 * oracle; a row with no visible key yields zeros (SDPA would give NaN);
 * K/V heads may be grouped (heads % heads_kv == 0). amask (optional) is the
 * additive float mask of IBackend::attention (ops/attention.h:16), expanded
 * to [B, Lq, Lk]: it is added to the scaled logit, as torch SDPA adds a float
 * attn_mask; a -inf entry drops the key.
 * Layout: contiguous [B, H, L, D] float arrays.
 */
void sfo_attention(const float* q, const float* k, const float* v, float* out,
                   int B, int H, int Hkv, int Lq, int Lk, int D, float scale,
                   int causal, const int32_t* kv_len, const uint8_t* key_mask,
                   int nthreads, const float* amask) {
    if (scale == 0.f) scale = 1.f / sqrtf((float)D);
    const int64_t rows = (int64_t)B * H * Lq;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 4) num_threads(nthreads)
#endif
    for (int64_t r = 0; r < rows; ++r) {
        const int qi = (int)(r % Lq);
        const int h = (int)((r / Lq) % H);
        const int b = (int)(r / ((int64_t)Lq * H));
        const int hk = h / (H / Hkv);
        const float* qr = q + r * D;
        const float* kb = k + ((int64_t)b * Hkv + hk) * (int64_t)Lk * D;
        const float* vb = v + ((int64_t)b * Hkv + hk) * (int64_t)Lk * D;
        double acc[256];
        double m = -INFINITY, sum = 0.0;
        for (int d = 0; d < D; ++d) acc[d] = 0.0;
        int kend = Lk;
        if (kv_len) kend = kv_len[b] < kend ? (kv_len[b] < 0 ? 0 : kv_len[b]) : kend;
        for (int j = 0; j < kend; ++j) {
            if (causal && j > qi) break;
            if (key_mask && !key_mask[(int64_t)b * Lk + j]) continue;
            double dot = 0.0;
            for (int d = 0; d < D; ++d) dot += (double)qr[d] * (double)kb[(int64_t)j * D + d];
            dot *= (double)scale;
            if (amask) {
                dot += (double)amask[((int64_t)b * Lq + qi) * Lk + j];
                if (isinf(dot) && dot < 0) continue;
            }
            const double mn = dot > m ? dot : m;
            const double e_old = exp(m - mn);   /* m = -inf on the first key → 0 */
            const double e_new = exp(dot - mn);
            for (int d = 0; d < D; ++d) acc[d] = acc[d] * e_old + e_new * (double)vb[(int64_t)j * D + d];
            sum = sum * e_old + e_new;
            m = mn;
        }
        float* o = out + r * D;
        for (int d = 0; d < D; ++d) o[d] = sum > 0.0 ? (float)(acc[d] / sum) : 0.f;
    }
}

/* ── fp16 / bf16 rounding (round to nearest even), for dequant semantics ─── */
static float f32_round_to_f16(float x) {
    /* exact RNE to IEEE binary16, returned as float */
    if (isnan(x) || isinf(x)) return x;
    const float ax = fabsf(x);
    if (ax >= 65520.f) return x > 0 ? INFINITY : -INFINITY;
    int e;
    frexpf(ax, &e);                 /* ax = f · 2^e, f in [0.5, 1) */
    int ulp_exp = e - 11;           /* 11 significant bits */
    if (ulp_exp < -24) ulp_exp = -24; /* subnormal spacing 2^-24 */
    const float ulp = ldexpf(1.f, ulp_exp);
    const float rq = nearbyintf(ax / ulp) * ulp;   /* default rounding mode is RNE */
    return x < 0 ? -rq : rq;
}

float sfo_round_f16(float x) { return f32_round_to_f16(x); }

float sfo_round_bf16(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) return x;
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
    float r;
    memcpy(&r, &u, 4);
    return r;
}

/* ── int8 dequantisation ─────────────────────────────────────────────────────
 * Follows src/backend/cuda/ops/quantization.cu:18-95: out[n,k] = q[n,k]·s[n]
 * (per output channel, scale_numel == rows) or q·s[0] (per tensor). With
 * round_mode 1 the product is rounded to fp16 as the reference's
 * __hmul(__int2half_rn(q), s) does (:44); 2 rounds to bf16; 0 keeps fp32.
 */
void sfo_dequant_int8(const int8_t* in, const float* scale, int64_t scale_numel, float* out,
                      int64_t rows, int64_t cols, int round_mode) {
    for (int64_t r = 0; r < rows; ++r) {
        const float s = scale[scale_numel == 1 ? 0 : r];
        for (int64_t c = 0; c < cols; ++c) {
            float y = (float)in[r * cols + c] * s;
            if (round_mode == 1) y = f32_round_to_f16(y);
            else if (round_mode == 2) y = sfo_round_bf16(y);
            out[r * cols + c] = y;
        }
    }
}

int sfo_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ── int8-weight linear layer ────────────────────────────────────────────────
 * The reference computes this in two steps: dequantise the weight,
 * w[n,k] = q[n,k]·s[n] (src/backend/cuda/ops/quantization.cu:18-51), then
 * gemm_bias_act (src/backend/cuda/cuda_backend.cu:337-467):
 *   y[m,n] = act( Σ_k x[m,k]·w[n,k] + bias[n] ) + residual[m,n]
 * with act = GELU in its tanh form (the RDT-1B MLPs, F.gelu(approximate="tanh")
 * in tests/alignment/test_rdt1b_alignment.py:104,119). Evaluated in double.
 * bias / residual may be NULL.
 */
void sfo_w8a16_linear(const float* x, const int8_t* q, const float* s, const float* bias,
                      const float* residual, float* y, int M, int N, int K, int act,
                      int nthreads) {
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(nthreads)
#endif
    for (int64_t mn = 0; mn < (int64_t)M * N; ++mn) {
        const int m = (int)(mn / N), n = (int)(mn % N);
        double acc = 0.0;
        for (int k = 0; k < K; ++k) acc += (double)x[(int64_t)m * K + k] * (double)q[(int64_t)n * K + k];
        double v = acc * (double)s[n] + (bias ? (double)bias[n] : 0.0);
        if (act == 1) v = 0.5 * v * (1.0 + tanh(0.7978845608028654 * (v + 0.044715 * v * v * v)));
        else if (act == 2) v = v / (1.0 + exp(-v));
        if (residual) v += (double)residual[mn];
        y[mn] = (float)v;
    }
}
