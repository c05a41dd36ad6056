/*
 * sfb200.h — C ABI of the B200-native servoflow attention path.
 *
 * Every entry point takes plain device pointers, sizes and an opaque
 * cudaStream_t (passed as void*), returns an int status (0 = OK, negative =
 * error, never throws) and never allocates device memory on the hot path.
 * The reference's C++ CUDABackend binds these in place of its own ops (its
 * attention, dequantize and graph hooks forward to the functions below).
 *
 * dtype codes are the numeric values of sf::DType in the reference
 * (include/servoflow/core/dtype.h:11-19), so a caller can pass
 * static_cast<int>(tensor.dtype()) straight through.
 */
#ifndef SFB200_H
#define SFB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ── status codes ─────────────────────────────────────────────────────────── */
#define SFB_OK                 0
#define SFB_ERR_INVALID       -1  /* null pointer / bad argument            */
#define SFB_ERR_DTYPE         -2  /* dtype not supported by this op         */
#define SFB_ERR_SHAPE         -3  /* inconsistent or unsupported shape      */
#define SFB_ERR_ALIGN         -4  /* pointer/stride alignment (TMA: 16 B)   */
#define SFB_ERR_WORKSPACE     -5  /* workspace missing or too small         */
#define SFB_ERR_LAUNCH        -6  /* kernel launch failed                   */
#define SFB_ERR_UNSUPPORTED   -7  /* no sm_100a device / feature missing    */
#define SFB_ERR_CUDA          -8  /* other CUDA runtime error               */
#define SFB_ERR_DEVICE_TIMEOUT -9 /* a bounded device-side wait expired     */
#define SFB_ERR_RANGE        -10  /* input outside the kernel's value range */
#define SFB_ERR_IO           -11  /* file missing, unreadable or malformed  */

/* ── dtype codes (== sf::DType, reference dtype.h:11-19) ──────────────────── */
#define SFB_F32   0
#define SFB_F16   1
#define SFB_BF16  2
#define SFB_I8    3
#define SFB_I32   5
#define SFB_BOOL  6

/* Human-readable message for a status code (static string). */
const char* sfb_status_string(int status);

/* Text of the last CUDA error this library saw on the calling thread
 * ("" if none): the detail behind SFB_ERR_LAUNCH / SFB_ERR_CUDA. */
const char* sfb_last_error(void);

/* Library version string, e.g. "0.1.0 sm_100a". */
const char* sfb_version(void);

/* Reads (and with reset != 0 clears) the device-side error word that bounded
 * waits inside the kernels set when they time out. *code = 0 means no error.
 * Synchronous: it waits for the device. */
int sfb_device_error(int* code, int reset);

/* Diagnostic of the kernels' failure path: one warp waits, with the bounded
 * mbarrier wait every kernel uses, on a barrier that nothing arrives at. The
 * wait gives up after timeout_ns (1e5 .. 2e9), the kernel records
 * SFB_ERR_DEVICE_TIMEOUT in the device error word (read it with
 * sfb_device_error) and returns, and the context stays usable. *completed = 0
 * when the wait gave up as it must, 1 if it completed. Synchronous. */
int sfb_selftest_bounded_wait(int64_t timeout_ns, int32_t* completed);

/* Synchronous copy between any two addresses (cudaMemcpyDefault); a helper
 * for hosts without their own CUDA runtime binding (tests read parameters). */
int sfb_copy_device(void* dst, const void* src, int64_t bytes);

/* ── attention ────────────────────────────────────────────────────────────────
 * Replaces IBackend::attention (reference include/servoflow/backend/backend.h:
 * 102-110) as implemented by CUDABackend::attention
 * (src/backend/cuda/cuda_backend.cu:470-501) → cuda_ops::flash_attention
 * (src/backend/cuda/ops/attention.cu:183-197).
 *
 *   out[b,h,i,:] = softmax_j( scale · q[b,h,i,:]·k[b,hk,j,:] + mask ) · v[b,hk,j,:]
 *
 * - Layout: the last (head_dim) dimension is contiguous; the other three
 *   dimensions are addressed by element strides, so BHSD (the reference's
 *   layout) and BSHD (a fused projection's layout) both work without copies.
 * - scale == 0 means 1/sqrt(head_dim) (reference attention.cu:41,150).
 * - is_causal: key j is visible to query i iff j <= i (reference
 *   attention.cu:117, top-left aligned like torch SDPA).
 * - kv_len (optional, int32 [batch], device): keys j >= kv_len[b] are masked.
 * - key_mask (optional, uint8/bool [batch, seq_k], device, row stride
 *   key_mask_stride_b elements): key j of batch b is kept iff the byte is
 *   nonzero, masked (logit −inf) otherwise. This is the [B, Sk] key-padding
 *   convention of the reference model (include/servoflow/models/rdt1b/
 *   dit_block.h:141,153); the reference backend ignores masks
 *   (attention.cu:30), this one applies them.
 * - attn_mask (optional, device): the additive float mask of the reference's
 *   interface, [B, 1, Sq, Sk] (ops/attention.h:16, backend.h:104; the
 *   reference's Octo passes one, octo.cpp:79,209): the logit of (b, h, i, j)
 *   becomes scale·q·k + attn_mask[b·attn_mask_stride[0] + i·attn_mask_stride[1] + j],
 *   keys contiguous. A stride of 0 broadcasts that dimension ([1, 1, Sq, Sk],
 *   [B, 1, 1, Sk]). attn_mask_dtype: SFB_F32, SFB_F16 or SFB_BF16; -inf masks a
 *   key. It combines with kv_len, key_mask and is_causal. The base address and
 *   the non-zero strides need no alignment.
 * - A query row whose keys are all masked produces zeros (torch SDPA would
 *   produce NaN).
 * - heads % heads_kv == 0 (grouped K/V heads, as flash_attn::mha_fwd's H_k).
 * - dtype: SFB_BF16 / SFB_F16 (tcgen05 tensor-core kernel, head_dim 64) or
 *   SFB_F32 (SIMT kernel, head_dim <= 128). q, k, v, out share the dtype,
 *   except that v_dtype = SFB_F16 with dtype SFB_BF16 takes V in fp16.
 * - Tensor-core path: softmax in fp32; the probabilities and V enter the P·V
 *   product as fp16 (bf16 V is converted exactly in shared memory). bf16 V
 *   entries beyond the fp16 range (|v| > 65504) are not supported: the kernel
 *   then records SFB_ERR_RANGE in the device error word (sfb_device_error).
 */
typedef struct sfb_attn_args {
    const void* q;
    const void* k;
    const void* v;
    void*       out;
    int64_t q_stride[3];    /* element strides: batch, head, seq */
    int64_t k_stride[3];
    int64_t v_stride[3];
    int64_t out_stride[3];
    int32_t batch;
    int32_t heads;
    int32_t heads_kv;
    int32_t seq_q;
    int32_t seq_k;
    int32_t head_dim;
    int32_t dtype;
    int32_t is_causal;
    float   scale;
    const int32_t* kv_len;        /* optional */
    const uint8_t* key_mask;      /* optional */
    int64_t key_mask_stride_b;
    /* Number of key splits merged inside one thread-block cluster
     * (0 = choose automatically, else 1..16). Tuning knob only. */
    int32_t num_splits;
    int32_t v_dtype;        /* 0: V has `dtype`; SFB_F16 with dtype SFB_BF16: V is already
                               fp16 (a cache stored in the P·V operand type: no conversion) */
    int32_t attn_mask_dtype;      /* dtype of attn_mask (ignored when it is NULL) */
    const void* attn_mask;        /* optional additive mask, see above */
    int64_t attn_mask_stride[2];  /* element strides: batch, query row (0 = broadcast) */
} sfb_attn_args;

int sfb_attention_fwd(const sfb_attn_args* args, void* stream);

/* Convenience wrapper for contiguous BHSD tensors — the exact argument list
 * of IBackend::attention with the Tensor metadata unpacked. mask may be NULL
 * or a [batch, seq_k] byte key-padding mask. */
int sfb_attention_bhsd(const void* q, const void* k, const void* v, void* out,
                       int32_t batch, int32_t heads, int32_t heads_kv,
                       int32_t seq_q, int32_t seq_k, int32_t head_dim,
                       int32_t dtype, const uint8_t* key_mask, float scale,
                       int32_t is_causal, void* stream);

/* ── int8 dequantisation ──────────────────────────────────────────────────────
 * Replaces IBackend::dequantize (backend.h:201-206) → CUDABackend::dequantize
 * (cuda_backend.cu:565-569) → cuda_ops::dequantize_int8
 * (src/backend/cuda/ops/quantization.cu:53-95).
 *   out[n,k] = in[n,k] · scale[n]   (per output channel, scale_numel == rows)
 *   out[n,k] = in[n,k] · scale[0]   (per tensor, scale_numel == 1)
 * scale_dtype: SFB_F16 (the reference's only accepted type) or SFB_F32.
 * out_dtype:   SFB_F16 (reference behaviour: the product is rounded to fp16,
 *              quantization.cu:44), SFB_BF16 or SFB_F32.
 */
int sfb_dequantize_int8(const int8_t* in, const void* scale, int32_t scale_dtype,
                        int64_t scale_numel, void* out, int32_t out_dtype,
                        int64_t rows, int64_t cols, void* stream);

/* ── int8-weight linear layer (dequantisation fused into the GEMM) ─────────────
 * Replaces, for the RDT-1B projections (Q/K/V/O, MLP fc1/fc2), the pair
 * IBackend::dequantize (backend.h:201-206, quantization.cu:18-95) followed by
 * IBackend::gemm_bias_act (backend.h:160-185, cuda_backend.cu:337-467):
 *
 *   y[m,n] = act( w_scale[n] · Σ_k x[m,k]·w[n,k] + bias[n] ) + residual[m,n]
 *
 * x: bf16 [M, K], row stride ldx (elements, ldx·2 a multiple of 16 bytes);
 * w: int8 [N, K] row-major, contiguous (one row per output channel);
 * w_scale: fp32 [N]; bias: bf16 [N] or NULL; residual: [M, N] in y_dtype with
 * row stride ldr, or NULL (may alias y); y: y_dtype (SFB_BF16 or SFB_F32) [M, N]
 * with row stride ldy. act: 0 none, 1 GELU (tanh form, as the reference's
 * cuBLASLt GELU epilogue and the RDT-1B MLPs use), 2 SiLU (timestep MLP). K % 64 == 0, N % 32 == 0.
 * num_splits: split-K cluster size for M <= 128: 1, 2, 4 or 8 (0 = automatic).
 * The result equals dequantise-then-GEMM up to fp32 summation order.
 */
int sfb_w8a16_linear(const void* x, int64_t ldx, const int8_t* w, const float* w_scale,
                     const void* bias, const void* residual, int64_t ldr, void* y, int64_t ldy,
                     int32_t y_dtype, int32_t M, int32_t N, int32_t K, int32_t act,
                     int32_t num_splits, void* stream);

/* ── two int8-weight linear layers as one launch (one session) ────────────────
 * Replaces, for a block's MLP at one session (Mlp::forward, reference
 * src/models/rdt1b/dit_block.cu:143-163: fc1 → GELU → fc2), the pair of
 * dequantize + gemm_bias_act calls of each layer (quantization.cu:18-95,
 * cuda_backend.cu:337-467):
 *
 *   h = act( x · (w1 · s1)ᵀ + b1 )          (bf16 [M, F], in the workspace)
 *   y = h · (w2 · s2)ᵀ + b2 [+ residual]    (y_dtype [M, N]; residual in y_dtype, may alias y)
 *
 * run as two stages of the persistent projection kernel, ordered on the device
 * (no kernel boundary between them). x: bf16 [M, K] (row stride ldx); w1:
 * int8 [F, K], w2: int8 [N, F], row-major; s1, s2: fp32 per output channel;
 * b1, b2: bf16 or NULL. act: 0 none, 1 GELU (tanh), 2 SiLU. M <= 80;
 * K and F multiples of 256 and at most 2048; F and N multiples of 64.
 * workspace: device memory of at least sfb_w8a16_mlp_workspace_bytes(M, F)
 * bytes, 256-byte aligned; it holds the stage counters (cleared by every
 * call) and h. Calls that share a workspace must not overlap on the GPU.
 * The result equals two sfb_w8a16_linear calls up to fp32 summation order. */
size_t sfb_w8a16_mlp_workspace_bytes(int32_t M, int32_t F);
int sfb_w8a16_mlp(const void* x, int64_t ldx, const int8_t* w1, const float* s1, const void* b1,
                  const int8_t* w2, const float* s2, const void* b2, const void* residual, int64_t ldr,
                  void* y, int64_t ldy, int32_t y_dtype, int32_t M, int32_t K, int32_t F, int32_t N,
                  int32_t act, void* workspace, size_t workspace_bytes, void* stream);

/* sfb_w8a16_mlp without a workspace: no counterpart in the reference. For
 * callers that cannot allocate device memory where they run the MLP (a
 * real-time loop that forbids cudaMalloc after start-up, a framework whose
 * allocator owns all device memory, a plugin handed only its inputs and
 * outputs). Its scratch (the stage counters and h) is a fixed array inside
 * this library, sfb_w8a16_mlp_noalloc_max_bytes() bytes (about 320 KB: M·F <=
 * 163840, e.g. M = 80 with F = 2048), which every GPU that loads the library
 * holds until the process exits. Larger M·F return SFB_ERR_WORKSPACE with a
 * message in sfb_last_error. The call allocates nothing: it clears the
 * counters with cudaMemsetAsync on `stream` and launches. Every call shares
 * the one array, so calls that overlap on the GPU (other streams, other
 * threads) race; serialise them. The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress, once per device, with that
 * device current); make that first call before any stream capture.
 * Arguments and result as sfb_w8a16_mlp. */
size_t sfb_w8a16_mlp_noalloc_max_bytes(void);
int sfb_w8a16_mlp_noalloc(const void* x, int64_t ldx, const int8_t* w1, const float* s1, const void* b1,
                          const int8_t* w2, const float* s2, const void* b2, const void* residual, int64_t ldr,
                          void* y, int64_t ldy, int32_t y_dtype, int32_t M, int32_t K, int32_t F, int32_t N,
                          int32_t act, void* stream);

/* ── RDT-1B denoising runtime ──────────────────────────────────────────────────
 * The model-level path around the kernels above, replacing for RDT-1B the
 * reference's RDT1BModel::encode_condition / denoise_step
 * (src/models/rdt1b/rdt1b.cpp:167-369), RDTBlock / SelfAttention /
 * CrossAttention (dit_block.cu:198-387) and the CUDA-graph sampling loop of
 * FlowMatchingSampler::sample (src/sampling/flow_matching.cpp:25-93), with a
 * DPM-Solver++ (2M) sampler. Weights are seeded random values quantised to
 * int8 per output channel (the reference loads checkpoints; none is available).
 * All tensors are device memory; `sessions` independent robot sessions run
 * batched (1 <= sessions <= max_sessions).
 */
typedef struct sfb_rdt1b_config {
    int32_t num_layers;     /* 28 */
    int32_t hidden;         /* 2048 (= heads · 64) */
    int32_t heads;          /* 32 */
    int32_t action_dim;     /* 128 */
    int32_t horizon;        /* 64 action tokens */
    int32_t state_dim;      /* 128 (must equal action_dim) */
    int32_t lang_dim;       /* 4096 (T5-XXL features) */
    int32_t img_dim;        /* 1152 (SigLIP features) */
    int32_t max_lang_len;   /* 1024 */
    int32_t img_len;        /* 4374 */
    int32_t max_sessions;   /* batch capacity */
    int32_t num_steps;      /* 5 DPM-Solver++ steps */
    int32_t ctrl_freq;      /* 25 Hz */
    float   weight_std;     /* 0.02, std of the random weights before quantisation */
} sfb_rdt1b_config;

int sfb_rdt1b_default_config(sfb_rdt1b_config* cfg);
/* Allocates and initialises the model on the current device (setup-time
 * cudaMalloc; nothing allocates afterwards). */
int sfb_rdt1b_create(const sfb_rdt1b_config* cfg, uint64_t seed, void** handle);
int sfb_rdt1b_destroy(void* handle);
/* Per control tick: lang_tokens bf16 [sessions, max_lang_len, lang_dim],
 * lang_len int32 [sessions] (valid language tokens; the rest are masked),
 * img_tokens bf16 [sessions, img_len, img_dim], state bf16 [sessions,
 * state_dim]. Runs the adaptors and fills every block's cross-attention K/V
 * cache. */
int sfb_rdt1b_encode(void* handle, int32_t sessions, const void* lang_tokens, const int32_t* lang_len,
                     const void* img_tokens, const void* state, void* stream);
/* One network evaluation: x_t fp32 [sessions, horizon, action_dim] at timestep
 * t → x0 prediction fp32, same shape. */
int sfb_rdt1b_forward(void* handle, int32_t sessions, const float* x_t, float t, float* x0_out,
                      void* stream);
/* Full sampling: noise fp32 [sessions, horizon, action_dim] → actions (same
 * shape) after num_steps DPM-Solver++ steps. noise and actions may be device
 * pointers or host pointers (pinned host memory keeps the copies
 * asynchronous); the call returns once the work is queued on `stream`. With use_graph != 0 the loop is
 * captured into a CUDA graph on the first call for a given session count (that
 * call runs eagerly, then captures; make it before any capture of your own) and
 * replayed afterwards. */
int sfb_rdt1b_sample(void* handle, int32_t sessions, const float* noise, float* actions,
                     int32_t use_graph, void* stream);
/* One control tick of the inference engine: replaces InferenceEngine::infer
 * (src/engine/inference_engine.cpp:99-174) with its condition cache keyed by
 * a caller-supplied frame id (mark_new_frame, :90-93).
 * - When frame_id differs from the frame the K/V cache was built from (or
 *   the cache was invalidated, or `sessions` changed), the conditions are
 *   copied in and encoded (adaptors + every block's cross-attention K/V) on
 *   the model's encode stream, after the caller's prior work and the previous
 *   denoise, and an event orders the denoise after it. Otherwise lang_tokens,
 *   lang_len and img_tokens may be NULL and nothing is re-encoded.
 * - The robot state is copied every tick (the reference caches it with the
 *   condition, rdt1b.cpp:207-231; here each tick's actions see its state).
 * - Then sfb_rdt1b_sample(..., use_graph = 1): noise in, actions out.
 * Every buffer may be host memory (pinned keeps the copies asynchronous) or
 * device memory, with the shapes of sfb_rdt1b_encode / sfb_rdt1b_sample. The
 * first tick creates the encode stream and the device staging buffers of the
 * conditions (setup-time allocation, like create); later ticks allocate
 * nothing. Returns once the work is queued on `stream`. */
int sfb_rdt1b_tick(void* handle, int32_t sessions, uint64_t frame_id, const void* lang_tokens,
                   const int32_t* lang_len, const void* img_tokens, const void* state, const float* noise,
                   float* actions, void* stream);
/* Forces the next tick to re-encode (InferenceEngine::invalidate_condition_cache). */
int sfb_rdt1b_invalidate_condition(void* handle);
/* Ticks run and conditions encoded so far on this handle (diagnostic). */
int sfb_rdt1b_tick_stats(void* handle, int64_t* ticks, int64_t* encodes);
/* Execution path of a one-session call (sessions == 1): 0 runs the network
 * evaluation as stages of the persistent kernel (every projection,
 * self-attention and cross-attention, with the pre-norms folded into the
 * projections), in launches of up to 48 stages; 1 (the default, the fastest
 * measured) runs one kernel per projection, norm and attention (the path
 * every batch of two or more sessions takes); 2 runs the persistent kernel between separate
 * cross-attention kernels. Results agree within the model's tolerance, not
 * bit for bit. Changing it drops the captured graphs. No counterpart in the
 * reference. */
int sfb_rdt1b_set_path(void* handle, int32_t path);
/* Profiles one network evaluation of session 0 at timestep t on the
 * persistent-kernel path (path 0, whatever the handle's path): CUDA events
 * around each of its launches on `stream`. Writes the launch count to
 * *n_launches and, when max_launches is large enough, each launch's
 * algorithmic bytes (weights, scales and biases read, activations read and
 * written, the K/V rows the cross-attention reads: the language blocks' valid
 * keys only) and its duration in microseconds. Synchronises `stream`.
 * Diagnostic; no counterpart in the reference. */
int sfb_rdt1b_profile_dense(void* handle, float t, int32_t max_launches, int32_t* n_launches,
                            double* alg_bytes, float* us, void* stream);
/* Kernel launches in the captured sampling graph for `sessions` (known after
 * the first use_graph call for that session count). Diagnostic; no
 * counterpart in the reference. */
int sfb_rdt1b_graph_kernels(void* handle, int32_t sessions, int64_t* kernels);
/* Device pointer, element count and dtype of a named parameter (names follow
 * the reference checkpoint: "blocks.3.attn.qkv.weight_q", "...weight_scale",
 * "...bias", "x_pos_embed", ...). */
int sfb_rdt1b_param(void* handle, const char* name, void** ptr, int64_t* numel, int32_t* dtype);
/* The sampler's timesteps and per-step update x ← a·x + b·x0 + c·x0_prev. */
int sfb_rdt1b_schedule(void* handle, float* timesteps, float* coef_a, float* coef_b, float* coef_c,
                       int32_t n);

/* ── Octo policy (model path) ─────────────────────────────────────────────────
 * Replaces the reference's OctoModel / OctoBlock / OctoDiffusionHead
 * (include/servoflow/models/octo/octo.h:18-132, src/models/octo/octo.cpp) on
 * the same kernels: LayerNorm, the int8-weight linear layer, the tensor-core
 * attention. Weights are seeded random values quantised to int8 per output
 * channel (the reference's load_octo reads none, octo.cpp:247-260). All
 * tensors are device memory except where stated; `sessions` independent
 * robot sessions run batched (1 <= sessions <= max_sessions). */
typedef struct sfb_octo_config {
    int32_t num_layers;      /* 12 (OctoConfig, config.h:17-46) */
    int32_t hidden;          /* 384 (= heads · 64) */
    int32_t heads;           /* 6 */
    int32_t head_dim;        /* 64 (the only value supported) */
    int32_t intermediate;    /* 1536, multiple of 64 */
    int32_t action_dim;      /* 7 */
    int32_t action_horizon;  /* 4 */
    int32_t head_hidden;     /* 256, multiple of 64 */
    int32_t seq_len;         /* 64 backbone tokens (octo.cpp:202) */
    int32_t max_sessions;    /* batch capacity */
    int32_t num_steps;       /* 10 flow-matching steps (Schedule, sampler.h:24) */
    int32_t readout_token;   /* -1: the reference's readout, a 0.1 fill
                                (octo.cpp:218-223); k >= 0: backbone output token k */
    float   weight_std;      /* 0.02, std of the random weights before quantisation */
} sfb_octo_config;

int sfb_octo_default_config(sfb_octo_config* cfg);
int sfb_octo_create(const sfb_octo_config* cfg, uint64_t seed, void** handle);
int sfb_octo_destroy(void* handle);
/* OctoModel::encode_condition (octo.cpp:196-224): runs the backbone blocks
 * over tokens bf16 [sessions, seq_len, hidden] (NULL: the reference's 0.1
 * fill), writes the output tokens to `features` (optional, same shape) and
 * sets each session's condition per readout_token. */
int sfb_octo_encode(void* handle, int32_t sessions, const void* tokens, void* features, void* stream);
/* Sets the condition directly: context bf16 [sessions, hidden], as the
 * reference's tests pass it to denoise_step (tests/models/test_octo.cpp:30-45). */
int sfb_octo_set_condition(void* handle, int32_t sessions, const void* context, void* stream);
/* OctoModel::denoise_step (octo.cpp:226-238): x_t fp32 [sessions,
 * action_horizon, action_dim] → velocity fp32 (same shape) from the
 * diffusion head. t is accepted and, as in the reference, not used. */
int sfb_octo_denoise_step(void* handle, int32_t sessions, const float* x_t, float t, float* velocity,
                          void* stream);
/* FlowMatchingSampler::sample (src/sampling/flow_matching.cpp:25-93): noise
 * fp32 [sessions, action_horizon, action_dim] → actions after num_steps Euler
 * steps x ← x + (t_{i+1} − t_i)·v over linspace(1, 0, num_steps + 1). noise
 * and actions may be device or host pointers; the call returns once the work
 * is queued on `stream`. use_graph as sfb_rdt1b_sample. */
int sfb_octo_sample(void* handle, int32_t sessions, const float* noise, float* actions, int32_t use_graph,
                    void* stream);
/* The sampler's num_steps + 1 timesteps (host memory; n = num_steps + 1). */
int sfb_octo_timesteps(void* handle, float* timesteps, int32_t n);
/* Device pointer, element count and dtype of a parameter: "blocks.<l>.norm1.weight",
 * "...norm1.bias", "...attn.qkv.weight_q", "...weight_scale", "...bias",
 * "...attn.proj.*", "...norm2.*", "...mlp.fc1.*", "...mlp.fc2.*",
 * "head.fc1.*" ([head_hidden, K] with K = action_dim·action_horizon + 128 +
 * hidden rounded up to 64, zero columns past the valid width), "head.fc2.*",
 * "head.fc3.*" ([action_dim·action_horizon rounded up to 128, head_hidden],
 * zero rows past the valid count). */
int sfb_octo_param(void* handle, const char* name, void** ptr, int64_t* numel, int32_t* dtype);
/* Kernel launches in the captured sampling graph for `sessions`. */
int sfb_octo_graph_kernels(void* handle, int32_t sessions, int64_t* kernels);

/* ── checkpoints (setup time; host code except the uploads) ──────────────────
 * A tensor entry of a .safetensors file: replaces SafeTensorsLoader::TensorMeta
 * (reference include/servoflow/loader/safetensors.h:46-52). dtype is an SFB
 * code (4 = packed int4); offsets are relative to the data section. */
typedef struct sfb_tensor_info {
    char     name[256];
    int32_t  dtype;
    int32_t  ndim;
    int64_t  shape[8];
    uint64_t data_begin;
    uint64_t data_end;
} sfb_tensor_info;

/* Lists the tensors of a safetensors file sorted by name, without reading
 * their data: replaces SafeTensorsLoader::inspect (safetensors.h:53,
 * src/loader/safetensors.cpp:65-108). Writes min(capacity, *count) entries;
 * *count is the total; *data_offset (optional) = 8 + header length. Errors as
 * the reference's parse_header: SFB_ERR_IO for a short file, a header past the
 * end or malformed JSON; SFB_ERR_DTYPE for a dtype outside F32, F16, BF16, I8,
 * I4, I32, BOOL. Needs no GPU. */
int sfb_safetensors_inspect(const char* path, sfb_tensor_info* out, int32_t capacity, int32_t* count,
                            uint64_t* data_offset);
/* The reference converter's weight-name mapping (remap_key, tools/convert/
 * hf_to_servoflow.py:41-66): returns 1 and writes the ServoFlow name, or 0 for
 * an entry the converter drops (EMA shadows, optimizer/scheduler state, other
 * modules). Needs no GPU. */
int sfb_checkpoint_key(const char* hf_name, char* out, int32_t out_len);
/* Fills *cfg from a checkpoint's config.json (RDT1BConfig::from_json,
 * src/models/rdt1b/config.cpp:10-66: the converter's flat keys and the HF
 * nested "rdt"/"noise_scheduler" keys over the defaults). max_sessions stays 1.
 * SFB_ERR_UNSUPPORTED for num_train_timesteps != 1000, freq_dim != 256 or
 * rms_norm_eps != 1e-6, which this runtime fixes. Needs no GPU. */
int sfb_rdt1b_config_from_json(const char* path, sfb_rdt1b_config* cfg);
/* Writes the model parameters one safetensors file provides. Names are taken
 * as stored or mapped as sfb_checkpoint_key does. A float "<linear>.weight"
 * [N, K] is quantised on the device into "<linear>.weight_q" (int8) and
 * "<linear>.weight_scale" (fp32 [N]): s = max|row| / 127 (1 for a zero row),
 * q = clamp(round-half-even(w / s), -127, 127). Other tensors are copied, or
 * converted to the parameter's dtype (round-to-nearest-even), as
 * load_weight_from_map does (src/loader/safetensors.cpp:156-183). *loaded
 * counts the tensors written, *ignored the entries that name no parameter.
 * Allocates a staging buffer and synchronises the device: setup time only.
 * The K/V cache is stale until the next sfb_rdt1b_encode. */
int sfb_rdt1b_load_safetensors(void* handle, const char* path, int64_t* loaded, int64_t* ignored);
/* Loads every *.safetensors file of a checkpoint directory (name order; the
 * first file providing a parameter keeps it), as RDT1BModel::load_weights
 * (src/models/rdt1b/rdt1b.cpp:97-111). Fails (SFB_ERR_INVALID, message in
 * sfb_last_error) when a model parameter is missing from every file. */
int sfb_rdt1b_load_checkpoint(void* handle, const char* dir, int64_t* loaded, int64_t* ignored);
/* Parameters not written by any load since create (seeded values remain);
 * the first one's name goes to first_missing (optional). */
int sfb_rdt1b_params_missing(void* handle, int64_t* missing, char* first_missing, int32_t buflen);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* SFB200_H */
