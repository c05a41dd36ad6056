// dense_noalloc.cu — sfb_w8a16_mlp_noalloc: the two-layer int8-weight MLP of
// sfb_w8a16_mlp without a caller-provided workspace.
//
// Some callers cannot allocate device memory at the point where they run the
// MLP: a real-time control loop that forbids cudaMalloc after start-up, a
// host framework whose allocator owns all device memory and exposes no
// scratch API, a plugin that only receives its inputs and outputs. For them
// the scratch the kernel needs (its stage counters and the hidden activation
// h) lives in one file-scope __device__ array of this library, which every GPU
// that loads the library holds until the process exits.
#include "common.cuh"

namespace sfb {

// Scratch of the no-allocation MLP: the stage counters, then h [M, F] bf16.
// Sized for M <= 80 tokens and F <= 2048 (80 · 2048 · 2 B = 320 KB).
constexpr size_t kNoAllocScratchBytes = 256 + 80 * 2048 * 2;
static __device__ __align__(256) uint8_t g_mlp_noalloc_scratch[kNoAllocScratchBytes];

size_t w8a16_mlp_workspace_bytes(int M, int F);
int w8a16_mlp_launch(const void* x, int64_t ldx, const int8_t* w1, const float* s1, const void* b1,
                     const int8_t* w2, const float* s2, const void* b2, const void* residual, int64_t ldr,
                     void* y, int64_t ldy, int32_t y_dtype, int32_t M, int32_t K, int32_t F, int32_t N,
                     int32_t act, void* workspace, size_t workspace_bytes, cudaStream_t stream);

// Device address of the scratch array on the current device. In host code the
// array's name is only a host-side stand-in, so the address is looked up once
// per device (cudaGetSymbolAddress, with that device current) and cached.
static int noalloc_scratch(void** out) {
    static std::mutex mu;
    static void* addr[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { record_cuda_error(e, "no-alloc scratch: current device"); return SFB_ERR_CUDA; }
    std::lock_guard<std::mutex> lk(mu);
    void*& slot = addr[dev & 63];
    if (slot == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_mlp_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            record_cuda_error(e != cudaSuccess ? e : cudaErrorInvalidSymbol, "no-alloc scratch address");
            return SFB_ERR_CUDA;
        }
        slot = p;
    }
    *out = slot;
    return SFB_OK;
}

}  // namespace sfb

extern "C" {

size_t sfb_w8a16_mlp_noalloc_max_bytes(void) { return sfb::kNoAllocScratchBytes; }

int sfb_w8a16_mlp_noalloc(const void* x, int64_t ldx, const int8_t* w1, const float* s1, const void* b1,
                          const int8_t* w2, const float* s2, const void* b2, const void* residual, int64_t ldr,
                          void* y, int64_t ldy, int32_t y_dtype, int32_t M, int32_t K, int32_t F, int32_t N,
                          int32_t act, void* stream) {
    if (M < 1 || F < 1) return SFB_ERR_SHAPE;
    const size_t need = sfb::w8a16_mlp_workspace_bytes(M, F);
    if (need > sfb::kNoAllocScratchBytes) {
        snprintf(sfb::last_error_buf(), 256,
                 "sfb_w8a16_mlp_noalloc: M=%d, F=%d need %zu bytes of scratch; the static scratch holds %zu "
                 "(M*F <= 163840); use sfb_w8a16_mlp with a workspace", M, F, need, sfb::kNoAllocScratchBytes);
        return SFB_ERR_WORKSPACE;
    }
    void* scratch = nullptr;
    SFB_TRY(sfb::noalloc_scratch(&scratch));
    // the launch clears the counters at the start of the scratch on `stream`
    // (cudaMemsetAsync) and allocates nothing
    return sfb::w8a16_mlp_launch(x, ldx, w1, s1, b1, w2, s2, b2, residual, ldr, y, ldy, y_dtype, M, K, F, N, act,
                                 scratch, sfb::kNoAllocScratchBytes, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
