// common.cuh — shared host/device infrastructure of libsfb200.
//
// The library is built as one translation unit (sfb200.cu includes every
// kernel file), so the definitions here exist exactly once.
#pragma once

#include <atomic>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "../../include/sfb200.h"

namespace sfb {

// Error word written by bounded device-side waits that expired (0 = none).
__device__ int g_sfb_device_error = 0;

struct DeviceInfo {
    int ordinal = -1;
    int major = 0, minor = 0;
    int num_sms = 0;
    bool valid = false;
};

// Cached properties of the current device (one entry per ordinal).
inline const DeviceInfo& device_info() {
    static DeviceInfo infos[64];
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    DeviceInfo& d = infos[dev & 63];
    if (!d.valid) {
        std::lock_guard<std::mutex> lk(mu);
        if (!d.valid) {
            cudaDeviceProp prop{};
            if (cudaGetDeviceProperties(&prop, dev) == cudaSuccess) {
                d.ordinal = dev;
                d.major = prop.major;
                d.minor = prop.minor;
                d.num_sms = prop.multiProcessorCount;
                d.valid = true;
            }
        }
    }
    return d;
}

inline bool is_sm100(const DeviceInfo& d) { return d.valid && d.major == 10 && d.minor == 0; }

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library does not link libcuda directly.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

inline int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dt, int rank, void* base,
                             const cuuint64_t* dims, const cuuint64_t* strides,
                             const cuuint32_t* box, const cuuint32_t* estr,
                             CUtensorMapSwizzle swz) {
    EncodeTiledFn fn = get_encode_fn();
    if (fn == nullptr) return SFB_ERR_UNSUPPORTED;
    CUresult r = fn(map, dt, static_cast<cuuint32_t>(rank), base, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? SFB_OK : SFB_ERR_SHAPE;
}

// Text of the last CUDA error seen by this library on the calling thread.
inline char* last_error_buf() {
    static thread_local char buf[256] = "";
    return buf;
}
inline void record_cuda_error(cudaError_t e, const char* where) {
    snprintf(last_error_buf(), 256, "%s: %s (%s)", where, cudaGetErrorName(e), cudaGetErrorString(e));
    (void)cudaGetLastError();   // reported here; do not leak into the next launch check
}

// Every kernel of the library prefers the maximal shared-memory carveout, so
// that alternating between the big tcgen05 kernels (~225 KB of shared memory)
// and the small row kernels never forces an L1/shared reconfiguration of the
// SMs between launches. Applied once per kernel and device.
template <typename K>
inline void prefer_max_shared(K kernel) {
    static std::atomic<bool> done[64];      // idempotent: a race only repeats the call
    int dev = 0;
    cudaGetDevice(&dev);
    if (!done[dev & 63].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 static_cast<int>(cudaSharedmemCarveoutMaxShared)) != cudaSuccess)
            (void)cudaGetLastError();       // a hint only: clear its own error, no other
        done[dev & 63].store(true, std::memory_order_release);
    }
}

#ifdef SFB_TRACE
// Timeline of kernel launches (debug builds only): per launch and CTA, the
// global-timer start, the time past griddepcontrol.wait and the end.
inline unsigned long long*& tl_buf() { static unsigned long long* b = nullptr; return b; }
inline int& tl_count() { static int n = 0; return n; }
inline int tl_next() { return tl_buf() ? tl_count()++ : -1; }
__device__ __forceinline__ void tl_record(unsigned long long* buf, int launch, int kind,
                                          unsigned long long t0, unsigned long long t1) {
    if (buf == nullptr || launch < 0 || threadIdx.x != 0) return;
    const int cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    if (cta >= 512 || launch >= 4096) return;
    unsigned long long* e = buf + (static_cast<size_t>(launch) * 512 + cta) * 4;
    unsigned long long t2;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t2));
    e[0] = t0; e[1] = t1; e[2] = t2;
    e[3] = (static_cast<unsigned long long>(kind) << 32) | (gridDim.x * gridDim.y * gridDim.z);
}
#endif

// Element idx of an additive attention mask of dtype dt (SFB_F32/F16/BF16).
__device__ __forceinline__ float attn_mask_at(const void* m, int dt, int64_t idx) {
    if (dt == SFB_F32) return static_cast<const float*>(m)[idx];
    if (dt == SFB_F16) return __half2float(static_cast<const __half*>(m)[idx]);
    return __bfloat162float(static_cast<const __nv_bfloat16*>(m)[idx]);
}

// Options of the tensor-core attention launch beyond sfb_attn_args (model path).
struct AttnOpts {
    bool pdl = false;              // programmatic dependent launch
    bool v_f16 = false;            // bf16 Q/K, V already fp16
    const void* qn_w = nullptr;    // bf16 [64] per-head RMSNorm weight applied to Q rows
    const void* kn_w = nullptr;    // the same for K rows
    float norm_eps = 1e-6f;
};

// Makes a model's device current for the guard's lifetime and restores the
// caller's device afterwards, so a handle created on GPU k works from a thread
// whose current device is another one (every model entry point opens one).
struct DeviceGuard {
    int prev = -1, status = SFB_OK;
    bool switched = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) { (void)cudaGetLastError(); prev = -1; }
        if (prev != dev) {
            const cudaError_t e = cudaSetDevice(dev);
            if (e != cudaSuccess) { record_cuda_error(e, "model device"); status = SFB_ERR_CUDA; }
            else switched = true;
        }
    }
    ~DeviceGuard() {
        if (switched && prev >= 0 && cudaSetDevice(prev) != cudaSuccess) (void)cudaGetLastError();
    }
    DeviceGuard(const DeviceGuard&) = delete;
    DeviceGuard& operator=(const DeviceGuard&) = delete;
};

// Opens a model entry point: the model's lock (calls on one handle from
// several threads are serialised on the host) and its device.
#define SFB_MODEL_ENTRY(m)                                            \
    std::lock_guard<std::recursive_mutex> _sfb_lock((m)->mu);         \
    DeviceGuard _sfb_dev((m)->device);                                \
    if (_sfb_dev.status != SFB_OK) return _sfb_dev.status

// Returns the status of `expr` from the enclosing function unless it is SFB_OK.
#define SFB_TRY(expr) do { int _rc = (expr); if (_rc != SFB_OK) return _rc; } while (0)

// ── programmatic dependent launch (model path only) ───────────────────────
// A kernel launched with programmatic stream serialization may start while
// the previous kernel of the stream is still running. It must execute
// pdl_wait() before it reads or writes any memory that earlier kernels write
// or read (it returns once they have completed and their writes are
// visible); everything before that touches only its own shared memory,
// TMEM and constant weights. pdl_trigger() lets the next kernel be scheduled;
// kernels that allocate TMEM call it only after their allocation, so a later
// kernel never holds TMEM an earlier one waits for. Both are no-ops in a
// kernel launched without the attribute. The C-ABI entry points launch
// without it; SFB_PDL=0 turns it off for the model as well.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

inline bool pdl_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("SFB_PDL");
        return !(e != nullptr && e[0] == '0');
    }();
    return on;
}

// Fills the launch attribute for programmatic stream serialization; returns
// the number of attributes written (0 or 1).
inline int pdl_attr(cudaLaunchAttribute* at, bool pdl) {
    if (!pdl || !pdl_enabled()) return 0;
    at->id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at->val.programmaticStreamSerializationAllowed = 1;
    return 1;
}

// Launches a plain (non-cluster) kernel, optionally with programmatic
// dependent launch; returns an SFB status.
template <typename... KArgs, typename... Args>
inline int launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                         bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    cfg.numAttrs = pdl_attr(at, pdl);
    cfg.attrs = at;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        record_cuda_error(e, "kernel launch");
        return SFB_ERR_LAUNCH;
    }
    return SFB_OK;
}

inline int launch_status() {
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) return SFB_OK;
    record_cuda_error(e, "kernel launch");
    return SFB_ERR_LAUNCH;
}

}  // namespace sfb
