// common.cuh — shared device helpers and the context definition for libk3xb.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <string>

#include "k3xb.h"

struct k3xb_ctx {
    int device = 0;
    int sm_count = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    cudaStream_t side_stream = nullptr;   // work forked off `stream` within one call
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    std::string error;
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    void* io = nullptr;               // device side of the host-I/O entry points (*_host)
    size_t io_bytes = 0;
    k3xb_stats stats{};
    int32_t* status_word = nullptr;   // device-side validation status (route, plan)
    void* mxf4_scratch = nullptr;     // MXF4-engine region inside `scratch`
    void* mxf4_state = nullptr;       // MXF4-engine resources (tensor maps, attributes)
    void* ep_state = nullptr;         // expert parallelism: NCCL communicator
    void* resident = nullptr;         // resident weight table (resident.cu)
    void* profiler = nullptr;         // phase timing (profile.cu), NULL when off
    void* kda_held = nullptr;         // device-held KDA states (k3xb_kda_block_held)
};

namespace k3xb {

// Records a failure on the context and returns its status.
int fail(k3xb_ctx* ctx, int status, const std::string& message);
// Maps a CUDA error to K3XB_BACKEND_UNAVAILABLE with a message.
int cuda_fail(k3xb_ctx* ctx, cudaError_t err, const char* where);
// Grow-only device scratch (the reference's device_memory.cu keeps a
// grow-only scratch too). Growing synchronises the stream first.
int ensure_scratch(k3xb_ctx* ctx, size_t bytes, void** out);
// Grow-only device buffer for the inputs and results of the host-I/O entry
// points, apart from `scratch` so the device entry points they call may
// grow the scratch.
int ensure_io(k3xb_ctx* ctx, size_t bytes, void** out);
// Waits for ctx->stream; with expert parallelism on, under the
// communicator's bound (ep.cu), so a failed peer cannot hold it for ever.
int stream_wait(k3xb_ctx* ctx);

#define K3XB_CUDA(ctx, call)                                        \
    do {                                                            \
        cudaError_t k3xb_err_ = (call);                             \
        if (k3xb_err_ != cudaSuccess) return k3xb::cuda_fail((ctx), k3xb_err_, #call); \
    } while (0)

// Entry of a C ABI call on a context: a null context is INVALID_EXTENT, and
// the calling thread's current device becomes the context's when it is not
// already (a process may hold contexts on several GPUs).
#define K3XB_ENTER(ctx)                                                         \
    do {                                                                        \
        if (!(ctx)) return K3XB_INVALID_EXTENT;                                 \
        int k3xb_dev_ = -1;                                                     \
        if (cudaGetDevice(&k3xb_dev_) != cudaSuccess || k3xb_dev_ != (ctx)->device) \
            K3XB_CUDA((ctx), cudaSetDevice((ctx)->device));                     \
    } while (0)

#define K3XB_LAUNCHED(ctx)                                          \
    do {                                                            \
        cudaError_t k3xb_err_ = cudaGetLastError();                 \
        if (k3xb_err_ != cudaSuccess) return k3xb::cuda_fail((ctx), k3xb_err_, "kernel launch"); \
        ++(ctx)->stats.kernel_launches;                             \
    } while (0)

// Function attributes (cudaFuncSetAttribute) belong to a device: `set` runs
// once per device id, recorded in `done` (device ids below 64).
template <typename F>
int configure_once(k3xb_ctx* ctx, std::atomic<uint64_t>& done, F&& set) {
    const uint64_t bit = 1ull << (static_cast<unsigned>(ctx->device) & 63u);
    if (done.load(std::memory_order_acquire) & bit) return K3XB_OK;
    const int st = set();
    if (st == K3XB_OK) done.fetch_or(bit, std::memory_order_acq_rel);
    return st;
}

// Carves aligned sub-buffers out of one scratch allocation.
struct Carver {
    uintptr_t base;
    size_t used = 0;
    explicit Carver(void* p) : base(reinterpret_cast<uintptr_t>(p)) {}
    template <typename T>
    T* take(size_t count, size_t align = 256) {
        used = (used + align - 1) / align * align;
        T* p = reinterpret_cast<T*>(base + used);
        used += count * sizeof(T);
        return p;
    }
};
// Same arithmetic with no base, to size a scratch request.
struct Sizer {
    size_t used = 0;
    template <typename T>
    T* take(size_t count, size_t align = 256) {
        used = (used + align - 1) / align * align;
        used += count * sizeof(T);
        return nullptr;
    }
};

// ---- bf16 (official_moe.cpp:18-26, official_kda.cpp:31-39) ---------------
__host__ __device__ __forceinline__ float round_bf16(float value) {
#ifdef __CUDA_ARCH__
    uint32_t bits = __float_as_uint(value);
#else
    uint32_t bits;
    memcpy(&bits, &value, 4);
#endif
    if ((bits & 0x7f800000u) == 0x7f800000u) {
        if (bits & 0x007fffffu) bits |= 0x00400000u;
        bits &= 0xffff0000u;
    } else {
        bits += 0x7fffu + ((bits >> 16) & 1u);
        bits &= 0xffff0000u;
    }
#ifdef __CUDA_ARCH__
    return __uint_as_float(bits);
#else
    float out;
    memcpy(&out, &bits, 4);
    return out;
#endif
}

__device__ __forceinline__ float decode_bf16(uint16_t word) {
    return __uint_as_float(static_cast<uint32_t>(word) << 16);
}

__device__ __forceinline__ uint16_t encode_bf16(float value) {
    return static_cast<uint16_t>(__float_as_uint(round_bf16(value)) >> 16);
}

// ---- E2M1 / E8M0 --------------------------------------------------------------
// 2^s for s in [-127, 127] (2^-127 is the one subnormal case).
__device__ __forceinline__ float exp2i(int s) {
    return s >= -126 ? __uint_as_float(static_cast<uint32_t>(s + 127) << 23)
                     : __uint_as_float(0x00400000u);
}

// E2M1 magnitude table (runtime/src/ops.cpp:40-43, positive half).
__device__ __forceinline__ float e2m1_magnitude(uint32_t code3) {
    // 0, .5, 1, 1.5, 2, 3, 4, 6 from the 3-bit code: exponent e = code>>1,
    // mantissa m = code&1: e == 0 -> 0.5*m, else 2^(e-1) * (1 + m/2).
    const uint32_t e = code3 >> 1, m = code3 & 1u;
    return e == 0 ? 0.5f * static_cast<float>(m)
                  : exp2i(static_cast<int>(e) - 1) * (1.0f + 0.5f * static_cast<float>(m));
}

// Round-to-nearest-even onto the E2M1 grid, saturating at 6.
__device__ __forceinline__ uint32_t e2m1_code(float a) {
    if (a <= 0.25f) return 0;
    if (a < 0.75f) return 1;
    if (a <= 1.25f) return 2;
    if (a < 1.75f) return 3;
    if (a <= 2.5f) return 4;
    if (a < 3.5f) return 5;
    if (a <= 5.0f) return 6;
    return 7;
}

// Smallest s with amax <= 6 * 2^s (amax > 0), clamped to the E8M0 range.
__device__ __forceinline__ int e2m1_block_exponent(float amax) {
    int e = 0;
    const float m = frexpf(amax, &e);
    int s = (m <= 0.75f) ? e - 3 : e - 2;
    s = s < -127 ? -127 : s;
    return s > 127 ? 127 : s;
}

// ---- warp helpers ---------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace k3xb
