// route_static.cu — a router entry point that allocates no device memory.
//
// Who needs it: callers that are not allowed to allocate device memory
// while they run. Examples are a serving loop that has handed the whole HBM
// budget to weights and KDA state up front, a host application whose own
// caching allocator owns the device and forbids raw cudaMalloc next to it,
// and latency-critical loops where cudaMalloc/cudaFree would implicitly
// synchronise the device and stall every other stream. k3xb_route keeps
// its [tokens][experts] logits in the context's grow-only scratch, which
// calls cudaMalloc on first use and whenever a larger batch arrives.
// k3xb_route_static keeps them in a fixed array compiled into this library
// instead, so a call only launches kernels and issues one small memset.
//
// Limits and sharing:
//  * tokens * experts <= 262144 (1 MiB of float logits). Larger requests
//    are rejected with K3XB_INVALID_EXTENT before anything is launched.
//  * Every GPU that loads the library holds this 1 MiB array until the
//    process exits.
//  * All calls on a device share the one array and it keeps the last
//    call's contents. Calls whose work overlaps on the GPU (different
//    streams, or different host threads) race on it and must be
//    serialised by the caller.
//  * The first call on each device looks the array's device address up
//    once (cudaGetSymbolAddress, with that device current) and keeps it with
//    a small host-side launch record. Make that first call before any stream
//    capture begins.
//  * Device-side failures (a non-finite input, a bounded wait in the logits
//    kernel that ran out) are written to the caller's `status` word. With
//    status NULL they go to a word inside the array that nothing reads: the
//    call still returns K3XB_OK and ids/contributions are then undefined.
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace k3xb {
namespace {

constexpr size_t kStaticLogits = 262144;
constexpr size_t kStatusOffset = kStaticLogits * sizeof(float);
constexpr size_t kStaticBytes = kStatusOffset + 256;

// Logits [tokens][experts] followed by a device status word.
static __device__ __align__(256) unsigned char g_route_scratch[kStaticBytes];

// Per device: the array's device address and a launch context that carries
// the stream and status word for the shared launchers. Both are made by the
// first call on the device and kept until exit, so later calls do no
// host-side set-up (the launch context also keeps the tensor-map encoder it
// resolved). The context owns no device memory.
struct Site {
    void* base = nullptr;
    k3xb_ctx launch;
};
std::mutex g_lock;   // held for the host side of each call (set-up and launches)
constexpr int kMaxDevices = 128;
Site* g_site[kMaxDevices] = {};

// With g_lock held: the site of `device`, made with that device current.
int site_of(int device, Site** out) {
    if (device < 0 || device >= kMaxDevices) return K3XB_INVALID_EXTENT;
    if (!g_site[device]) {
        // the array's name is only a host-side handle; kernels need its
        // device address, resolved once per device with that device current
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_route_scratch) != cudaSuccess || !p) return K3XB_BACKEND_UNAVAILABLE;
        Site* s = new (std::nothrow) Site();
        if (!s) return K3XB_BACKEND_UNAVAILABLE;
        s->base = p;
        s->launch.device = device;
        if (cudaDeviceGetAttribute(&s->launch.sm_count, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
            delete s;
            return K3XB_BACKEND_UNAVAILABLE;
        }
        g_site[device] = s;
    }
    *out = g_site[device];
    return K3XB_OK;
}

}  // namespace
}  // namespace k3xb

extern "C" int k3xb_route_static(const float* hidden, uint32_t tokens, uint32_t hidden_size,
                                 const uint16_t* router, const float* correction, uint32_t experts,
                                 uint32_t top_k, uint32_t* ids, float* contributions, int32_t* status,
                                 void* stream) {
    using namespace k3xb;
    if (!hidden || !router || !correction || !ids || !contributions) return K3XB_INVALID_EXTENT;
    if (!tokens || !hidden_size || !experts || !top_k || top_k > experts || top_k > 32 || experts > 1024)
        return K3XB_INVALID_EXTENT;
    if (static_cast<size_t>(tokens) * experts > kStaticLogits) return K3XB_INVALID_EXTENT;
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return K3XB_BACKEND_UNAVAILABLE;
    std::lock_guard<std::mutex> guard(g_lock);
    Site* site = nullptr;
    int st = site_of(device, &site);
    if (st) return st;
    float* logits = static_cast<float*>(site->base);
    int32_t* word = status ? status : reinterpret_cast<int32_t*>(static_cast<unsigned char*>(site->base) + kStatusOffset);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // the status word must start at zero; the logits are fully overwritten
    if (cudaMemsetAsync(word, 0, sizeof(int32_t), s) != cudaSuccess) return K3XB_BACKEND_UNAVAILABLE;
    site->launch.stream = s;
    site->launch.status_word = word;
    st = launch_router_logits(&site->launch, hidden, tokens, hidden_size, router, experts, logits);
    if (st) return st;
    return launch_topk(&site->launch, logits, correction, tokens, experts, top_k, ids, contributions, nullptr, word);
}
