// ep.cu — expert parallelism: the routed experts of a MoE layer sharded over
// the GPUs of one box, tokens exchanged with NCCL all-to-all over NVLink.
//
// Rank r owns experts [r*E_r, (r+1)*E_r) (E_r = E / world) and T_r tokens
// of its own sequences (data parallel); the router, the shared expert and
// the combine stay on the token's home rank. Per MoE layer:
//   route           all E logits, Top-k (router.cu), on the home rank
//   dispatch        every token row to every rank plus k entries of (local
//                   expert, slot) metadata per row; fixed capacity (T_r rows
//                   per destination), so the exchange needs no host-side
//                   counts and every step moves the same bytes
//   all-to-all #1   ncclSend/ncclRecv per peer in one group
//   local plan      expert-major over the received rows (ascending local
//                   expert, (row, slot) order inside a group)
//   experts         the tcgen05 engine (experts_tc.cu) on the local experts
//   all-to-all #2   each (row, slot) output back to the home rank (bf16)
//   combine         slot-ordered weighted sum + shared expert (the single-GPU
//                   arithmetic, official_moe.cpp:313-322), so the output is
//                   bit-identical to the one-GPU layer for any world size
//
// NCCL is opened at run time (dlopen "libnccl.so.2"), which picks the copy
// the process already loaded (torch's, when torch is imported first).
//
// Failure detection (ep_guard.hpp): every wait on the communicator has a
// deadline (k3xb_ep_config.timeout_ms) — creation and group launch of a
// nonblocking communicator, and the stream drain of k3xb_sync, of scratch
// growth and of k3xb_destroy. On expiry, or on an asynchronous NCCL error,
// the communicator is aborted (its kernels in flight return) and the
// expert-parallel entry points refuse until k3xb_ep_finalize and a new init.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <memory>
#include <mutex>
#include <thread>

#include "common.cuh"
#include "ep_guard.hpp"
#include "kernels.cuh"
#include "profile.cuh"

namespace k3xb {

namespace {

struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclSend) send = nullptr;
    decltype(&ncclRecv) recv = nullptr;
    decltype(&ncclGroupStart) group_start = nullptr;
    decltype(&ncclGroupEnd) group_end = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    decltype(&ncclCommInitRankConfig) comm_init_rank_config = nullptr;
    decltype(&ncclCommGetAsyncError) comm_get_async_error = nullptr;
    decltype(&ncclCommAbort) comm_abort = nullptr;
    decltype(&ncclCommFinalize) comm_finalize = nullptr;
    bool ok = false;
};

static_assert(ncclSuccess == kCommSuccess && ncclInProgress == kCommInProgress, "ep_guard.hpp codes are nccl.h's");

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        api.send = reinterpret_cast<decltype(api.send)>(dlsym(h, "ncclSend"));
        api.recv = reinterpret_cast<decltype(api.recv)>(dlsym(h, "ncclRecv"));
        api.group_start = reinterpret_cast<decltype(api.group_start)>(dlsym(h, "ncclGroupStart"));
        api.group_end = reinterpret_cast<decltype(api.group_end)>(dlsym(h, "ncclGroupEnd"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
        api.comm_init_rank_config =
            reinterpret_cast<decltype(api.comm_init_rank_config)>(dlsym(h, "ncclCommInitRankConfig"));
        api.comm_get_async_error =
            reinterpret_cast<decltype(api.comm_get_async_error)>(dlsym(h, "ncclCommGetAsyncError"));
        api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(dlsym(h, "ncclCommAbort"));
        api.comm_finalize = reinterpret_cast<decltype(api.comm_finalize)>(dlsym(h, "ncclCommFinalize"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.send && api.recv &&
                 api.group_start && api.group_end && api.error_string && api.comm_init_rank_config &&
                 api.comm_get_async_error && api.comm_abort && api.comm_finalize;
    });
    return api;
}

struct EpState;

// The communicator and stream operations ep_guard.hpp waits with.
struct NcclOps {
    EpState* ep;
    k3xb_ctx* ctx;
    cudaError_t last_cuda = cudaSuccess;
    int async_error(int* state);
    int abort();
    int stream_query() {
        const cudaError_t e = cudaStreamQuery(ctx->stream);
        if (e == cudaSuccess) return 0;
        if (e == cudaErrorNotReady) {
            if (cudaPeekAtLastError() == cudaErrorNotReady) cudaGetLastError();
            return 1;
        }
        last_cuda = e;
        return -1;
    }
    uint64_t now_ms() const {
        return static_cast<uint64_t>(std::chrono::duration_cast<std::chrono::milliseconds>(
                                         std::chrono::steady_clock::now().time_since_epoch())
                                         .count());
    }
    void pause(uint32_t polls) const {
        if (polls < 1024) std::this_thread::yield();
        else std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
    const char* describe(int r) const { return nccl().error_string(static_cast<ncclResult_t>(r)); }
};

struct EpState {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    bool nonblocking = false;
    CommGuard<NcclOps> guard;
    EpState(k3xb_ctx* ctx, uint32_t timeout_ms) : guard(NcclOps{this, ctx}, timeout_ms) {}
};

int NcclOps::async_error(int* state) {
    ncclResult_t s = ncclSuccess;
    const ncclResult_t r = nccl().comm_get_async_error(ep->comm, &s);
    *state = static_cast<int>(s);
    return static_cast<int>(r);
}

int NcclOps::abort() { return static_cast<int>(nccl().comm_abort(ep->comm)); }

// Status of a guard outcome; the reason is the guard's.
int guard_fail(k3xb_ctx* ctx, EpState* ep, CommWait w) {
    if (w == CommWait::stuck)
        return fail(ctx, K3XB_BACKEND_UNAVAILABLE,
                    "expert parallelism: the stream did not drain within the bound after the communicator was "
                    "aborted (" + ep->guard.reason() + ")");
    if (w == CommWait::refused)
        return fail(ctx, K3XB_INVALID_STATE,
                    "expert parallelism: communicator aborted (" + ep->guard.reason() +
                        "); k3xb_ep_finalize and k3xb_ep_init again");
    return fail(ctx, K3XB_BACKEND_UNAVAILABLE, "expert parallelism: " + ep->guard.reason());
}

// One NCCL group: `body` issues the sends and receives and returns the
// first failing result. The group is always closed; an error or a launch
// that does not settle in time aborts the communicator.
template <typename F>
int nccl_group(k3xb_ctx* ctx, EpState* ep, const char* what, F&& body) {
    const NcclApi& api = nccl();
    ncclResult_t r = api.group_start();
    if (r == ncclSuccess) {
        const ncclResult_t rb = body();
        const ncclResult_t re = api.group_end();
        r = rb != ncclSuccess ? rb : re;
    }
    const CommWait w = ep->guard.settle(static_cast<int>(r), what);
    return w == CommWait::ok ? K3XB_OK : guard_fail(ctx, ep, w);
}

constexpr uint32_t kNoEntry = 0xffffffffu;

// One thread per (destination, token, slot): meta[g][t][j] = local expert
// << 8 | slot when the slot's expert lives on rank g, else kNoEntry.
__global__ void ep_dispatch_kernel(const uint32_t* __restrict__ ids, uint32_t T, uint32_t K, uint32_t E_r,
                                   uint32_t G, uint32_t* __restrict__ send_meta) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<size_t>(G) * T * K) return;
    const uint32_t j = static_cast<uint32_t>(i % K);
    const uint32_t t = static_cast<uint32_t>((i / K) % T), g = static_cast<uint32_t>(i / K / T);
    const uint32_t e = ids[static_cast<size_t>(t) * K + j];
    send_meta[i] = e / E_r == g ? ((e - g * E_r) << 8 | j) : kNoEntry;
}

// One CTA per (destination, token): every row goes to every destination
// (fixed capacity; rows without an entry there are computed and dropped),
// so no buffer holds stale data.
__global__ void ep_rows_kernel(const float* __restrict__ hidden, uint32_t T, uint32_t H, float* __restrict__ send_x) {
    const uint32_t t = blockIdx.x, g = blockIdx.y;
    const float* src = hidden + static_cast<size_t>(t) * H;
    float* dst = send_x + (static_cast<size_t>(g) * T + t) * H;
    for (uint32_t h = threadIdx.x; h < H; h += blockDim.x) dst[h] = src[h];
}

// Expert-major plan over the received rows (one CTA): groups are the local
// experts with work in ascending order; inside a group (row, slot) order.
__global__ void __launch_bounds__(1024) ep_plan_kernel(const uint32_t* __restrict__ meta, uint32_t rows, uint32_t K,
                                                       uint32_t E_r, k3xb_plan plan) {
    extern __shared__ uint32_t cnt[];   // [E_r + 1]
    for (uint32_t e = threadIdx.x; e <= E_r; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    const size_t n = static_cast<size_t>(rows) * K;
    for (size_t i = threadIdx.x; i < n; i += blockDim.x)
        if (meta[i] != kNoEntry) atomicAdd(&cnt[meta[i] >> 8], 1u);
    __syncthreads();
    if (threadIdx.x == 0) {   // E_r <= 1024: a serial scan is short
        uint32_t off = 0, g = 0;
        for (uint32_t e = 0; e < E_r; ++e) {
            const uint32_t c = cnt[e];
            cnt[e] = off;
            if (c) {
                plan.group_expert[g] = e;
                plan.group_offset[g] = off;
                ++g;
            }
            off += c;
        }
        plan.group_offset[g] = off;
        *plan.group_count = g;
    }
    __syncthreads();
    // stable fill in (row, slot) order: one warp walks the entries 32 at a
    // time; lanes with the same expert take consecutive positions
    if (threadIdx.x < 32) {
        const uint32_t lane = threadIdx.x;
        for (size_t base = 0; base < n; base += 32) {
            const size_t i = base + lane;
            const uint32_t m = i < n ? meta[i] : kNoEntry;
            const uint32_t key = m == kNoEntry ? kNoEntry : (m >> 8);
            const uint32_t peers = __match_any_sync(0xffffffffu, key);
            const uint32_t pos = __popc(peers & ((1u << lane) - 1u));
            uint32_t at = 0;
            if (m != kNoEntry) at = cnt[key] + pos;
            __syncwarp();
            if (m != kNoEntry) {
                plan.assign_token[at] = static_cast<uint32_t>(i / K);
                plan.assign_slot[at] = m & 0xffu;
                plan.assign_contrib[at] = 0.0f;
                if (lane == 31u - __clz(peers)) cnt[key] += __popc(peers);   // last lane of the group
            }
            __syncwarp();
        }
    }
}

// combine (official_moe.cpp:313-322, then + shared): slot j's output comes
// from the rank that owns expert ids[t][j]: y[g][t][j][H] (bf16 words; the
// expert outputs are bf16-rounded, so the words are exact).
__global__ void ep_combine_kernel(const uint16_t* __restrict__ y, const uint32_t* __restrict__ ids,
                                  const float* __restrict__ contrib, const float* __restrict__ shared, uint32_t T,
                                  uint32_t K, uint32_t H, uint32_t E_r, float* __restrict__ out) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<size_t>(T) * H) return;
    const size_t t = i / H, h = i % H;
    float mixed = 0.0f;
    for (uint32_t j = 0; j < K; ++j) {
        const uint32_t g = ids[t * K + j] / E_r;
        const float v = decode_bf16(y[((static_cast<size_t>(g) * T + t) * K + j) * H + h]);
        mixed = __fadd_rn(mixed, __fmul_rn(contrib[t * K + j], v));
    }
    mixed = round_bf16(mixed);
    const float sh = shared ? shared[i] : 0.0f;
    out[i] = round_bf16(__fadd_rn(mixed, sh));
}

EpState* ep_of(k3xb_ctx* ctx) { return static_cast<EpState*>(ctx->ep_state); }

// All-to-all of `per_peer` elements of `type` (peer g's block at g*per_peer).
int all_to_all(k3xb_ctx* ctx, const void* send, void* recv, size_t per_peer, ncclDataType_t type, size_t elem) {
    EpState* ep = ep_of(ctx);
    const NcclApi& api = nccl();
    return nccl_group(ctx, ep, "return exchange", [&]() -> ncclResult_t {
        for (int g = 0; g < ep->world; ++g) {
            ncclResult_t r = api.send(static_cast<const char*>(send) + g * per_peer * elem, per_peer, type, g,
                                      ep->comm, ctx->stream);
            if (r == ncclSuccess)
                r = api.recv(static_cast<char*>(recv) + g * per_peer * elem, per_peer, type, g, ep->comm,
                             ctx->stream);
            if (r != ncclSuccess) return r;
        }
        return ncclSuccess;
    });
}

}  // namespace

int ep_world(const k3xb_ctx* ctx) {
    return ctx->ep_state ? static_cast<const EpState*>(ctx->ep_state)->world : 0;
}

int ep_drain(k3xb_ctx* ctx) {
    EpState* ep = ep_of(ctx);
    if (!ep) return K3XB_OK;
    bool cuda_error = false;
    const CommWait w = ep->guard.drain("stream drain", &cuda_error);
    if (cuda_error) return cuda_fail(ctx, ep->guard.ops().last_cuda, "cudaStreamQuery");
    return w == CommWait::ok ? K3XB_OK : guard_fail(ctx, ep, w);
}

void release_ep(k3xb_ctx* ctx) {
    EpState* ep = ep_of(ctx);
    if (!ep) return;
    // an aborted communicator is already freed (ncclCommAbort)
    if (ep->comm && !ep->guard.aborted()) {
        const NcclApi& api = nccl();
        if (ep->nonblocking) {   // finalize settles like any nonblocking call, then destroy
            const CommWait w = ep->guard.settle(static_cast<int>(api.comm_finalize(ep->comm)), "ncclCommFinalize");
            if (w == CommWait::ok) api.comm_destroy(ep->comm);
        } else {
            api.comm_destroy(ep->comm);
        }
    }
    delete ep;
    ctx->ep_state = nullptr;
}

// Scratch of one EP layer call (after the MoE scratch of the local layer).
size_t ep_scratch_bytes(uint32_t G, uint32_t T, uint32_t K, uint32_t H, uint32_t E_r) {
    Sizer s;
    s.take<float>(static_cast<size_t>(G) * T * H);       // send_x
    s.take<float>(static_cast<size_t>(G) * T * H);       // recv_x
    s.take<uint32_t>(static_cast<size_t>(G) * T * K);    // send_meta
    s.take<uint32_t>(static_cast<size_t>(G) * T * K);    // recv_meta
    s.take<uint16_t>(static_cast<size_t>(G) * T * K * H);   // y (rows received, per slot)
    s.take<uint16_t>(static_cast<size_t>(G) * T * K * H);   // y_home
    s.take<uint32_t>(E_r + 1);                           // plan
    s.take<uint32_t>(E_r + 1);
    s.take<uint32_t>(static_cast<size_t>(G) * T * K);
    s.take<uint32_t>(static_cast<size_t>(G) * T * K);
    s.take<float>(static_cast<size_t>(G) * T * K);
    s.take<uint32_t>(1);
    return s.used + 1024;
}

int ep_moe_forward(k3xb_ctx* ctx, const k3xb_moe_layer& L, uint32_t E, const float* hidden, uint32_t T,
                   const uint32_t* ids, const float* contrib, const float* shared, void* region, float* out) {
    EpState* ep = ep_of(ctx);
    {   // a failure NCCL saw since the last call (a peer's) ends the communicator before new work is queued
        const CommWait w = ep->guard.check("expert parallelism");
        if (w != CommWait::ok) return guard_fail(ctx, ep, w);
    }
    const uint32_t G = static_cast<uint32_t>(ep->world), K = L.top_k, H = L.hidden, E_r = L.experts;
    Carver c(region);
    float* send_x = c.take<float>(static_cast<size_t>(G) * T * H);
    float* recv_x = c.take<float>(static_cast<size_t>(G) * T * H);
    uint32_t* send_meta = c.take<uint32_t>(static_cast<size_t>(G) * T * K);
    uint32_t* recv_meta = c.take<uint32_t>(static_cast<size_t>(G) * T * K);
    uint16_t* y = c.take<uint16_t>(static_cast<size_t>(G) * T * K * H);
    uint16_t* y_home = c.take<uint16_t>(static_cast<size_t>(G) * T * K * H);
    k3xb_plan plan{};
    plan.group_expert = c.take<uint32_t>(E_r + 1);
    plan.group_offset = c.take<uint32_t>(E_r + 1);
    plan.assign_token = c.take<uint32_t>(static_cast<size_t>(G) * T * K);
    plan.assign_slot = c.take<uint32_t>(static_cast<size_t>(G) * T * K);
    plan.assign_contrib = c.take<float>(static_cast<size_t>(G) * T * K);
    plan.group_count = c.take<uint32_t>(1);
    plan.status = ctx->status_word;
    const size_t nm = static_cast<size_t>(G) * T * K;
    {
        PhaseScope ph(ctx, K3XB_PHASE_EP_DISPATCH);
        ep_dispatch_kernel<<<static_cast<unsigned>((nm + 255) / 256), 256, 0, ctx->stream>>>(ids, T, K, E_r, G,
                                                                                             send_meta);
        K3XB_LAUNCHED(ctx);
        ep_rows_kernel<<<dim3(T, G), 256, 0, ctx->stream>>>(hidden, T, H, send_x);
        K3XB_LAUNCHED(ctx);
    }
    int st;
    {   // metadata and rows in one NCCL group
        PhaseScope ph(ctx, K3XB_PHASE_EP_EXCHANGE);
        const NcclApi& api = nccl();
        st = nccl_group(ctx, ep, "dispatch exchange", [&]() -> ncclResult_t {
            const size_t nm_g = static_cast<size_t>(T) * K, nx_g = static_cast<size_t>(T) * H;
            for (uint32_t g = 0; g < G; ++g) {
                const int peer = static_cast<int>(g);
                ncclResult_t r = api.send(send_meta + g * nm_g, nm_g, ncclUint32, peer, ep->comm, ctx->stream);
                if (r == ncclSuccess) r = api.recv(recv_meta + g * nm_g, nm_g, ncclUint32, peer, ep->comm, ctx->stream);
                if (r == ncclSuccess) r = api.send(send_x + g * nx_g, nx_g, ncclFloat32, peer, ep->comm, ctx->stream);
                if (r == ncclSuccess) r = api.recv(recv_x + g * nx_g, nx_g, ncclFloat32, peer, ep->comm, ctx->stream);
                if (r != ncclSuccess) return r;
            }
            return ncclSuccess;
        });
        if (st) return st;
    }
    {
        PhaseScope ph(ctx, K3XB_PHASE_PLAN);
        ep_plan_kernel<<<1, 1024, (E_r + 1) * sizeof(uint32_t), ctx->stream>>>(recv_meta, G * T, K, E_r, plan);
        K3XB_LAUNCHED(ctx);
    }
    if ((st = launch_mxf4_experts(ctx, L, recv_x, G * T, plan, nullptr, y))) return st;
    {
        PhaseScope ph(ctx, K3XB_PHASE_EP_RETURN);
        if ((st = all_to_all(ctx, y, y_home, static_cast<size_t>(T) * K * H, ncclBfloat16, 2))) return st;
    }
    const size_t n = static_cast<size_t>(T) * H;
    PhaseScope ph(ctx, K3XB_PHASE_COMBINE);
    ep_combine_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, ctx->stream>>>(y_home, ids, contrib, shared,
                                                                                       T, K, H, E_r, out);
    K3XB_LAUNCHED(ctx);
    (void)E;
    return K3XB_OK;
}

}  // namespace k3xb

using namespace k3xb;

extern "C" {

int k3xb_ep_unique_id(uint8_t* out) {
    if (!out) return K3XB_INVALID_EXTENT;
    if (!nccl().ok) return K3XB_BACKEND_UNAVAILABLE;
    ncclUniqueId id;
    if (nccl().get_unique_id(&id) != ncclSuccess) return K3XB_BACKEND_UNAVAILABLE;
    std::memcpy(out, &id, sizeof id);
    return K3XB_OK;
}

int k3xb_ep_init_config(k3xb_ctx* ctx, const uint8_t* unique_id, int32_t rank, int32_t world,
                        const k3xb_ep_config* config) {
    K3XB_ENTER(ctx);
    if (!unique_id || world < 1 || rank < 0 || rank >= world)
        return fail(ctx, K3XB_INVALID_EXTENT, "ep_init arguments");
    if (config && config->nonblocking > 1) return fail(ctx, K3XB_INVALID_EXTENT, "ep_config.nonblocking is 0 or 1");
    if (ctx->ep_state) return fail(ctx, K3XB_INVALID_STATE, "expert parallelism already initialised");
    if (!nccl().ok) return fail(ctx, K3XB_BACKEND_UNAVAILABLE, "libnccl.so.2 could not be opened");
    const uint32_t timeout = config && config->timeout_ms ? config->timeout_ms : K3XB_EP_DEFAULT_TIMEOUT_MS;
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof id);
    std::unique_ptr<EpState> ep(new (std::nothrow) EpState(ctx, timeout));
    if (!ep) return fail(ctx, K3XB_BACKEND_UNAVAILABLE, "ep_init: out of host memory");
    ep->rank = rank;
    ep->world = world;
    ep->nonblocking = config && config->nonblocking;
    if (!ep->nonblocking) {   // creation blocks until every rank has joined
        const ncclResult_t r = nccl().comm_init_rank(&ep->comm, world, id, rank);
        if (r != ncclSuccess)
            return fail(ctx, K3XB_BACKEND_UNAVAILABLE, std::string("ncclCommInitRank: ") + nccl().error_string(r));
    } else {   // creation returns at once and settles under the deadline
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.blocking = 0;
        const ncclResult_t r = nccl().comm_init_rank_config(&ep->comm, world, id, rank, &cfg);
        if (!ep->comm)
            return fail(ctx, K3XB_BACKEND_UNAVAILABLE,
                        std::string("ncclCommInitRankConfig: ") + nccl().error_string(r));
        const CommWait w = ep->guard.settle(static_cast<int>(r), "ncclCommInitRankConfig");
        if (w != CommWait::ok)
            return fail(ctx, K3XB_BACKEND_UNAVAILABLE, "expert parallelism: " + ep->guard.reason());
    }
    ctx->ep_state = ep.release();
    return K3XB_OK;
}

int k3xb_ep_init(k3xb_ctx* ctx, const uint8_t* unique_id, int32_t rank, int32_t world) {
    return k3xb_ep_init_config(ctx, unique_id, rank, world, nullptr);
}

int k3xb_ep_status(k3xb_ctx* ctx) {
    K3XB_ENTER(ctx);
    EpState* ep = ep_of(ctx);
    if (!ep) return fail(ctx, K3XB_INVALID_STATE, "expert parallelism not initialised");
    const CommWait w = ep->guard.check("expert parallelism");
    return w == CommWait::ok ? K3XB_OK : guard_fail(ctx, ep, w);
}

int k3xb_ep_abort(k3xb_ctx* ctx) {
    K3XB_ENTER(ctx);
    EpState* ep = ep_of(ctx);
    if (!ep) return fail(ctx, K3XB_INVALID_STATE, "expert parallelism not initialised");
    ep->guard.abort_now("aborted by the caller");
    const int st = ep_drain(ctx);
    if (st != K3XB_INVALID_STATE) return st;   // a CUDA error, or still busy after the bound
    ctx->error.clear();                        // drained: the refusal is the state asked for
    return K3XB_OK;
}

int k3xb_ep_finalize(k3xb_ctx* ctx) {
    K3XB_ENTER(ctx);
    int st = K3XB_OK;
    if (ep_of(ctx) && !ep_of(ctx)->guard.aborted()) st = ep_drain(ctx);   // bounded: aborts on expiry
    release_ep(ctx);
    return st == K3XB_INVALID_STATE ? K3XB_OK : st;
}

}  // extern "C"
