// ep.cu — expert parallelism: the routed experts of a MoE layer sharded over
// the GPUs of one box, rows and expert outputs moved through peer memory
// over NVLink.
//
// Rank r owns experts [r*E_r, (r+1)*E_r) (E_r = E / world), or those a
// placement table gives it (k3xb_moe_layer.ep_owner), and T tokens of
// its own sequences (data parallel); the router, the shared expert and the
// combine stay on the token's home rank. Every rank owns an exchange window
// that the other ranks map (CUDA IPC; the handles are all-gathered over an
// NCCL communicator once, when the window is made). Per MoE layer:
//   route           all E logits, Top-k (router.cu), on the home rank
//   dispatch        one kernel stores, into every rank's window, the token's
//                   k metadata words (local expert << 8 | slot, or none)
//                   and, only where one of its experts lives, the row
//                   (bf16 words when the rows are bf16-valued); its last CTA
//                   raises this rank's dispatch flag in every window
//   local plan      waits (bounded) for every rank's dispatch flag, then
//                   builds the expert-major plan over the received rows
//                   (ascending local expert, (row, slot) order in a group)
//   experts         the tcgen05 engine (experts_tc.cu) on the local
//                   experts; the down projection's epilogue stores each
//                   (token, slot) output row straight into the home rank's
//                   window, so only computed rows cross NVLink, and its last
//                   CTA raises this rank's return flag in every window
//   combine         waits (bounded) for every rank's return flag, then the
//                   slot-ordered weighted sum + shared expert (the one-GPU
//                   arithmetic, official_moe.cpp:313-322), so the output is
//                   bit-identical to the one-GPU layer for any world size
// No collective library kernel and no TMA multicast touches peer memory:
// the peer stores are plain st.global from this library's own kernels.
//
// NCCL is opened at run time (dlopen "libnccl.so.2"), which picks the copy
// the process already loaded (torch's, when torch is imported first).
//
// Failure detection (ep_guard.hpp): every host wait on the communicator has
// a deadline (k3xb_ep_config.timeout_ms) — creation and launches of a
// nonblocking communicator, and the stream drains of k3xb_sync, of scratch
// and window growth and of k3xb_destroy — and every device wait for the
// other ranks' flags gives up after ep_sync.cuh's bound. On expiry, or on an
// asynchronous NCCL error, the exchange is aborted and the expert-parallel
// entry points refuse until k3xb_ep_finalize and a new init.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include "common.cuh"
#include "ep_guard.hpp"
#include "ep_sync.cuh"
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
    decltype(&ncclAllGather) all_gather = nullptr;
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
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.send && api.recv &&
                 api.group_start && api.group_end && api.error_string && api.comm_init_rank_config &&
                 api.comm_get_async_error && api.comm_abort && api.comm_finalize && api.all_gather;
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

constexpr uint64_t kOffDispatchFlags = 0, kOffReturnFlags = 32, kOffCounters = 64, kOffGaveUp = 72;
constexpr uint64_t kHeaderBytes = 256;

struct EpWindow {
    uint8_t* own = nullptr;
    size_t bytes = 0;
    uint8_t* peer[8] = {};   // every rank's window as mapped here (peer[rank] = own)
    uint32_t cap_t = 0, cap_k = 0, cap_d = 0;
    uint64_t off_meta[2] = {}, off_rows[2] = {}, off_y[2] = {};
};

struct EpState {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    bool nonblocking = false;
    EpWindow window;
    uint32_t epoch = 0;   // calls so far (the flags' values)
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

// ---- the exchange window ------------------------------------------------------
// Every rank owns one device buffer that the other ranks map through CUDA IPC
// and write into over NVLink. Regions (byte offsets, the same on every rank):
//   header   dispatch flags [8] u32 (word g: the last call whose rows and
//            metadata rank g has stored here), return flags [8] u32 (word g:
//            the last call whose expert outputs rank g has stored here), the
//            grid-completion counters [2] u32 and the gave-up word
//   meta[b]  [G][T][K] u32 per received row: local expert << 8 | slot, or
//            kNoEntry for a slot whose expert lives elsewhere
//   rows[b]  [G][T][D] received rows (bf16 words or floats)
//   y[b]     [T][K][D] bf16 expert outputs of this rank's own tokens
// b = call parity. Region sizes come from the window's capacity (tokens,
// slots, width), the packing inside a region from the call's own dims, so a
// call never writes into a region another call may still read: when rank r
// stores call c+2's rows into rank g's parity-c region, rank g has finished
// call c+1's down projection (rank r's combine of c+1 waited for it), which
// came after its reads of call c's rows; y regions the same way round.
uint64_t align256(uint64_t x) { return (x + 255) / 256 * 256; }

// One thread per (destination, token) CTA: the K metadata words of the row
// for rank g, and the row itself when one of its slots' experts lives there.
// The last CTA of the grid then raises this rank's dispatch flag in every
// window (ep_signal_grid_done).
struct DispatchArgs {
    uint8_t* win[8];
    uint64_t off_meta, off_rows;
    uint32_t rank, world, epoch, T, K, D, E_r;
    int rows_bf16;
    uint32_t* done;
    const uint32_t* owner;   // k3xb_moe_layer.ep_owner, or NULL: contiguous ranges
    int32_t* status;
};

__global__ void __launch_bounds__(256) ep_dispatch_kernel(const float* __restrict__ x,
                                                          const uint32_t* __restrict__ ids, DispatchArgs a) {
    const uint32_t t = blockIdx.x, g = blockIdx.y;
    __shared__ int present;
    if (threadIdx.x == 0) present = 0;
    __syncthreads();
    uint32_t* meta = reinterpret_cast<uint32_t*>(a.win[g] + a.off_meta) + (static_cast<size_t>(a.rank) * a.T + t) * a.K;
    for (uint32_t j = threadIdx.x; j < a.K; j += blockDim.x) {
        const uint32_t e = ids[static_cast<size_t>(t) * a.K + j];
        uint32_t owner_rank = e / a.E_r, local = e - owner_rank * a.E_r;
        if (a.owner) {
            const uint32_t o = __ldg(a.owner + e);
            owner_rank = o >> 16;
            local = o & 0xffffu;
            if (owner_rank >= a.world || local >= a.E_r) {   // not a placement of this world: drop, report
                if (g == 0) atomicExch(a.status, K3XB_INVALID_STATE);
                owner_rank = a.world;
            }
        }
        const bool here = owner_rank == g;
        meta[j] = here ? (local << 8 | j) : kNoEntry;
        if (here) present = 1;
    }
    __syncthreads();
    if (present) {
        const size_t row = static_cast<size_t>(a.rank) * a.T + t;
        const float4* src = reinterpret_cast<const float4*>(x + static_cast<size_t>(t) * a.D);
        if (a.rows_bf16) {   // the rows are bf16-valued: 8 words per 16-byte store
            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(a.win[g] + a.off_rows) + row * a.D);
            for (uint32_t i = threadIdx.x; i < a.D / 8; i += blockDim.x) {
                const float4 u = src[2 * i], v = src[2 * i + 1];
                uint4 w;
                w.x = encode_bf16(u.x) | static_cast<uint32_t>(encode_bf16(u.y)) << 16;
                w.y = encode_bf16(u.z) | static_cast<uint32_t>(encode_bf16(u.w)) << 16;
                w.z = encode_bf16(v.x) | static_cast<uint32_t>(encode_bf16(v.y)) << 16;
                w.w = encode_bf16(v.z) | static_cast<uint32_t>(encode_bf16(v.w)) << 16;
                dst[i] = w;
            }
        } else {
            float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(a.win[g] + a.off_rows) + row * a.D);
            for (uint32_t i = threadIdx.x; i < a.D / 4; i += blockDim.x) dst[i] = src[i];
        }
    }
    ep_signal_grid_done(a.done, a.win, kOffDispatchFlags, a.rank, a.world, a.epoch);
}

// Expert-major plan over the received rows (one CTA), after every rank's
// dispatch flag shows this call: groups are the local experts with work in
// ascending order; inside a group (row, slot) order.
__global__ void __launch_bounds__(1024) ep_plan_kernel(const uint8_t* __restrict__ win, uint64_t off_meta,
                                                       uint32_t rows, uint32_t K, uint32_t E_r, uint32_t world,
                                                       uint32_t epoch, k3xb_plan plan, int32_t* status) {
    extern __shared__ uint32_t cnt[];   // [E_r + 1]
    __shared__ int ready;
    if (threadIdx.x == 0)
        ready = ep_wait_flags(reinterpret_cast<const uint32_t*>(win + kOffDispatchFlags), world, epoch,
                              reinterpret_cast<volatile int32_t*>(const_cast<uint8_t*>(win) + kOffGaveUp), status);
    for (uint32_t e = threadIdx.x; e <= E_r; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    if (!ready) {   // gave up: no work this call (the status word carries the failure)
        if (threadIdx.x == 0) {
            plan.group_offset[0] = 0;
            *plan.group_count = 0;
        }
        return;
    }
    const uint32_t* meta = reinterpret_cast<const uint32_t*>(win + off_meta);
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

// combine (official_moe.cpp:313-322, then + shared) over the y region, after
// every rank's return flag shows this call: slot j's output row was stored by
// the rank that owns expert ids[t][j] (bf16 words: the expert outputs are
// bf16-rounded, so the words are exact).
__global__ void __launch_bounds__(256) ep_combine_kernel(const uint8_t* __restrict__ win, uint64_t off_y,
                                                         const uint32_t* __restrict__ ids,
                                                         const float* __restrict__ contrib,
                                                         const float* __restrict__ shared, uint32_t T, uint32_t K,
                                                         uint32_t H, uint32_t world, uint32_t epoch,
                                                         float* __restrict__ out, int32_t* status) {
    __shared__ int ready;
    if (threadIdx.x == 0)
        ready = ep_wait_flags(reinterpret_cast<const uint32_t*>(win + kOffReturnFlags), world, epoch,
                              reinterpret_cast<volatile int32_t*>(const_cast<uint8_t*>(win) + kOffGaveUp), status);
    __syncthreads();
    if (!ready) return;
    const uint16_t* y = reinterpret_cast<const uint16_t*>(win + off_y);
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<size_t>(T) * H) return;
    const size_t t = i / H, h = i % H;
    float mixed = 0.0f;
    for (uint32_t j = 0; j < K; ++j)
        mixed = __fadd_rn(mixed, __fmul_rn(contrib[t * K + j], decode_bf16(y[(t * K + j) * H + h])));
    mixed = round_bf16(mixed);
    const float sh = shared ? shared[i] : 0.0f;
    out[i] = round_bf16(__fadd_rn(mixed, sh));
}

EpState* ep_of(k3xb_ctx* ctx) { return static_cast<EpState*>(ctx->ep_state); }

void unmap_window(k3xb_ctx* ctx, EpState* ep) {
    EpWindow& w = ep->window;
    for (int g = 0; g < ep->world; ++g)
        if (g != ep->rank && w.peer[g]) cudaIpcCloseMemHandle(w.peer[g]);
    if (w.own) cudaFree(w.own);
    w = EpWindow{};
    (void)ctx;
}

// Makes the window hold `t` tokens x `k` slots of width `d` (collective: every
// rank makes the same calls with the same dims, so every rank grows at the
// same call). Growth drains this rank's stream, allocates and zeroes the new
// window, all-gathers the IPC handles over the communicator (which every
// rank enters only after draining its own stream, so no store into an old
// window is in flight) and maps the peers' windows.
int ensure_window(k3xb_ctx* ctx, EpState* ep, uint32_t t, uint32_t k, uint32_t d) {
    EpWindow& w = ep->window;
    if (w.own && t <= w.cap_t && k <= w.cap_k && d <= w.cap_d) return K3XB_OK;
    const uint32_t G = static_cast<uint32_t>(ep->world);
    const uint32_t ct = std::max(t, w.cap_t), ck = std::max(k, w.cap_k), cd = std::max(d, w.cap_d);
    int st;
    if ((st = ep_drain(ctx))) return st;
    unmap_window(ctx, ep);
    EpWindow n;
    n.cap_t = ct;
    n.cap_k = ck;
    n.cap_d = cd;
    uint64_t off = kHeaderBytes;
    const uint64_t meta = align256(uint64_t(G) * ct * ck * 4), rows = align256(uint64_t(G) * ct * cd * 4),
                   y = align256(uint64_t(ct) * ck * cd * 2);
    for (int b = 0; b < 2; ++b) {
        n.off_meta[b] = off;
        off += meta;
        n.off_rows[b] = off;
        off += rows;
        n.off_y[b] = off;
        off += y;
    }
    n.bytes = off;
    K3XB_CUDA(ctx, cudaMalloc(&n.own, n.bytes));
    K3XB_CUDA(ctx, cudaMemset(n.own, 0, kHeaderBytes));
    K3XB_CUDA(ctx, cudaDeviceSynchronize());
    n.peer[ep->rank] = n.own;
    ep->window = n;
    if (G == 1) return K3XB_OK;
    cudaIpcMemHandle_t mine;
    K3XB_CUDA(ctx, cudaIpcGetMemHandle(&mine, n.own));
    uint8_t* d_handles = nullptr;
    K3XB_CUDA(ctx, cudaMalloc(&d_handles, (G + 1) * sizeof(cudaIpcMemHandle_t)));
    std::vector<cudaIpcMemHandle_t> all(G);
    {
        const NcclApi& api = nccl();
        uint8_t* d_mine = d_handles + G * sizeof(cudaIpcMemHandle_t);
        cudaError_t ce = cudaMemcpy(d_mine, &mine, sizeof mine, cudaMemcpyHostToDevice);
        if (ce == cudaSuccess) {
            st = nccl_group(ctx, ep, "window handle exchange", [&]() -> ncclResult_t {
                return api.all_gather(d_mine, d_handles, sizeof mine, ncclUint8, ep->comm, ctx->stream);
            });
            if (!st) st = ep_drain(ctx);
            if (!st) ce = cudaMemcpy(all.data(), d_handles, G * sizeof mine, cudaMemcpyDeviceToHost);
        }
        cudaFree(d_handles);
        if (st) return st;
        if (ce != cudaSuccess) return cuda_fail(ctx, ce, "window handle exchange");
    }
    for (uint32_t g = 0; g < G; ++g) {
        if (static_cast<int>(g) == ep->rank) continue;
        void* p = nullptr;
        K3XB_CUDA(ctx, cudaIpcOpenMemHandle(&p, all[g], cudaIpcMemLazyEnablePeerAccess));
        ep->window.peer[g] = static_cast<uint8_t*>(p);
    }
    return K3XB_OK;
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

int ep_check_waits(k3xb_ctx* ctx) {
    EpState* ep = ep_of(ctx);
    if (!ep || !ep->window.own || ep->guard.aborted()) return K3XB_OK;
    int32_t gave_up = 0;
    K3XB_CUDA(ctx, cudaMemcpy(&gave_up, ep->window.own + kOffGaveUp, sizeof gave_up, cudaMemcpyDeviceToHost));
    if (gave_up) ep->guard.abort_now("a rank's exchange flags did not arrive within the bound");
    return K3XB_OK;
}

void release_ep(k3xb_ctx* ctx) {
    EpState* ep = ep_of(ctx);
    if (!ep) return;
    unmap_window(ctx, ep);
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

// Scratch of one EP layer call: the local plan over the received rows.
size_t ep_scratch_bytes(uint32_t G, uint32_t T, uint32_t K, uint32_t H, uint32_t E_r) {
    Sizer s;
    s.take<uint32_t>(E_r + 1);
    s.take<uint32_t>(E_r + 1);
    s.take<uint32_t>(static_cast<size_t>(G) * T * K);
    s.take<uint32_t>(static_cast<size_t>(G) * T * K);
    s.take<float>(static_cast<size_t>(G) * T * K);
    s.take<uint32_t>(1);
    (void)H;
    return s.used + 1024;
}

int ep_reserve(k3xb_ctx* ctx, uint32_t T, uint32_t K, uint32_t D) {
    EpState* ep = ep_of(ctx);
    if (!ep) return fail(ctx, K3XB_INVALID_STATE, "expert parallelism not initialised (k3xb_ep_init)");
    const CommWait w = ep->guard.check("expert parallelism");
    if (w != CommWait::ok) return guard_fail(ctx, ep, w);
    return ensure_window(ctx, ep, T, K, D);
}

int ep_moe_forward(k3xb_ctx* ctx, const k3xb_moe_layer& L, uint32_t E, const float* hidden, uint32_t T,
                   const uint32_t* ids, const float* contrib, const float* shared, void* region, float* out,
                   bool rows_bf16) {
    EpState* ep = ep_of(ctx);
    {   // a failure seen since the last call (a peer's) ends the exchange before new work is queued
        const CommWait w = ep->guard.check("expert parallelism");
        if (w != CommWait::ok) return guard_fail(ctx, ep, w);
    }
    const uint32_t G = static_cast<uint32_t>(ep->world), K = L.top_k, D = L.hidden, E_r = L.experts;
    if (D % 8) return fail(ctx, K3XB_INVALID_EXTENT, "expert parallelism: row width must be a multiple of 8");
    int st;
    if ((st = ensure_window(ctx, ep, T, K, D))) return st;
    const EpWindow& w = ep->window;
    const uint32_t epoch = ++ep->epoch, b = epoch & 1u;
    uint32_t* counters = reinterpret_cast<uint32_t*>(w.own + kOffCounters);
    int32_t* status = ctx->status_word;
    Carver c(region);
    k3xb_plan plan{};
    plan.group_expert = c.take<uint32_t>(E_r + 1);
    plan.group_offset = c.take<uint32_t>(E_r + 1);
    plan.assign_token = c.take<uint32_t>(static_cast<size_t>(G) * T * K);
    plan.assign_slot = c.take<uint32_t>(static_cast<size_t>(G) * T * K);
    plan.assign_contrib = c.take<float>(static_cast<size_t>(G) * T * K);
    plan.group_count = c.take<uint32_t>(1);
    plan.status = status;
    {
        PhaseScope ph(ctx, K3XB_PHASE_EP_DISPATCH);
        DispatchArgs a{};
        for (uint32_t g = 0; g < G; ++g) a.win[g] = w.peer[g];
        a.off_meta = w.off_meta[b];
        a.off_rows = w.off_rows[b];
        a.rank = static_cast<uint32_t>(ep->rank);
        a.world = G;
        a.epoch = epoch;
        a.T = T;
        a.K = K;
        a.D = D;
        a.E_r = E_r;
        a.rows_bf16 = rows_bf16 ? 1 : 0;
        a.done = counters;
        a.owner = L.ep_owner;
        a.status = status;
        ep_dispatch_kernel<<<dim3(T, G), 256, 0, ctx->stream>>>(hidden, ids, a);
        K3XB_LAUNCHED(ctx);
    }
    {
        PhaseScope ph(ctx, K3XB_PHASE_PLAN);
        ep_plan_kernel<<<1, 1024, (E_r + 1) * sizeof(uint32_t), ctx->stream>>>(w.own, w.off_meta[b], G * T, K, E_r,
                                                                               G, epoch, plan, status);
        K3XB_LAUNCHED(ctx);
    }
    EpTarget tgt{};
    for (uint32_t g = 0; g < G; ++g) tgt.win[g] = w.peer[g];
    tgt.y_off = w.off_y[b];
    tgt.flag_off = kOffReturnFlags;
    tgt.done = counters + 1;
    tgt.home_rows = T;
    tgt.rank = static_cast<uint32_t>(ep->rank);
    tgt.world = G;
    tgt.epoch = epoch;
    const uint8_t* rows = w.own + w.off_rows[b];
    // the default term count from the whole batch (every rank's tokens over
    // all experts), as the one-GPU layer chooses it
    k3xb_moe_layer LT = L;
    if (!LT.act_terms)
        LT.act_terms = static_cast<int32_t>(mxf4_default_terms(static_cast<uint64_t>(G) * T * K, E));
    if ((st = launch_mxf4_experts(ctx, LT, rows_bf16 ? nullptr : reinterpret_cast<const float*>(rows), G * T, plan,
                                  nullptr, nullptr, &tgt,
                                  rows_bf16 ? reinterpret_cast<const uint16_t*>(rows) : nullptr)))
        return st;
    const size_t n = static_cast<size_t>(T) * D;
    PhaseScope ph(ctx, K3XB_PHASE_COMBINE);
    ep_combine_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, ctx->stream>>>(
        w.own, w.off_y[b], ids, contrib, shared, T, K, D, G, epoch, out, status);
    K3XB_LAUNCHED(ctx);
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
    if (world > 8) return fail(ctx, K3XB_INVALID_EXTENT, "expert parallelism spans one box: at most 8 ranks");
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
