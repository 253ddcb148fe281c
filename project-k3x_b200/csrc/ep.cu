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
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "common.cuh"
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
    bool ok = false;
};

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
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.send && api.recv &&
                 api.group_start && api.group_end && api.error_string;
    });
    return api;
}

struct EpState {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
};

int nccl_fail(k3xb_ctx* ctx, ncclResult_t r, const char* where) {
    const char* msg = nccl().error_string ? nccl().error_string(r) : "?";
    return fail(ctx, K3XB_BACKEND_UNAVAILABLE, std::string(where) + ": " + msg);
}

#define K3XB_NCCL(ctx, call)                                                \
    do {                                                                    \
        ncclResult_t k3xb_nr_ = (call);                                     \
        if (k3xb_nr_ != ncclSuccess) return nccl_fail((ctx), k3xb_nr_, #call); \
    } while (0)

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
    K3XB_NCCL(ctx, api.group_start());
    for (int g = 0; g < ep->world; ++g) {
        K3XB_NCCL(ctx, api.send(static_cast<const char*>(send) + g * per_peer * elem, per_peer, type, g, ep->comm,
                                ctx->stream));
        K3XB_NCCL(ctx, api.recv(static_cast<char*>(recv) + g * per_peer * elem, per_peer, type, g, ep->comm,
                                ctx->stream));
    }
    K3XB_NCCL(ctx, api.group_end());
    return K3XB_OK;
}

}  // namespace

int ep_world(const k3xb_ctx* ctx) {
    return ctx->ep_state ? static_cast<const EpState*>(ctx->ep_state)->world : 0;
}

void release_ep(k3xb_ctx* ctx) {
    EpState* ep = ep_of(ctx);
    if (!ep) return;
    if (ep->comm && nccl().ok) nccl().comm_destroy(ep->comm);
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
        K3XB_NCCL(ctx, api.group_start());
        for (uint32_t g = 0; g < G; ++g) {
            const size_t nm_g = static_cast<size_t>(T) * K, nx_g = static_cast<size_t>(T) * H;
            K3XB_NCCL(ctx, api.send(send_meta + g * nm_g, nm_g, ncclUint32, g, ep->comm, ctx->stream));
            K3XB_NCCL(ctx, api.recv(recv_meta + g * nm_g, nm_g, ncclUint32, g, ep->comm, ctx->stream));
            K3XB_NCCL(ctx, api.send(send_x + g * nx_g, nx_g, ncclFloat32, g, ep->comm, ctx->stream));
            K3XB_NCCL(ctx, api.recv(recv_x + g * nx_g, nx_g, ncclFloat32, g, ep->comm, ctx->stream));
        }
        K3XB_NCCL(ctx, api.group_end());
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

int k3xb_ep_init(k3xb_ctx* ctx, const uint8_t* unique_id, int32_t rank, int32_t world) {
    K3XB_ENTER(ctx);
    if (!unique_id || world < 1 || rank < 0 || rank >= world)
        return fail(ctx, K3XB_INVALID_EXTENT, "ep_init arguments");
    if (ctx->ep_state) return fail(ctx, K3XB_INVALID_STATE, "expert parallelism already initialised");
    if (!nccl().ok) return fail(ctx, K3XB_BACKEND_UNAVAILABLE, "libnccl.so.2 could not be opened");
    K3XB_CUDA(ctx, cudaSetDevice(ctx->device));
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof id);
    auto* ep = new EpState();
    ep->rank = rank;
    ep->world = world;
    ncclResult_t r = nccl().comm_init_rank(&ep->comm, world, id, rank);
    if (r != ncclSuccess) {
        delete ep;
        return nccl_fail(ctx, r, "ncclCommInitRank");
    }
    ctx->ep_state = ep;
    return K3XB_OK;
}

int k3xb_ep_finalize(k3xb_ctx* ctx) {
    K3XB_ENTER(ctx);
    release_ep(ctx);
    return K3XB_OK;
}

}  // extern "C"
