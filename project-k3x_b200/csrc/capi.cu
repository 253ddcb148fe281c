// capi.cu — the extern "C" boundary of libk3xb (include/k3xb.h).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <new>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"
#include "profile.cuh"

namespace k3xb {

int fail(k3xb_ctx* ctx, int status, const std::string& message) {
    if (ctx) ctx->error = message;
    return status;
}

int cuda_fail(k3xb_ctx* ctx, cudaError_t err, const char* where) {
    std::string msg = std::string(where) + ": " + cudaGetErrorName(err) + " (" + cudaGetErrorString(err) + ")";
    return fail(ctx, K3XB_BACKEND_UNAVAILABLE, msg);
}

int stream_wait(k3xb_ctx* ctx) {
    if (ep_world(ctx)) return ep_drain(ctx);
    K3XB_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    return K3XB_OK;
}

int ensure_scratch(k3xb_ctx* ctx, size_t bytes, void** out) {
    if (bytes > ctx->scratch_bytes) {
        if (const int st = stream_wait(ctx)) return st;
        if (ctx->scratch) K3XB_CUDA(ctx, cudaFree(ctx->scratch));
        ctx->scratch = nullptr;
        ctx->scratch_bytes = 0;
        const size_t grown = bytes + bytes / 4 + (1u << 20);
        K3XB_CUDA(ctx, cudaMalloc(&ctx->scratch, grown));
        ctx->scratch_bytes = grown;
        ctx->stats.scratch_bytes = grown;
        if (grown > ctx->stats.peak_scratch_bytes) ctx->stats.peak_scratch_bytes = grown;
    }
    *out = ctx->scratch;
    return K3XB_OK;
}

// One device-held KDA state slot (k3xb_kda_block_held): two states in one
// allocation, `cur` the one that holds the slot's state; a call reads it and
// its commit writes the other, so nothing aliases.
struct KdaHeld {
    void* buf = nullptr;
    size_t state_bytes = 0, conv_n = 0, rec_n = 0;
    int cur = 0;
    bool valid = false;
};

void release_kda_held(k3xb_ctx* ctx) {
    if (!ctx->kda_held) return;
    KdaHeld* slots = static_cast<KdaHeld*>(ctx->kda_held);
    for (int i = 0; i < K3XB_KDA_HELD_SLOTS; ++i)
        if (slots[i].buf) cudaFree(slots[i].buf);
    delete[] slots;
    ctx->kda_held = nullptr;
}

int ensure_io(k3xb_ctx* ctx, size_t bytes, void** out) {
    if (bytes > ctx->io_bytes) {
        if (const int st = stream_wait(ctx)) return st;
        if (ctx->io) K3XB_CUDA(ctx, cudaFree(ctx->io));
        ctx->io = nullptr;
        ctx->io_bytes = 0;
        const size_t grown = bytes + bytes / 4 + (1u << 20);
        K3XB_CUDA(ctx, cudaMalloc(&ctx->io, grown));
        ctx->io_bytes = grown;
    }
    *out = ctx->io;
    return K3XB_OK;
}

namespace {

struct MoeScratch {
    float* logits;
    uint32_t* ids;
    float* contrib;
    k3xb_plan plan;
    float* act;
    float* slot_out;
    float* sg;
    float* su;
    float* sa;
    float* shared_out;
    uint16_t* sxb;   // tensor-core shared expert: input terms [2T][H]
    uint16_t* sbd;   // tensor-core shared expert: down operand [2T][Is]
    float* hidden;   // host path only
    float* out;      // host path only
    // LatentMoE only
    float* lat;      // [T][L] latent rows (the experts' input)
    float* mixed;    // [T][L]
    float* normed;   // [T][L]
    float* routed;   // [T][H]
    uint16_t* xt;    // linear input terms [2][T][max(H, L)]
};

// The experts' view of a layer: its width is the latent width for a
// LatentMoE layer, the hidden width otherwise.
k3xb_moe_layer expert_view(const k3xb_moe_layer& L) {
    k3xb_moe_layer v = L;
    if (L.latent) v.hidden = L.latent;
    v.latent = 0;
    return v;
}

// ep_E: the experts a route picks from in an expert-parallel layer (L then
// holds this rank's slice); 0 otherwise.
template <typename A>
void layout_moe(A& a, const k3xb_moe_layer& L, uint32_t T, bool host, MoeScratch* s, uint32_t ep_E = 0) {
    const size_t E = ep_E ? ep_E : L.experts, K = L.top_k, H = L.hidden, I = L.inter, Is = L.shared_inter;
    const size_t D = L.latent ? L.latent : H;   // the experts' width
    MoeScratch tmp{};
    MoeScratch& r = s ? *s : tmp;
    r.logits = a.template take<float>(T * E);
    r.ids = a.template take<uint32_t>(T * K);
    r.contrib = a.template take<float>(T * K);
    r.plan.group_expert = a.template take<uint32_t>(E);
    r.plan.group_offset = a.template take<uint32_t>(E + 1);
    r.plan.assign_token = a.template take<uint32_t>(T * K);
    r.plan.assign_slot = a.template take<uint32_t>(T * K);
    r.plan.assign_contrib = a.template take<float>(T * K);
    r.plan.group_count = a.template take<uint32_t>(1);
    r.act = L.engine == K3XB_ENGINE_SIMT ? a.template take<float>(T * K * I) : nullptr;
    r.slot_out = a.template take<float>(T * K * D);
    r.sg = a.template take<float>(T * Is);
    r.su = a.template take<float>(T * Is);
    r.sa = a.template take<float>(T * Is);
    r.shared_out = a.template take<float>(T * H);
    const bool tc_shared = L.engine == K3XB_ENGINE_MXF4 && L.shared_gate;
    r.sxb = tc_shared ? a.template take<uint16_t>(2 * T * H) : nullptr;
    r.sbd = tc_shared ? a.template take<uint16_t>(2 * T * Is) : nullptr;
    r.hidden = host ? a.template take<float>(T * H) : nullptr;
    r.out = host ? a.template take<float>(T * H) : nullptr;
    const bool latent = L.latent != 0;
    r.lat = latent ? a.template take<float>(T * D) : nullptr;
    r.mixed = latent ? a.template take<float>(T * D) : nullptr;
    r.normed = latent ? a.template take<float>(T * D) : nullptr;
    r.routed = latent ? a.template take<float>(T * H) : nullptr;
    r.xt = latent ? a.template take<uint16_t>(2 * T * (H > D ? H : D)) : nullptr;
}

int validate_layer(k3xb_ctx* ctx, const k3xb_moe_layer* L) {
    if (!L) return fail(ctx, K3XB_INVALID_EXTENT, "null layer");
    if (!L->hidden || !L->inter || !L->experts || !L->top_k || L->top_k > L->experts)
        return fail(ctx, K3XB_INVALID_EXTENT, "layer dimensions");
    if (L->hidden % 32 || L->inter % 32)
        return fail(ctx, K3XB_INVALID_MXFP4, "hidden and inter must be multiples of the MXFP4 group (32)");
    if (!L->router || !L->correction || !L->gate_packed || !L->gate_scales || !L->up_packed ||
        !L->up_scales || !L->down_packed || !L->down_scales)
        return fail(ctx, K3XB_INVALID_EXTENT, "missing layer weights");
    if (L->shared_gate && (!L->shared_up || !L->shared_down || !L->shared_inter))
        return fail(ctx, K3XB_INVALID_EXTENT, "incomplete shared expert");
    if (L->activation != K3XB_ACT_SWIGLU && L->activation != K3XB_ACT_SITU)
        return fail(ctx, K3XB_INVALID_STATE, "unknown activation");
    if (L->activation == K3XB_ACT_SITU && !(L->situ_beta > 0.0f))
        return fail(ctx, K3XB_INVALID_STATE, "SiTU beta must be positive");
    if (L->engine != K3XB_ENGINE_SIMT && L->engine != K3XB_ENGINE_MXF4)
        return fail(ctx, K3XB_INVALID_STATE, "unknown expert engine");
    if (L->latent) {   // official_moe.cpp:296, :323-331
        if (L->latent % 32)
            return fail(ctx, K3XB_INVALID_MXFP4, "latent must be a multiple of the MXFP4 group (32)");
        if (L->hidden % 8 || L->latent % 8)
            return fail(ctx, K3XB_INVALID_EXTENT, "latent projections need hidden and latent multiples of 8");
        if (!L->routed_down || !L->routed_norm || !L->routed_up)
            return fail(ctx, K3XB_INVALID_EXTENT, "missing latent projections");
        if (!(L->latent_eps > 0.0f)) return fail(ctx, K3XB_INVALID_EXTENT, "latent_eps must be positive");
    }
    return K3XB_OK;
}

// With ep_E != 0 the layer is expert parallel: L is this rank's slice of
// ep_E experts, the route picks from all ep_E, and the experts run through
// the exchange (ep.cu) with the plan and engine scratch in ep_region; the
// rows it sends are bf16-valued (the MoE input and the latent rows are).
int moe_forward_device(k3xb_ctx* ctx, const k3xb_moe_layer& L, const float* hidden, uint32_t T,
                       float* out, uint32_t* ids_out, float* contrib_out, MoeScratch& s, uint32_t ep_E = 0,
                       void* ep_region = nullptr) {
    const uint32_t E = ep_E ? ep_E : L.experts, K = L.top_k, H = L.hidden;
    uint32_t* ids = ids_out ? ids_out : s.ids;
    float* contrib = contrib_out ? contrib_out : s.contrib;
    s.plan.status = ctx->status_word;
    int st;
    if (L.shared_gate && L.engine == K3XB_ENGINE_MXF4) {
        K3XB_CUDA(ctx, cudaEventRecord(ctx->ev_fork, ctx->stream));
        K3XB_CUDA(ctx, cudaStreamWaitEvent(ctx->side_stream, ctx->ev_fork, 0));
        cudaStream_t main = ctx->stream;
        ctx->stream = ctx->side_stream;
        {
            PhaseScope ph(ctx, K3XB_PHASE_SHARED);
            st = launch_shared_tc(ctx, L, hidden, T, s.sxb, s.sbd, s.shared_out);
        }
        ctx->stream = main;
        if (st) return st;
        K3XB_CUDA(ctx, cudaEventRecord(ctx->ev_join, ctx->side_stream));
    }
    {
        PhaseScope ph(ctx, K3XB_PHASE_ROUTE);
        if ((st = launch_router_logits(ctx, hidden, T, H, L.router, E, s.logits))) return st;
        if ((st = launch_topk(ctx, s.logits, L.correction, T, E, K, ids, contrib, nullptr, s.plan.status)))
            return st;
    }
    if (ep_E) {
        const k3xb_moe_layer LE = expert_view(L);
        const float* shared = L.shared_gate ? s.shared_out : nullptr;
        if (!L.latent) {
            if (shared) K3XB_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, ctx->ev_join, 0));
            if ((st = ep_moe_forward(ctx, L, E, hidden, T, ids, contrib, shared, ep_region, out, true))) return st;
        } else {   // official_moe.cpp:296, the experts on latent rows, then :322-336
            {
                PhaseScope ph(ctx, K3XB_PHASE_LATENT);
                if ((st = launch_linear_bf16(ctx, hidden, L.routed_down, T, LE.hidden, H, 1, s.xt, s.lat))) return st;
            }
            if ((st = ep_moe_forward(ctx, LE, E, s.lat, T, ids, contrib, nullptr, ep_region, s.mixed, true)))
                return st;
            PhaseScope ph(ctx, K3XB_PHASE_LATENT);
            if ((st = launch_rms_norm(ctx, s.mixed, L.routed_norm, T, LE.hidden, L.latent_eps, s.normed))) return st;
            if ((st = launch_linear_bf16(ctx, s.normed, L.routed_up, T, H, LE.hidden, 1, s.xt, s.routed))) return st;
            if (shared) K3XB_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, ctx->ev_join, 0));
            const size_t n = static_cast<size_t>(T) * H;
            st = shared ? launch_residual(ctx, s.routed, shared, n, out) : launch_residual_round(ctx, s.routed, n, out);
            if (st) return st;
        }
        ++ctx->stats.moe_layer_calls;
        return K3XB_OK;
    }
    {
        PhaseScope ph(ctx, K3XB_PHASE_PLAN);
        if ((st = launch_plan(ctx, ids, contrib, T, K, E, s.plan))) return st;
    }
    const k3xb_moe_layer LE = expert_view(L);
    const uint32_t D = LE.hidden;
    const float* xe = hidden;
    if (L.latent) {   // official_moe.cpp:296: latent = bf16_matvec(hidden, routed_down)
        PhaseScope ph(ctx, K3XB_PHASE_LATENT);
        if ((st = launch_linear_bf16(ctx, hidden, L.routed_down, T, D, H, 1, s.xt, s.lat))) return st;
        xe = s.lat;
    }
    // the MXF4 engine stores its bf16-rounded expert rows as bf16 words (in
    // the slot_out region): half the bytes written and read by the combine
    uint16_t* y16 = L.engine == K3XB_ENGINE_MXF4 ? reinterpret_cast<uint16_t*>(s.slot_out) : nullptr;
    if (L.engine == K3XB_ENGINE_SIMT) {
        PhaseScope ph(ctx, K3XB_PHASE_EXPERT_GATEUP);
        if ((st = launch_simt_experts(ctx, LE, xe, T, s.plan, s.act, s.slot_out))) return st;
    } else {
        if ((st = launch_mxf4_experts(ctx, LE, xe, T, s.plan, nullptr, y16))) return st;
    }
    auto combine = [&](const float* sh, uint32_t width, float* dst) {
        return y16 ? launch_combine16(ctx, y16, contrib, sh, T, K, width, dst)
                   : launch_combine(ctx, s.slot_out, contrib, sh, T, K, width, dst);
    };
    const float* shared = nullptr;
    if (L.shared_gate && L.engine == K3XB_ENGINE_MXF4) {
        // the shared expert depends on the hidden rows only: it runs on the
        // side stream, forked before the router, on the SMs the router leaves
        // free; the main stream joins it before the combine
        K3XB_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, ctx->ev_join, 0));
        shared = s.shared_out;
    } else if (L.shared_gate) {
        PhaseScope ph(ctx, K3XB_PHASE_SHARED);
        const uint32_t Is = L.shared_inter;
        if ((st = launch_bf16_rows(ctx, hidden, L.shared_gate, T, Is, H, s.sg))) return st;
        if ((st = launch_bf16_rows(ctx, hidden, L.shared_up, T, Is, H, s.su))) return st;
        if ((st = launch_act(ctx, s.sg, s.su, static_cast<size_t>(T) * Is, L.activation, L.situ_beta,
                             L.situ_linear_beta, s.sa))) return st;
        if ((st = launch_bf16_rows(ctx, s.sa, L.shared_down, T, H, Is, s.shared_out))) return st;
        shared = s.shared_out;
    }
    if (L.latent) {
        {   // :313-322: mixed = round_bf16(slot-ordered combine), in the latent width
            PhaseScope ph(ctx, K3XB_PHASE_COMBINE);
            if ((st = combine(nullptr, D, s.mixed))) return st;
        }
        // :323-331: routed = bf16_matvec(normalized(mixed, routed_norm), routed_up); then
        // :336 combined = round_bf16(routed + shared)
        PhaseScope ph(ctx, K3XB_PHASE_LATENT);
        if ((st = launch_rms_norm(ctx, s.mixed, L.routed_norm, T, D, L.latent_eps, s.normed))) return st;
        if ((st = launch_linear_bf16(ctx, s.normed, L.routed_up, T, H, D, 1, s.xt, s.routed))) return st;
        const size_t n = static_cast<size_t>(T) * H;
        st = shared ? launch_residual(ctx, s.routed, shared, n, out) : launch_residual_round(ctx, s.routed, n, out);
        if (st) return st;
    } else {
        PhaseScope ph(ctx, K3XB_PHASE_COMBINE);
        if ((st = combine(shared, H, out))) return st;
    }
    ++ctx->stats.moe_layer_calls;
    return K3XB_OK;
}

}  // namespace

}  // namespace k3xb

using namespace k3xb;

extern "C" {

uint32_t k3xb_default_act_terms(uint64_t assignments, uint32_t experts) {
    return mxf4_default_terms(assignments, experts);
}

int k3xb_create(int device, k3xb_ctx** out) {
    if (!out) return K3XB_INVALID_EXTENT;
    *out = nullptr;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) return K3XB_BACKEND_UNAVAILABLE;
    if (device < 0 || device >= count) return K3XB_INVALID_EXTENT;
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return K3XB_BACKEND_UNAVAILABLE;
    if (prop.major != 10) return K3XB_UNSUPPORTED_ARCHITECTURE;   // sm_100a code only
    k3xb_ctx* ctx = new (std::nothrow) k3xb_ctx();
    if (!ctx) return K3XB_BACKEND_UNAVAILABLE;
    ctx->device = device;
    ctx->sm_count = prop.multiProcessorCount;
    if (cudaSetDevice(device) != cudaSuccess ||
        cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&ctx->side_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->ev_fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->ev_join, cudaEventDisableTiming) != cudaSuccess ||
        cudaMalloc(&ctx->status_word, sizeof(int32_t)) != cudaSuccess ||
        cudaMemset(ctx->status_word, 0, sizeof(int32_t)) != cudaSuccess) {
        k3xb_destroy(ctx);
        return K3XB_BACKEND_UNAVAILABLE;
    }
    ctx->stream = ctx->own_stream;
    *out = ctx;
    return K3XB_OK;
}

int k3xb_destroy(k3xb_ctx* ctx) {
    if (!ctx) return K3XB_OK;
    cudaSetDevice(ctx->device);
    if (ep_world(ctx)) ep_drain(ctx);   // bounded: a failed peer's exchange is aborted, not waited for
    if (ctx->own_stream) cudaStreamSynchronize(ctx->own_stream);
    if (ctx->side_stream) cudaStreamSynchronize(ctx->side_stream);
    if (ctx->scratch) cudaFree(ctx->scratch);
    if (ctx->io) cudaFree(ctx->io);
    if (ctx->status_word) cudaFree(ctx->status_word);
    release_mxf4_resources(ctx);
    release_resident(ctx);
    release_profiler(ctx);
    release_kda_held(ctx);
    release_ep(ctx);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    if (ctx->side_stream) cudaStreamDestroy(ctx->side_stream);
    if (ctx->ev_fork) cudaEventDestroy(ctx->ev_fork);
    if (ctx->ev_join) cudaEventDestroy(ctx->ev_join);
    delete ctx;
    return K3XB_OK;
}

int k3xb_last_error(const k3xb_ctx* ctx, char* buf, size_t len) {
    if (!ctx || !buf || !len) return K3XB_INVALID_EXTENT;
    std::snprintf(buf, len, "%s", ctx->error.c_str());
    return K3XB_OK;
}

int k3xb_set_stream(k3xb_ctx* ctx, void* stream) {
    K3XB_ENTER(ctx);
    ctx->stream = stream ? static_cast<cudaStream_t>(stream) : ctx->own_stream;
    return K3XB_OK;
}

int k3xb_sync(k3xb_ctx* ctx) {
    K3XB_ENTER(ctx);
    if (const int st = stream_wait(ctx)) return st;
    if (const int st = ep_check_waits(ctx)) return st;
    int32_t st = 0;
    K3XB_CUDA(ctx, cudaMemcpy(&st, ctx->status_word, sizeof st, cudaMemcpyDeviceToHost));
    if (st) {
        K3XB_CUDA(ctx, cudaMemset(ctx->status_word, 0, sizeof st));
        return fail(ctx, st, "device-side validation failed (route/plan input)");
    }
    return K3XB_OK;
}

int k3xb_get_stats(const k3xb_ctx* ctx, k3xb_stats* out) {
    if (!ctx || !out) return K3XB_INVALID_EXTENT;
    *out = ctx->stats;
    resident_stats(ctx, out);
    return K3XB_OK;
}

int k3xb_route(k3xb_ctx* ctx, const float* hidden, uint32_t T, uint32_t H, const uint16_t* router,
               const float* correction, uint32_t E, uint32_t K, uint32_t* ids, float* contrib,
               float* scores) {
    K3XB_ENTER(ctx);
    if (!T || !H || !E || !K || K > E || !hidden || !router || !correction || !ids || !contrib)
        return fail(ctx, K3XB_INVALID_EXTENT, "route arguments");
    void* base;
    Sizer sz;
    sz.take<float>(static_cast<size_t>(T) * E);
    int st = ensure_scratch(ctx, sz.used, &base);
    if (st) return st;
    Carver c(base);
    float* logits = c.take<float>(static_cast<size_t>(T) * E);
    PhaseScope ph(ctx, K3XB_PHASE_ROUTE);
    if ((st = launch_router_logits(ctx, hidden, T, H, router, E, logits))) return st;
    if ((st = launch_topk(ctx, logits, correction, T, E, K, ids, contrib, scores, ctx->status_word))) return st;
    ++ctx->stats.route_calls;
    return K3XB_OK;
}

int k3xb_router_logits(k3xb_ctx* ctx, const float* hidden, uint32_t T, uint32_t H, const uint16_t* router,
                       uint32_t E, float* logits) {
    K3XB_ENTER(ctx);
    if (!T || !H || !E || !hidden || !router || !logits) return fail(ctx, K3XB_INVALID_EXTENT, "router_logits arguments");
    PhaseScope ph(ctx, K3XB_PHASE_ROUTE);
    const int st = launch_router_logits(ctx, hidden, T, H, router, E, logits);
    if (st) return st;
    ++ctx->stats.route_calls;
    return K3XB_OK;
}

int k3xb_select_routing(k3xb_ctx* ctx, const float* scores, uint32_t T, uint32_t E, const float* bias, uint32_t K,
                        const k3xb_routing_policy* policy, uint32_t* ids, float* weights, uint32_t* selected,
                        uint32_t* escalated, float* stats) {
    K3XB_ENTER(ctx);
    if (!scores || !bias || !policy || !ids || !weights || !selected || !T)
        return fail(ctx, K3XB_INVALID_EXTENT, "select_routing arguments");
    // routing_policy.cpp:38-72
    auto allowed = [](uint32_t k) { return k == 4 || k == 6 || k == 8 || k == 12 || k == 16; };
    const k3xb_routing_policy& p = *policy;
    if (!E || !K || K > E) return fail(ctx, K3XB_INVALID_STATE, "invalid routing dimensions");
    if (K > 32 || E > 1024) return fail(ctx, K3XB_INVALID_EXTENT, "select_routing: natural_k <= 32, experts <= 1024");
    if (p.mode < K3XB_ROUTING_NATURAL || p.mode > K3XB_ROUTING_ADAPTIVE)
        return fail(ctx, K3XB_INVALID_STATE, "unknown routing mode");
    if (!std::isfinite(p.mass_target) || p.mass_target <= 0.0f || p.mass_target > 1.0f ||
        !std::isfinite(p.minimum_gap) || p.minimum_gap < 0.0f || p.minimum_gap > 1.0f)
        return fail(ctx, K3XB_INVALID_STATE, "invalid adaptive routing threshold");
    if (p.quality_floor_k != 0 &&
        (!allowed(p.quality_floor_k) || (p.mode != K3XB_ROUTING_NATURAL && p.quality_floor_k > K)))
        return fail(ctx, K3XB_INVALID_STATE, "invalid routing quality floor");
    if (p.mode == K3XB_ROUTING_FIXED && (!allowed(p.fixed_k) || p.fixed_k > K))
        return fail(ctx, K3XB_INVALID_STATE, "invalid fixed routing K");
    if (p.mode == K3XB_ROUTING_ADAPTIVE && K != 16)
        return fail(ctx, K3XB_INVALID_STATE, "adaptive routing requires natural Top-16");
    ++ctx->stats.route_calls;
    return launch_select_routing(ctx, scores, T, E, bias, K, p, ids, weights, selected, escalated, stats);
}

int k3xb_expert_major_plan(k3xb_ctx* ctx, const uint32_t* ids, const float* contrib, uint32_t T,
                           uint32_t K, uint32_t E, const k3xb_plan* plan) {
    K3XB_ENTER(ctx);
    if (!plan || !ids || !contrib) return fail(ctx, K3XB_INVALID_EXTENT, "plan arguments");
    if (!T || !K) return fail(ctx, K3XB_INVALID_EXTENT, "empty routes");   // expert_major.cpp:12-14
    k3xb_plan p = *plan;
    if (!p.status) p.status = ctx->status_word;
    PhaseScope ph(ctx, K3XB_PHASE_PLAN);
    return launch_plan(ctx, ids, contrib, T, K, E, p);
}

int k3xb_moe_layer_forward(k3xb_ctx* ctx, const k3xb_moe_layer* layer, const float* hidden, uint32_t T,
                           float* out, uint32_t* ids, float* contrib) {
    K3XB_ENTER(ctx);
    int st = validate_layer(ctx, layer);
    if (st) return st;
    if (!T || !hidden || !out) return fail(ctx, K3XB_INVALID_EXTENT, "moe forward arguments");
    Sizer sz;
    layout_moe(sz, *layer, T, false, nullptr);
    sz.used += mxf4_scratch_bytes(expert_view(*layer), T);
    void* base;
    if ((st = ensure_scratch(ctx, sz.used, &base))) return st;
    Carver c(base);
    MoeScratch s{};
    layout_moe(c, *layer, T, false, &s);
    set_mxf4_scratch(ctx, reinterpret_cast<char*>(base) + c.used);
    return moe_forward_device(ctx, *layer, hidden, T, out, ids, contrib, s);
}

int k3xb_moe_layer_forward_host(k3xb_ctx* ctx, const k3xb_moe_layer* layer, const float* hidden_host,
                                uint32_t T, float* out_host, uint32_t* ids_host, float* contrib_host) {
    K3XB_ENTER(ctx);
    int st = validate_layer(ctx, layer);
    if (st) return st;
    if (!T || !hidden_host || !out_host) return fail(ctx, K3XB_INVALID_EXTENT, "moe forward arguments");
    Sizer sz;
    layout_moe(sz, *layer, T, true, nullptr);
    sz.used += mxf4_scratch_bytes(expert_view(*layer), T);
    void* base;
    if ((st = ensure_scratch(ctx, sz.used, &base))) return st;
    Carver c(base);
    MoeScratch s{};
    layout_moe(c, *layer, T, true, &s);
    set_mxf4_scratch(ctx, reinterpret_cast<char*>(base) + c.used);
    const size_t hbytes = sizeof(float) * T * layer->hidden;
    K3XB_CUDA(ctx, cudaMemcpyAsync(s.hidden, hidden_host, hbytes, cudaMemcpyHostToDevice, ctx->stream));
    ctx->stats.h2d_bytes += hbytes;
    if ((st = moe_forward_device(ctx, *layer, s.hidden, T, s.out, nullptr, nullptr, s))) return st;
    K3XB_CUDA(ctx, cudaMemcpyAsync(out_host, s.out, hbytes, cudaMemcpyDeviceToHost, ctx->stream));
    ctx->stats.d2h_bytes += hbytes;
    const size_t rbytes = static_cast<size_t>(T) * layer->top_k * 4;
    if (ids_host) {
        K3XB_CUDA(ctx, cudaMemcpyAsync(ids_host, s.ids, rbytes, cudaMemcpyDeviceToHost, ctx->stream));
        ctx->stats.d2h_bytes += rbytes;
    }
    if (contrib_host) {
        K3XB_CUDA(ctx, cudaMemcpyAsync(contrib_host, s.contrib, rbytes, cudaMemcpyDeviceToHost, ctx->stream));
        ctx->stats.d2h_bytes += rbytes;
    }
    return k3xb_sync(ctx);
}

int k3xb_moe_experts(k3xb_ctx* ctx, const k3xb_moe_layer* layer, const float* hidden, uint32_t T,
                     const k3xb_plan* plan, float* slot_out) {
    K3XB_ENTER(ctx);
    int st = validate_layer(ctx, layer);
    if (st) return st;
    if (!T || !hidden || !plan || !slot_out) return fail(ctx, K3XB_INVALID_EXTENT, "experts arguments");
    Sizer sz;
    sz.take<float>(static_cast<size_t>(T) * layer->top_k * layer->inter);
    sz.used += mxf4_scratch_bytes(expert_view(*layer), T);
    void* base;
    if ((st = ensure_scratch(ctx, sz.used, &base))) return st;
    Carver c(base);
    float* act = c.take<float>(static_cast<size_t>(T) * layer->top_k * layer->inter);
    set_mxf4_scratch(ctx, reinterpret_cast<char*>(base) + c.used);
    const k3xb_moe_layer LE = expert_view(*layer);   // rows of the experts' width (latent rows for LatentMoE)
    if (layer->engine == K3XB_ENGINE_SIMT) return launch_simt_experts(ctx, LE, hidden, T, *plan, act, slot_out);
    return launch_mxf4_experts(ctx, LE, hidden, T, *plan, slot_out);
}

int k3xb_expert_grid_host(k3xb_ctx* ctx, const k3xb_moe_layer* layer, const uint32_t* expert_ids, uint32_t n,
                          const float* inputs_host, uint32_t T, float* out_host) {
    K3XB_ENTER(ctx);
    if (!layer || !expert_ids || !inputs_host || !out_host || !T || !n)
        return fail(ctx, K3XB_INVALID_EXTENT, "expert grid arguments");
    k3xb_moe_layer L = expert_view(*layer);   // inputs are rows of the experts' width
    L.top_k = n;   // every token through each listed expert: one routing slot per expert
    L.shared_gate = L.shared_up = L.shared_down = nullptr;
    L.shared_inter = 0;
    if (!L.hidden || !L.inter || !L.experts || n > L.experts || n > 32)
        return fail(ctx, K3XB_INVALID_EXTENT, "expert grid: 1 <= experts listed <= min(32, stack size)");
    if (L.hidden % 32 || L.inter % 32)
        return fail(ctx, K3XB_INVALID_MXFP4, "hidden and inter must be multiples of the MXFP4 group (32)");
    if (!L.gate_packed || !L.gate_scales || !L.up_packed || !L.up_scales || !L.down_packed || !L.down_scales)
        return fail(ctx, K3XB_INVALID_EXTENT, "missing expert weights");
    if (L.activation != K3XB_ACT_SWIGLU && L.activation != K3XB_ACT_SITU)
        return fail(ctx, K3XB_INVALID_STATE, "unknown activation");
    if (L.activation == K3XB_ACT_SITU && !(L.situ_beta > 0.0f))
        return fail(ctx, K3XB_INVALID_STATE, "SiTU beta must be positive");
    if (L.engine != K3XB_ENGINE_SIMT && L.engine != K3XB_ENGINE_MXF4)
        return fail(ctx, K3XB_INVALID_STATE, "unknown expert engine");
    // the reference rejects a repeated expert (backend_cpu.cpp:226-233 by tensor id)
    std::vector<uint8_t> seen(L.experts, 0);
    for (uint32_t j = 0; j < n; ++j) {
        if (expert_ids[j] >= L.experts || seen[expert_ids[j]])
            return fail(ctx, K3XB_INVALID_MXFP4, "expert grid: expert ids must be distinct and in the stack");
        seen[expert_ids[j]] = 1;
    }
    const size_t H = L.hidden;
    Sizer sz;
    layout_moe(sz, L, T, true, nullptr);
    sz.used += mxf4_scratch_bytes(L, T);
    void* base;
    int st;
    if ((st = ensure_scratch(ctx, sz.used, &base))) return st;
    Carver c(base);
    MoeScratch s{};
    layout_moe(c, L, T, true, &s);
    set_mxf4_scratch(ctx, reinterpret_cast<char*>(base) + c.used);
    std::vector<uint32_t> ids(static_cast<size_t>(T) * n);
    std::vector<float> contrib(static_cast<size_t>(T) * n, 1.0f);
    for (uint32_t t = 0; t < T; ++t)
        for (uint32_t j = 0; j < n; ++j) ids[static_cast<size_t>(t) * n + j] = expert_ids[j];
    const size_t hbytes = sizeof(float) * T * H;
    K3XB_CUDA(ctx, cudaMemcpyAsync(s.hidden, inputs_host, hbytes, cudaMemcpyHostToDevice, ctx->stream));
    K3XB_CUDA(ctx, cudaMemcpyAsync(s.ids, ids.data(), ids.size() * 4, cudaMemcpyHostToDevice, ctx->stream));
    K3XB_CUDA(ctx, cudaMemcpyAsync(s.contrib, contrib.data(), contrib.size() * 4, cudaMemcpyHostToDevice,
                                   ctx->stream));
    ctx->stats.h2d_bytes += hbytes + ids.size() * 8;
    s.plan.status = ctx->status_word;
    if ((st = launch_plan(ctx, s.ids, s.contrib, T, n, L.experts, s.plan))) return st;
    st = L.engine == K3XB_ENGINE_SIMT ? launch_simt_experts(ctx, L, s.hidden, T, s.plan, s.act, s.slot_out)
                                      : launch_mxf4_experts(ctx, L, s.hidden, T, s.plan, s.slot_out);
    if (st) return st;
    // slot_out [T][n][H] -> out [n][T][H]
    for (uint32_t j = 0; j < n; ++j)
        K3XB_CUDA(ctx, cudaMemcpy2DAsync(out_host + static_cast<size_t>(j) * T * H, H * sizeof(float),
                                         s.slot_out + static_cast<size_t>(j) * H, n * H * sizeof(float),
                                         H * sizeof(float), T, cudaMemcpyDeviceToHost, ctx->stream));
    ctx->stats.d2h_bytes += static_cast<uint64_t>(n) * hbytes;
    return k3xb_sync(ctx);
}

int k3xb_official_moe_ffn_host(k3xb_ctx* ctx, const k3xb_moe_layer* tail, const k3xb_moe_layer* slots, uint32_t K,
                               const float* contributions_host, const float* hidden_host, const float* prefix_host,
                               float* out_host) {
    K3XB_ENTER(ctx);
    if (!tail || !slots || !K || K > 64 || !contributions_host || !hidden_host || !prefix_host || !out_host)
        return fail(ctx, K3XB_INVALID_EXTENT, "official moe ffn arguments (1 <= slots <= 64)");
    const k3xb_moe_layer& W = *tail;
    const uint32_t H = W.hidden, D = W.latent, Is = W.shared_gate ? W.shared_inter : 0;
    if (!H || !D || H % 8 || D % 32 || !W.routed_down || !W.routed_norm || !W.routed_up || !(W.latent_eps > 0.0f))
        return fail(ctx, K3XB_INVALID_EXTENT, "official moe ffn: latent projections (hidden % 8, latent % 32)");
    if (W.shared_gate && (!W.shared_up || !W.shared_down || !Is))
        return fail(ctx, K3XB_INVALID_EXTENT, "official moe ffn: incomplete shared expert");
    if (W.activation != K3XB_ACT_SWIGLU && W.activation != K3XB_ACT_SITU)
        return fail(ctx, K3XB_INVALID_STATE, "unknown activation");
    if (W.activation == K3XB_ACT_SITU && !(W.situ_beta > 0.0f))
        return fail(ctx, K3XB_INVALID_STATE, "SiTU beta must be positive");
    // every slot: one expert of the latent width, the tail's activation
    const uint32_t I = slots[0].inter;
    const int engine = slots[0].engine;
    for (uint32_t k = 0; k < K; ++k) {
        const k3xb_moe_layer& e = slots[k];
        const uint32_t width = e.latent ? e.latent : e.hidden;   // the expert's input width
        if (e.experts != 1 || width != D || e.inter != I || !I || I % 32 || e.engine != engine ||
            !e.gate_packed || !e.gate_scales || !e.up_packed || !e.up_scales || !e.down_packed || !e.down_scales)
            return fail(ctx, K3XB_INVALID_MXFP4,
                        "official moe ffn: each slot one expert of the latent width, one inter, one engine");
        if (engine == K3XB_ENGINE_MXF4 && (!e.gate_scales_tc || !e.up_scales_tc || !e.down_scales_tc))
            return fail(ctx, K3XB_INVALID_MXFP4, "official moe ffn: the tcgen05 engine needs the *_scales_tc copies");
    }
    if (engine != K3XB_ENGINE_SIMT && engine != K3XB_ENGINE_MXF4)
        return fail(ctx, K3XB_INVALID_STATE, "unknown expert engine");
    k3xb_moe_layer E1 = slots[0];   // the per-slot view the engines run
    E1.hidden = D;
    E1.top_k = 1;
    E1.latent = 0;
    E1.shared_gate = E1.shared_up = E1.shared_down = nullptr;
    E1.shared_inter = 0;
    E1.activation = W.activation;
    E1.situ_beta = W.situ_beta;
    E1.situ_linear_beta = W.situ_linear_beta;

    const size_t HD = H > D ? H : D;
    Sizer sz;
    sz.take<float>(2 * size_t(H) + K);            // hidden, prefix, contributions (one upload)
    sz.take<uint32_t>(2);                         // the one-token plan's route: expert 0, contribution 1
    sz.take<float>(D);                            // latent
    sz.take<uint16_t>(2 * HD);                    // linear input terms
    sz.take<float>(size_t(K) * D);                // slot outputs
    for (int i = 0; i < 2; ++i) sz.take<float>(D);            // mixed, normed
    for (int i = 0; i < 3; ++i) sz.take<float>(H);            // routed, shared, combined
    for (int i = 0; i < 3; ++i) sz.take<float>(Is ? Is : 1);  // shared gate, up, activation
    sz.take<uint16_t>(2 * size_t(H));             // tensor-core shared expert: input terms
    sz.take<uint16_t>(2 * size_t(Is ? Is : 1));   // and its down operand
    sz.take<float>(H);                            // out
    for (int i = 0; i < 2; ++i) sz.take<uint32_t>(2);         // plan groups
    for (int i = 0; i < 4; ++i) sz.take<uint32_t>(1);         // plan assignments, group count
    sz.take<float>(I);                            // SIMT activations
    sz.used += mxf4_scratch_bytes(E1, 1) + 1024;
    void* base;
    int st;
    if ((st = ensure_scratch(ctx, sz.used, &base))) return st;
    Carver c(base);
    float* in = c.take<float>(2 * size_t(H) + K);
    float *hidden = in, *prefix = in + H, *contrib = in + 2 * size_t(H);
    uint32_t* route1 = c.take<uint32_t>(2);
    float* lat = c.take<float>(D);
    uint16_t* xt = c.take<uint16_t>(2 * HD);
    float* slot_out = c.take<float>(size_t(K) * D);
    float* mixed = c.take<float>(D);
    float* normed = c.take<float>(D);
    float* routed = c.take<float>(H);
    float* shared = c.take<float>(H);
    float* combined = c.take<float>(H);
    float* sg = c.take<float>(Is ? Is : 1);
    float* su = c.take<float>(Is ? Is : 1);
    float* sa = c.take<float>(Is ? Is : 1);
    uint16_t* sxb = c.take<uint16_t>(2 * size_t(H));
    uint16_t* sbd = c.take<uint16_t>(2 * size_t(Is ? Is : 1));
    float* out = c.take<float>(H);
    k3xb_plan plan{};
    plan.group_expert = c.take<uint32_t>(2);
    plan.group_offset = c.take<uint32_t>(2);
    plan.assign_token = c.take<uint32_t>(1);
    plan.assign_slot = c.take<uint32_t>(1);
    plan.assign_contrib = c.take<float>(1);
    plan.group_count = c.take<uint32_t>(1);
    plan.status = ctx->status_word;
    float* act = c.take<float>(I);
    set_mxf4_scratch(ctx, reinterpret_cast<char*>(base) + c.used);

    // official_moe_ffn inputs: hidden and prefix of one position, the route's contributions
    const size_t hbytes = sizeof(float) * H;
    K3XB_CUDA(ctx, cudaMemcpyAsync(hidden, hidden_host, hbytes, cudaMemcpyHostToDevice, ctx->stream));
    K3XB_CUDA(ctx, cudaMemcpyAsync(prefix, prefix_host, hbytes, cudaMemcpyHostToDevice, ctx->stream));
    K3XB_CUDA(ctx, cudaMemcpyAsync(contrib, contributions_host, sizeof(float) * K, cudaMemcpyHostToDevice,
                                   ctx->stream));
    const uint32_t one_route[2] = {0u, 0x3f800000u};   // expert 0, contribution 1.0f
    K3XB_CUDA(ctx, cudaMemcpyAsync(route1, one_route, sizeof one_route, cudaMemcpyHostToDevice, ctx->stream));
    ctx->stats.h2d_bytes += 2 * hbytes + sizeof(float) * K + sizeof one_route;

    // backend_cuda.cu:4036-4106 in this library's arithmetic (official_moe.cpp:296-341)
    {
        PhaseScope ph(ctx, K3XB_PHASE_LATENT);   // :296 latent = bf16_matvec(hidden, routed_down)
        if ((st = launch_linear_bf16(ctx, hidden, W.routed_down, 1, D, H, 1, xt, lat))) return st;
    }
    if ((st = launch_plan(ctx, route1, reinterpret_cast<const float*>(route1 + 1), 1, 1, 1, plan))) return st;
    for (uint32_t k = 0; k < K; ++k) {   // slot k's expert, its output unweighted in slot k
        k3xb_moe_layer Ek = E1;
        Ek.gate_packed = slots[k].gate_packed;
        Ek.gate_scales = slots[k].gate_scales;
        Ek.up_packed = slots[k].up_packed;
        Ek.up_scales = slots[k].up_scales;
        Ek.down_packed = slots[k].down_packed;
        Ek.down_scales = slots[k].down_scales;
        Ek.gate_scales_tc = slots[k].gate_scales_tc;
        Ek.up_scales_tc = slots[k].up_scales_tc;
        Ek.down_scales_tc = slots[k].down_scales_tc;
        float* yk = slot_out + size_t(k) * D;
        if (engine == K3XB_ENGINE_SIMT) {
            PhaseScope ph(ctx, K3XB_PHASE_EXPERT_GATEUP);
            st = launch_simt_experts(ctx, Ek, lat, 1, plan, act, yk);
        } else {
            st = launch_mxf4_experts(ctx, Ek, lat, 1, plan, yk);
        }
        if (st) return st;
    }
    {   // :313-322 mixed = round_bf16(slot-ordered combine)
        PhaseScope ph(ctx, K3XB_PHASE_COMBINE);
        if ((st = launch_combine(ctx, slot_out, contrib, nullptr, 1, K, D, mixed))) return st;
    }
    {   // :323-331 routed = bf16_matvec(normalized(mixed, routed_norm), routed_up)
        PhaseScope ph(ctx, K3XB_PHASE_LATENT);
        if ((st = launch_rms_norm(ctx, mixed, W.routed_norm, 1, D, W.latent_eps, normed))) return st;
        if ((st = launch_linear_bf16(ctx, normed, W.routed_up, 1, H, D, 1, xt, routed))) return st;
    }
    if (Is) {   // :332-335 the shared expert on the hidden row, with the layer path's kernels
        PhaseScope ph(ctx, K3XB_PHASE_SHARED);
        if (engine == K3XB_ENGINE_MXF4 && H % 128 == 0 && Is % 128 == 0) {
            if ((st = launch_shared_tc(ctx, W, hidden, 1, sxb, sbd, shared))) return st;
        } else {
            if ((st = launch_bf16_rows(ctx, hidden, W.shared_gate, 1, Is, H, sg))) return st;
            if ((st = launch_bf16_rows(ctx, hidden, W.shared_up, 1, Is, H, su))) return st;
            if ((st = launch_act(ctx, sg, su, Is, W.activation, W.situ_beta, W.situ_linear_beta, sa))) return st;
            if ((st = launch_bf16_rows(ctx, sa, W.shared_down, 1, H, Is, shared))) return st;
        }
        st = launch_residual(ctx, routed, shared, H, combined);   // :336 round_bf16(routed + shared)
    } else {
        st = launch_residual_round(ctx, routed, H, combined);
    }
    if (st) return st;
    // :337-341 out = round_bf16(round_bf16(prefix) + combined)
    if ((st = launch_residual(ctx, prefix, combined, H, out))) return st;
    K3XB_CUDA(ctx, cudaMemcpyAsync(out_host, out, hbytes, cudaMemcpyDeviceToHost, ctx->stream));
    ctx->stats.d2h_bytes += hbytes;
    ++ctx->stats.moe_layer_calls;
    return k3xb_sync(ctx);
}

// ---- KDA -------------------------------------------------------------------

namespace {

struct KdaSchedule {
    // per visited entry: node, depth (1 = root) and flags (kKdaReset: reload
    // the prefix state first; kKdaReplay: recompute only, no output)
    std::vector<int32_t> order, depth, from_stack;
    uint32_t levels = 0;
};

constexpr int32_t kKdaReset = 1, kKdaReplay = 2;

// DFS preorder of the draft forest (roots = parent -1, children in index
// order). A node whose parent is not the node visited just before it starts
// from the prefix state: the entries before it replay its ancestors root..
// parent (no output), so no state is kept per depth.
int schedule_tree(k3xb_ctx* ctx, const int32_t* parent, uint32_t n, KdaSchedule& out) {
    std::vector<std::vector<int32_t>> children(n);
    std::vector<int32_t> roots;
    for (uint32_t i = 0; i < n; ++i) {
        if (parent[i] < -1 || parent[i] >= static_cast<int32_t>(i))
            return fail(ctx, K3XB_INVALID_EXTENT, "draft tree: parent[n] must be -1 or < n");
        if (parent[i] < 0) roots.push_back(static_cast<int32_t>(i));
        else children[parent[i]].push_back(static_cast<int32_t>(i));
    }
    std::vector<std::pair<int32_t, int32_t>> stack;   // (node, depth)
    for (auto it = roots.rbegin(); it != roots.rend(); ++it) stack.push_back({*it, 1});
    int32_t prev = -1;
    std::vector<int32_t> path;
    while (!stack.empty()) {
        auto [node, d] = stack.back();
        stack.pop_back();
        const int32_t p = parent[node];
        int32_t flags = 0;
        if (p != prev && !out.order.empty()) {   // off the current chain: from the prefix
            path.clear();
            for (int32_t x = p; x >= 0; x = parent[x]) path.push_back(x);
            flags = kKdaReset;
            for (size_t i = path.size(); i-- > 0;) {
                out.order.push_back(path[i]);
                out.depth.push_back(static_cast<int32_t>(path.size() - i));
                out.from_stack.push_back(flags | kKdaReplay);
                flags = 0;
            }
        }
        out.order.push_back(node);
        out.depth.push_back(d);
        out.from_stack.push_back(flags);
        for (auto c = children[node].rbegin(); c != children[node].rend(); ++c) stack.push_back({*c, d + 1});
        prev = node;
    }
    return K3XB_OK;
}

int kda_common(k3xb_ctx* ctx, const float* state, uint32_t nodes, uint32_t S, uint32_t heads,
               uint32_t head_dim, const float* q, const float* k, const float* v, const float* ld,
               const float* beta, float* out, float* state_out, const KdaSchedule& sch) {
    const size_t visit = sch.order.size();
    Sizer sz;
    sz.take<int32_t>(3 * visit + 3);
    void* base;
    int st = ensure_scratch(ctx, sz.used, &base);
    if (st) return st;
    Carver c(base);
    int32_t* d = c.take<int32_t>(3 * visit + 3);
    std::vector<int32_t> packed;
    packed.insert(packed.end(), sch.order.begin(), sch.order.end());
    packed.insert(packed.end(), sch.depth.begin(), sch.depth.end());
    packed.insert(packed.end(), sch.from_stack.begin(), sch.from_stack.end());
    if (!packed.empty())
        K3XB_CUDA(ctx, cudaMemcpyAsync(d, packed.data(), packed.size() * 4, cudaMemcpyHostToDevice, ctx->stream));
    st = launch_kda(ctx, state, d, d + visit, d + 2 * visit, static_cast<uint32_t>(visit), nodes, S, heads,
                    head_dim, q, k, v, ld, beta, out, state_out, sch.levels);
    ++ctx->stats.kda_calls;
    return st;
}

}  // namespace

int k3xb_kda_tree(k3xb_ctx* ctx, const float* state, const int32_t* parent, uint32_t nodes,
                  uint32_t S, uint32_t heads, uint32_t head_dim, const float* q, const float* k,
                  const float* v, const float* ld, const float* beta, float* out) {
    K3XB_ENTER(ctx);
    if (!state || !parent || !nodes || !S || !heads || !q || !k || !v || !ld || !beta || !out)
        return fail(ctx, K3XB_INVALID_EXTENT, "kda_tree arguments");
    KdaSchedule sch;
    int st = schedule_tree(ctx, parent, nodes, sch);
    if (st) return st;
    PhaseScope ph(ctx, K3XB_PHASE_KDA_RECURRENCE);
    return kda_common(ctx, state, nodes, S, heads, head_dim, q, k, v, ld, beta, out, nullptr, sch);
}

int k3xb_kda_commit(k3xb_ctx* ctx, const float* state, const int32_t* parent, uint32_t nodes, uint32_t S,
                    uint32_t heads, uint32_t head_dim, const float* q, const float* k, const float* v,
                    const float* ld, const float* beta, const int32_t* commit_node, float* state_out) {
    K3XB_ENTER(ctx);
    if (!state || !parent || !S || !heads || !commit_node || !state_out)
        return fail(ctx, K3XB_INVALID_EXTENT, "kda_commit arguments");
    for (uint32_t i = 0; i < nodes; ++i)
        if (parent[i] < -1 || parent[i] >= static_cast<int32_t>(i))
            return fail(ctx, K3XB_INVALID_EXTENT, "draft tree: parent[n] must be -1 or < n");
    // sequences may commit different nodes: group them by path
    PhaseScope ph(ctx, K3XB_PHASE_COMMIT);
    const size_t sstride = static_cast<size_t>(heads) * head_dim * head_dim;
    for (uint32_t s = 0; s < S; ++s) {
        const int32_t node = commit_node[s];
        if (node < -1 || node >= static_cast<int32_t>(nodes))
            return fail(ctx, K3XB_INVALID_EXTENT, "commit node out of range");
        KdaSchedule sch;
        std::vector<int32_t> path;
        for (int32_t x = node; x >= 0; x = parent[x]) path.push_back(x);
        for (size_t i = 0; i < path.size(); ++i) {
            sch.order.push_back(path[path.size() - 1 - i]);
            sch.depth.push_back(static_cast<int32_t>(i + 1));
            sch.from_stack.push_back(0);
        }
        const size_t io = static_cast<size_t>(s) * nodes * heads * head_dim;
        int st = kda_common(ctx, state + s * sstride, nodes, 1, heads, head_dim, q + io, k + io, v + io,
                            ld + io, beta + static_cast<size_t>(s) * nodes * heads, nullptr,
                            state_out + s * sstride, sch);
        if (st) return st;
    }
    return K3XB_OK;
}

// ---- acceptance --------------------------------------------------------------

int k3xb_accept_greedy(k3xb_ctx* ctx, const float* logits, const uint32_t* drafts, uint32_t S, uint32_t p,
                       uint32_t V, uint32_t* targets, uint32_t* accepted, uint32_t* committed,
                       uint32_t* count) {
    K3XB_ENTER(ctx);
    if (!logits || (!drafts && p) || !S || !V || !accepted || !committed || !count)
        return fail(ctx, K3XB_INVALID_EXTENT, "accept_greedy arguments");
    uint32_t* t = targets;
    if (!t) {
        void* base;
        int st = ensure_scratch(ctx, sizeof(uint32_t) * S * (p + 1) + 256, &base);
        if (st) return st;
        t = static_cast<uint32_t*>(base);
    }
    ++ctx->stats.accept_calls;
    PhaseScope ph(ctx, K3XB_PHASE_ACCEPT);
    return launch_accept_greedy(ctx, logits, drafts, S, p, V, t, accepted, committed, count);
}

int k3xb_accept_rejection(k3xb_ctx* ctx, const float* tl, const float* dl, const uint32_t* drafts, uint32_t S,
                          uint32_t p, uint32_t V, float temperature, uint64_t seed, uint64_t seq_base,
                          uint32_t* accepted, uint32_t* committed, uint32_t* count) {
    K3XB_ENTER(ctx);
    if (!tl || (p && (!dl || !drafts)) || !S || !V || !accepted || !committed || !count)
        return fail(ctx, K3XB_INVALID_EXTENT, "accept_rejection arguments");
    if (!(temperature > 0.0f)) return fail(ctx, K3XB_INVALID_EXTENT, "temperature must be positive");
    void* base;
    int st = ensure_scratch(ctx, sizeof(double) * 2 * S * (p + 1) + 512, &base);
    if (st) return st;
    Carver c(base);
    double* pd = c.take<double>(static_cast<size_t>(S) * (p + 1));
    double* qd = c.take<double>(static_cast<size_t>(S) * (p + 1));
    ++ctx->stats.accept_calls;
    PhaseScope ph(ctx, K3XB_PHASE_ACCEPT);
    return launch_accept_rejection(ctx, tl, dl, drafts, S, p, V, temperature, seed, seq_base, pd, qd,
                                   accepted, committed, count);
}

// ---- synthetic data --------------------------------------------------------------

int k3xb_fill_normal_f32(k3xb_ctx* ctx, float* out, size_t n, uint64_t seed, uint64_t stream, float mean,
                         float sigma) {
    K3XB_ENTER(ctx);
    if (!out || !n) return fail(ctx, K3XB_INVALID_EXTENT, "fill arguments");
    return launch_fill_normal_f32(ctx, out, n, seed, stream, mean, sigma);
}

int k3xb_fill_normal_bf16(k3xb_ctx* ctx, uint16_t* out, size_t n, uint64_t seed, uint64_t stream, float sigma) {
    K3XB_ENTER(ctx);
    if (!out || !n) return fail(ctx, K3XB_INVALID_EXTENT, "fill arguments");
    return launch_fill_normal_bf16(ctx, out, n, seed, stream, sigma);
}

int k3xb_quantize_mxfp4(k3xb_ctx* ctx, const float* x, size_t rows, size_t cols, uint8_t* packed,
                        uint8_t* scales) {
    K3XB_ENTER(ctx);
    if (!x || !packed || !scales || !rows || !cols || cols % 32)
        return fail(ctx, K3XB_INVALID_MXFP4, "quantize arguments (cols % 32 == 0)");
    return launch_quantize_mxfp4(ctx, x, rows, cols, packed, scales);
}

int k3xb_linear_bf16(k3xb_ctx* ctx, const float* x, uint32_t tokens, uint32_t in_features, const uint16_t* weight,
                     uint32_t out_features, int32_t round_output, float* out) {
    K3XB_ENTER(ctx);
    if (!x || !weight || !out || !tokens || !in_features || !out_features)
        return fail(ctx, K3XB_INVALID_EXTENT, "linear arguments");
    void* base;
    int st = ensure_scratch(ctx, linear_scratch_bytes(tokens, in_features), &base);
    if (st) return st;
    return launch_linear_bf16(ctx, x, weight, tokens, out_features, in_features, round_output,
                              static_cast<uint16_t*>(base), out);
}

int k3xb_prepare_mxfp4_scales(k3xb_ctx* ctx, const uint8_t* scales, size_t rows, size_t cols, uint8_t* out) {
    K3XB_ENTER(ctx);
    return prepare_mxfp4_scales(ctx, scales, rows, cols, out);
}

int k3xb_fill_normal_mxfp4(k3xb_ctx* ctx, uint8_t* packed, uint8_t* scales, size_t rows, size_t cols,
                           uint64_t seed, uint64_t stream, float sigma) {
    K3XB_ENTER(ctx);
    if (!packed || !scales || !rows || !cols || cols % 32)
        return fail(ctx, K3XB_INVALID_MXFP4, "fill arguments (cols % 32 == 0)");
    return launch_fill_normal_mxfp4(ctx, packed, scales, rows, cols, seed, stream, sigma);
}

}  // extern "C"

// ---- full KDA block and the KDA + MoE layer ----------------------------------

namespace {

// Per-node values a commit replays (recurrence inputs) and reads (projected
// q, k, v for the conv windows).
struct KdaTrace {
    float *qn, *kn, *cv, *ld, *be, *pq, *pk, *pv;
};

template <typename A>
void layout_trace(A& a, size_t T, size_t P, size_t h, KdaTrace* out) {
    KdaTrace tmp{};
    KdaTrace& r = out ? *out : tmp;
    r.qn = a.template take<float>(T * P);
    r.kn = a.template take<float>(T * P);
    r.cv = a.template take<float>(T * P);
    r.ld = a.template take<float>(T * P);
    r.be = a.template take<float>(T * h);
    r.pq = a.template take<float>(T * P);
    r.pk = a.template take<float>(T * P);
    r.pv = a.template take<float>(T * P);
}

struct KdaWork {
    float *xr, *og, *fl, *bp, *fg, *cq, *ck, *ro, *gt;
    uint16_t *xt_h, *xt_d, *xt_p;
    int32_t* tables;   // anc [N][w-1], then the recurrence schedule
};

template <typename A>
void layout_kda_work(A& a, size_t T, size_t H, size_t P, size_t d, size_t h, size_t table_ints, KdaWork* out) {
    KdaWork tmp{};
    KdaWork& r = out ? *out : tmp;
    r.xr = a.template take<float>(T * H);
    r.og = a.template take<float>(T * P);
    r.fl = a.template take<float>(T * d);
    r.bp = a.template take<float>(T * h);
    r.fg = a.template take<float>(T * P);
    r.cq = a.template take<float>(T * P);
    r.ck = a.template take<float>(T * P);
    r.ro = a.template take<float>(T * P);
    r.gt = a.template take<float>(T * P);
    r.xt_h = a.template take<uint16_t>(2 * T * H, 1024);
    r.xt_d = a.template take<uint16_t>(2 * T * d, 1024);
    r.xt_p = a.template take<uint16_t>(2 * T * P, 1024);
    r.tables = a.template take<int32_t>(table_ints);
}

int validate_kda(k3xb_ctx* ctx, const k3xb_kda_layer* w, uint32_t H) {
    if (!w) return fail(ctx, K3XB_INVALID_EXTENT, "null KDA weights");
    if (!w->heads || !w->head_dim || w->conv_width < 2 || !H)
        return fail(ctx, K3XB_INVALID_EXTENT, "KDA dimensions (conv_width >= 2)");
    if (H % 8 || w->head_dim % 8)
        return fail(ctx, K3XB_INVALID_EXTENT, "KDA projections need hidden and head_dim multiples of 8");
    if (w->head_dim > 128) return fail(ctx, K3XB_INVALID_EXTENT, "KDA head_dim <= 128");
    if (!w->q_proj || !w->k_proj || !w->v_proj || !w->q_conv || !w->k_conv || !w->v_conv || !w->f_a_proj ||
        !w->f_b_proj || !w->a_log || !w->dt_bias || !w->b_proj || !w->g_proj || !w->o_norm || !w->o_proj)
        return fail(ctx, K3XB_INVALID_EXTENT, "missing KDA weights");
    if (!(w->eps > 0.0f)) return fail(ctx, K3XB_INVALID_EXTENT, "KDA eps must be positive");
    return K3XB_OK;
}

// anc[n][j-1]: node n's j-th ancestor (j = 1..w-1), or -(r+1) for conv
// history row r once the path leaves the tree (the row before a root is
// the newest, w-2).
void ancestor_table(const int32_t* parent, uint32_t N, uint32_t w, int32_t* anc) {
    for (uint32_t n = 0; n < N; ++n) {
        int32_t x = static_cast<int32_t>(n);
        uint32_t inside = 0;   // ancestors met inside the tree
        for (uint32_t j = 1; j < w; ++j) {
            if (x >= 0) x = parent[x];
            if (x >= 0) {
                ++inside;
                anc[n * (w - 1) + j - 1] = x;
            } else {
                const int32_t row = static_cast<int32_t>(w - 1) - static_cast<int32_t>(j - inside);
                anc[n * (w - 1) + j - 1] = -(row + 1);
            }
        }
    }
}

int kda_block_device(k3xb_ctx* ctx, const k3xb_kda_layer& w, uint32_t H, const float* x, bool x_is_bf16,
                     uint32_t N, uint32_t S, const uint16_t* conv, const float* rec, const KdaSchedule& sch,
                     const KdaTrace& tr, const KdaWork& wk, float* out) {
    const uint32_t T = N * S, h = w.heads, d = w.head_dim, P = h * d, cw = w.conv_width;
    int st;
    const float* xin = x;
    {
        PhaseScope ph(ctx, K3XB_PHASE_KDA_PROJECT);
        if (!x_is_bf16) {   // the block rounds its input first (official_kda.cpp:235-240)
            if ((st = launch_residual_round(ctx, x, static_cast<size_t>(T) * H, wk.xr))) return st;
            xin = wk.xr;
        }
        if ((st = launch_split_terms(ctx, xin, T, H, 1, wk.xt_h))) return st;
        // the six input projections of official_kda.cpp:228-245 in one launch
        const LinearJob jobs[6] = {{w.q_proj, P, tr.pq}, {w.k_proj, P, tr.pk},  {w.v_proj, P, tr.pv},
                                   {w.g_proj, P, wk.og}, {w.f_a_proj, d, wk.fl}, {w.b_proj, h, wk.bp}};
        if ((st = launch_linear_group(ctx, wk.xt_h, 1, T, H, jobs, 6, 1))) return st;
        if ((st = launch_split_terms(ctx, wk.fl, T, d, 1, wk.xt_d))) return st;
        if ((st = launch_linear_terms(ctx, wk.xt_d, 1, w.f_b_proj, T, P, d, 1, wk.fg))) return st;
    }
    {
        PhaseScope ph(ctx, K3XB_PHASE_KDA_CONV);
        const float* proj[3] = {tr.pq, tr.pk, tr.pv};
        const float* cwt[3] = {w.q_conv, w.k_conv, w.v_conv};
        float* const co[3] = {wk.cq, wk.ck, tr.cv};
        if ((st = launch_short_conv(ctx, proj, cwt, conv, wk.tables, S, N, P, cw, co))) return st;
        if ((st = launch_qk_gates(ctx, wk.cq, wk.ck, wk.fg, wk.bp, w.a_log, w.dt_bias, w.gate_lower_bound, T, h, d,
                                  tr.qn, tr.kn, tr.ld, tr.be)))
            return st;
    }
    {
        PhaseScope ph(ctx, K3XB_PHASE_KDA_RECURRENCE);
        const int32_t* sched = wk.tables + static_cast<size_t>(N) * (cw - 1);
        const size_t visit = sch.order.size();
        if ((st = launch_kda(ctx, rec, sched, sched + visit, sched + 2 * visit, static_cast<uint32_t>(visit), N, S, h,
                             d, tr.qn, tr.kn, tr.cv, tr.ld, tr.be, wk.ro, nullptr, sch.levels)))
            return st;
    }
    PhaseScope ph(ctx, K3XB_PHASE_KDA_OUTPUT);
    if ((st = launch_gated_norm(ctx, wk.ro, wk.og, w.o_norm, w.eps, T, h, d, wk.gt))) return st;
    if ((st = launch_split_terms(ctx, wk.gt, T, P, 1, wk.xt_p))) return st;
    ++ctx->stats.kda_calls;
    return launch_linear_terms(ctx, wk.xt_p, 1, w.o_proj, T, H, P, 1, out);
}

int validate_full_layer(k3xb_ctx* ctx, const k3xb_layer* L) {
    if (!L) return fail(ctx, K3XB_INVALID_EXTENT, "null layer");
    int st = validate_kda(ctx, &L->kda, L->hidden);
    if (st) return st;
    if ((st = validate_layer(ctx, &L->moe))) return st;
    if (L->moe.hidden != L->hidden) return fail(ctx, K3XB_INVALID_EXTENT, "moe.hidden must equal the layer width");
    if (!L->self_residual_norm || !L->self_residual_proj || !L->input_norm || !L->moe_residual_norm ||
        !L->moe_residual_proj || !L->post_norm || !(L->rms_eps > 0.0f))
        return fail(ctx, K3XB_INVALID_EXTENT, "missing layer norms");
    if (attnres_smem_bytes(L->hidden) > 200 * 1024) return fail(ctx, K3XB_INVALID_EXTENT, "hidden too large");
    return K3XB_OK;
}

// Scratch of one layer forward (its region starts at the scratch base).
template <typename A>
void layout_layer(A& a, const k3xb_layer& L, uint32_t N, uint32_t S, bool own_trace, KdaTrace* tr, KdaWork* wk,
                  float** bufs, MoeScratch* ms, uint32_t ep_E = 0, void** ep_region = nullptr) {
    const size_t T = static_cast<size_t>(N) * S, H = L.hidden;
    const size_t P = static_cast<size_t>(L.kda.heads) * L.kda.head_dim;
    if (own_trace) layout_trace(a, T, P, L.kda.heads, tr);
    layout_kda_work(a, T, H, P, L.kda.head_dim, L.kda.heads, 0, wk);
    for (int i = 0; i < 4; ++i) {   // xin, kda_out, prefix, moe_in
        float* b = a.template take<float>(T * H);
        if (bufs) bufs[i] = b;
    }
    layout_moe(a, L.moe, static_cast<uint32_t>(T), false, ms, ep_E);
    if (ep_E) {   // the local plan over the received rows (ep.cu)
        const uint32_t G = static_cast<uint32_t>(ep_E / L.moe.experts);
        void* r = a.template take<uint8_t>(ep_scratch_bytes(G, static_cast<uint32_t>(T), L.moe.top_k,
                                                            expert_view(L.moe).hidden, L.moe.experts), 1024);
        if (ep_region) *ep_region = r;
    }
}

// The engine's region comes last; expert parallel, it holds the rows that
// every rank sends (world x T).
size_t layer_work_bytes(const k3xb_layer& L, uint32_t N, uint32_t S, bool own_trace, uint32_t ep_E = 0) {
    Sizer sz;
    layout_layer(sz, L, N, S, own_trace, nullptr, nullptr, nullptr, nullptr, ep_E);
    const uint32_t rows = ep_E ? N * S * (ep_E / L.moe.experts) : N * S;
    return sz.used + mxf4_scratch_bytes(expert_view(L.moe), rows) + 1024;
}

// official_layer_cpu with the plain MoE; d_tables = device anc table +
// recurrence schedule for `sch`.
int layer_forward_impl(k3xb_ctx* ctx, const k3xb_layer& L, const float* hidden_in, const float* block, uint32_t N,
                       uint32_t S, const uint16_t* conv, const float* rec, float* hidden_out, uint32_t* ids_out,
                       void* trace, const KdaSchedule& sch, const int32_t* d_tables, uint32_t ep_E = 0) {
    const uint32_t T = N * S, H = L.hidden;
    const size_t P = static_cast<size_t>(L.kda.heads) * L.kda.head_dim;
    void* base;
    int st = ensure_scratch(ctx, layer_work_bytes(L, N, S, trace == nullptr, ep_E), &base);
    if (st) return st;
    Carver c(base);
    KdaTrace tr{};
    KdaWork wk{};
    float* bufs[4];
    MoeScratch ms{};
    void* ep_region = nullptr;
    layout_layer(c, L, N, S, trace == nullptr, &tr, &wk, bufs, &ms, ep_E, &ep_region);
    if (trace) {
        Carver t(trace);
        layout_trace(t, T, P, L.kda.heads, &tr);
    }
    set_mxf4_scratch(ctx, reinterpret_cast<char*>(base) + c.used);
    wk.tables = const_cast<int32_t*>(d_tables);
    float *xin = bufs[0], *kda_out = bufs[1], *prefix = bufs[2], *moe_in = bufs[3];
    {   // official_layer.cpp:159-172: attention residual + input norm
        PhaseScope ph(ctx, K3XB_PHASE_ATTN_RESIDUAL);
        if ((st = launch_attnres_norm(ctx, hidden_in, nullptr, block, L.self_residual_norm, L.self_residual_proj,
                                      L.input_norm, T, H, L.rms_eps, nullptr, xin)))
            return st;
    }
    if ((st = kda_block_device(ctx, L.kda, H, xin, true, N, S, conv, rec, sch, tr, wk, kda_out))) return st;
    {   // :190-205: prefix, MoE input preparation
        PhaseScope ph(ctx, K3XB_PHASE_ATTN_RESIDUAL);
        if ((st = launch_attnres_norm(ctx, hidden_in, kda_out, block, L.moe_residual_norm, L.moe_residual_proj,
                                      L.post_norm, T, H, L.rms_eps, prefix, moe_in)))
            return st;
    }
    // plain MoE: combined = round_bf16(routed + shared), then the residual (official_moe.cpp:336-341)
    if ((st = moe_forward_device(ctx, L.moe, moe_in, T, hidden_out, ids_out, nullptr, ms, ep_E, ep_region)))
        return st;
    return launch_residual(ctx, prefix, hidden_out, static_cast<size_t>(T) * H, hidden_out);
}

// anc table + schedule packed for one upload
std::vector<int32_t> kda_tables(const int32_t* parent, uint32_t N, uint32_t cw, const KdaSchedule& sch) {
    std::vector<int32_t> t(static_cast<size_t>(N) * (cw - 1));
    ancestor_table(parent, N, cw, t.data());
    t.insert(t.end(), sch.order.begin(), sch.order.end());
    t.insert(t.end(), sch.depth.begin(), sch.depth.end());
    t.insert(t.end(), sch.from_stack.begin(), sch.from_stack.end());
    return t;
}

}  // namespace

extern "C" {

size_t k3xb_kda_trace_bytes(const k3xb_kda_layer* w, uint32_t nodes, uint32_t S) {
    if (!w) return 0;
    Sizer sz;
    layout_trace(sz, static_cast<size_t>(nodes) * S, static_cast<size_t>(w->heads) * w->head_dim, w->heads, nullptr);
    return sz.used;
}

int k3xb_kda_block(k3xb_ctx* ctx, const k3xb_kda_layer* w, uint32_t H, const float* x, const int32_t* parent,
                   uint32_t N, uint32_t S, const uint16_t* conv, const float* rec, float* out, void* trace) {
    K3XB_ENTER(ctx);
    int st = validate_kda(ctx, w, H);
    if (st) return st;
    if (!x || !parent || !N || !S || !conv || !rec || !out) return fail(ctx, K3XB_INVALID_EXTENT, "kda_block arguments");
    KdaSchedule sch;
    if ((st = schedule_tree(ctx, parent, N, sch))) return st;
    const std::vector<int32_t> tables = kda_tables(parent, N, w->conv_width, sch);
    const size_t T = static_cast<size_t>(N) * S, P = static_cast<size_t>(w->heads) * w->head_dim;
    Sizer sz;
    if (!trace) layout_trace(sz, T, P, w->heads, nullptr);
    layout_kda_work(sz, T, H, P, w->head_dim, w->heads, tables.size(), nullptr);
    void* base;
    if ((st = ensure_scratch(ctx, sz.used, &base))) return st;
    Carver c(base);
    KdaTrace tr{};
    if (trace) {
        Carver t(trace);
        layout_trace(t, T, P, w->heads, &tr);
    } else {
        layout_trace(c, T, P, w->heads, &tr);
    }
    KdaWork wk{};
    layout_kda_work(c, T, H, P, w->head_dim, w->heads, tables.size(), &wk);
    K3XB_CUDA(ctx, cudaMemcpyAsync(wk.tables, tables.data(), tables.size() * sizeof(int32_t), cudaMemcpyHostToDevice,
                                   ctx->stream));
    return kda_block_device(ctx, *w, H, x, false, N, S, conv, rec, sch, tr, wk, out);
}

int k3xb_kda_block_commit(k3xb_ctx* ctx, const k3xb_kda_layer* w, const void* trace, const int32_t* parent,
                          uint32_t N, uint32_t S, const int32_t* commit_node, const uint16_t* conv, const float* rec,
                          uint16_t* conv_out, float* rec_out) {
    K3XB_ENTER(ctx);
    if (!w || !trace || !parent || !N || !S || !commit_node || !conv || !rec || !conv_out || !rec_out)
        return fail(ctx, K3XB_INVALID_EXTENT, "kda_block_commit arguments");
    if (rec_out == rec) return fail(ctx, K3XB_INVALID_EXTENT, "recurrent_out must not alias recurrent");
    const uint32_t cw = w->conv_width, h = w->heads, d = w->head_dim;
    if (cw < 2) return fail(ctx, K3XB_INVALID_EXTENT, "conv_width >= 2");
    for (uint32_t i = 0; i < N; ++i)
        if (parent[i] < -1 || parent[i] >= static_cast<int32_t>(i))
            return fail(ctx, K3XB_INVALID_EXTENT, "draft tree: parent[n] must be -1 or < n");
    // anc_commit[s][j]: the commit node (j = 0) and its ancestors, else history rows
    std::vector<int32_t> anc(static_cast<size_t>(S) * (cw - 1));
    for (uint32_t s = 0; s < S; ++s) {
        const int32_t node = commit_node[s];
        if (node < -1 || node >= static_cast<int32_t>(N)) return fail(ctx, K3XB_INVALID_EXTENT, "commit node out of range");
        int32_t x = node;
        uint32_t inside = 0;
        for (uint32_t j = 0; j + 1 < cw; ++j) {
            if (j > 0 && x >= 0) x = parent[x];
            if (x >= 0) {
                ++inside;
                anc[static_cast<size_t>(s) * (cw - 1) + j] = x;
            } else {
                const int32_t row = static_cast<int32_t>(cw) - 2 - static_cast<int32_t>(j - inside);
                anc[static_cast<size_t>(s) * (cw - 1) + j] = -(row + 1);
            }
        }
    }
    const size_t T = static_cast<size_t>(N) * S, P = static_cast<size_t>(h) * d;
    KdaTrace tr{};
    Carver t(const_cast<void*>(trace));
    layout_trace(t, T, P, h, &tr);
    void* base;
    int st = ensure_scratch(ctx, anc.size() * sizeof(int32_t), &base);
    if (st) return st;
    K3XB_CUDA(ctx, cudaMemcpyAsync(base, anc.data(), anc.size() * sizeof(int32_t), cudaMemcpyHostToDevice,
                                   ctx->stream));
    const float* proj[3] = {tr.pq, tr.pk, tr.pv};
    {
        PhaseScope ph(ctx, K3XB_PHASE_COMMIT);
        if ((st = launch_conv_commit(ctx, proj, conv, static_cast<const int32_t*>(base), S, N,
                                     static_cast<uint32_t>(P), cw, conv_out)))
            return st;
    }
    return k3xb_kda_commit(ctx, rec, parent, N, S, h, d, tr.qn, tr.kn, tr.cv, tr.ld, tr.be, commit_node, rec_out);
}

int k3xb_kda_block_host(k3xb_ctx* ctx, const k3xb_kda_layer* w, uint32_t H, const float* x_host, uint32_t T,
                        uint16_t* conv_host, float* rec_host, float* out_host) {
    K3XB_ENTER(ctx);
    int st = validate_kda(ctx, w, H);
    if (st) return st;
    if (!x_host || !T || !conv_host || !rec_host || !out_host)
        return fail(ctx, K3XB_INVALID_EXTENT, "kda_block_host arguments");
    const size_t P = static_cast<size_t>(w->heads) * w->head_dim;
    const size_t conv_n = 3 * static_cast<size_t>(w->conv_width - 1) * P;
    const size_t rec_n = static_cast<size_t>(w->heads) * w->head_dim * w->head_dim;
    const size_t xbytes = sizeof(float) * T * H;
    Sizer sz;
    sz.take<float>(static_cast<size_t>(T) * H);
    sz.take<float>(static_cast<size_t>(T) * H);
    sz.take<uint16_t>(2 * conv_n);
    sz.take<float>(2 * rec_n);
    sz.take<uint8_t>(k3xb_kda_trace_bytes(w, T, 1));
    void* base;
    if ((st = ensure_io(ctx, sz.used, &base))) return st;
    Carver c(base);
    float* x = c.take<float>(static_cast<size_t>(T) * H);
    float* out = c.take<float>(static_cast<size_t>(T) * H);
    uint16_t* conv = c.take<uint16_t>(2 * conv_n);
    float* rec = c.take<float>(2 * rec_n);
    void* trace = c.take<uint8_t>(k3xb_kda_trace_bytes(w, T, 1));
    K3XB_CUDA(ctx, cudaMemcpyAsync(x, x_host, xbytes, cudaMemcpyHostToDevice, ctx->stream));
    K3XB_CUDA(ctx, cudaMemcpyAsync(conv, conv_host, conv_n * 2, cudaMemcpyHostToDevice, ctx->stream));
    K3XB_CUDA(ctx, cudaMemcpyAsync(rec, rec_host, rec_n * 4, cudaMemcpyHostToDevice, ctx->stream));
    ctx->stats.h2d_bytes += xbytes + conv_n * 2 + rec_n * 4;
    // the positions are a chain; its last node is the state the call publishes
    std::vector<int32_t> parent(T);
    for (uint32_t n = 0; n < T; ++n) parent[n] = static_cast<int32_t>(n) - 1;
    const int32_t last = static_cast<int32_t>(T) - 1;
    if ((st = k3xb_kda_block(ctx, w, H, x, parent.data(), T, 1, conv, rec, out, trace))) return st;
    if ((st = k3xb_kda_block_commit(ctx, w, trace, parent.data(), T, 1, &last, conv, rec, conv + conv_n,
                                    rec + rec_n)))
        return st;
    K3XB_CUDA(ctx, cudaMemcpyAsync(out_host, out, xbytes, cudaMemcpyDeviceToHost, ctx->stream));
    K3XB_CUDA(ctx, cudaMemcpyAsync(conv_host, conv + conv_n, conv_n * 2, cudaMemcpyDeviceToHost, ctx->stream));
    K3XB_CUDA(ctx, cudaMemcpyAsync(rec_host, rec + rec_n, rec_n * 4, cudaMemcpyDeviceToHost, ctx->stream));
    ctx->stats.d2h_bytes += xbytes + conv_n * 2 + rec_n * 4;
    return k3xb_sync(ctx);
}

int k3xb_kda_block_held(k3xb_ctx* ctx, const k3xb_kda_layer* w, uint32_t H, const float* x_host, uint32_t T,
                        uint32_t slot, int32_t mode, uint16_t* conv_host, float* rec_host, float* out_host) {
    K3XB_ENTER(ctx);
    int st = validate_kda(ctx, w, H);
    if (st) return st;
    if (!x_host || !T || !out_host || slot >= K3XB_KDA_HELD_SLOTS)
        return fail(ctx, K3XB_INVALID_EXTENT, "kda_block_held arguments (slot < K3XB_KDA_HELD_SLOTS)");
    if (mode != K3XB_KDA_SEED && mode != K3XB_KDA_CONTINUE && mode != K3XB_KDA_PUBLISH)
        return fail(ctx, K3XB_INVALID_STATE, "kda_block_held: unknown mode");
    if ((mode != K3XB_KDA_CONTINUE) && (!conv_host || !rec_host))
        return fail(ctx, K3XB_INVALID_EXTENT, "kda_block_held: seed and publish take the host state arrays");
    const size_t P = static_cast<size_t>(w->heads) * w->head_dim;
    const size_t conv_n = 3 * static_cast<size_t>(w->conv_width - 1) * P;
    const size_t rec_n = static_cast<size_t>(w->heads) * w->head_dim * w->head_dim;
    if (!ctx->kda_held) {
        ctx->kda_held = new (std::nothrow) KdaHeld[K3XB_KDA_HELD_SLOTS];
        if (!ctx->kda_held) return fail(ctx, K3XB_BACKEND_UNAVAILABLE, "kda_block_held: out of host memory");
    }
    KdaHeld& h = static_cast<KdaHeld*>(ctx->kda_held)[slot];
    Sizer one;   // one state: conv words, then the recurrent state
    one.take<uint16_t>(conv_n);
    one.take<float>(rec_n);
    const size_t state_bytes = (one.used + 255) / 256 * 256;
    if (mode == K3XB_KDA_SEED) {
        if (h.state_bytes != state_bytes) {   // (re)shape the slot: two states, read one, write the other
            if ((st = stream_wait(ctx))) return st;
            if (h.buf) K3XB_CUDA(ctx, cudaFree(h.buf));
            h = KdaHeld{};
            K3XB_CUDA(ctx, cudaMalloc(&h.buf, 2 * state_bytes));
            h.state_bytes = state_bytes;
            h.conv_n = conv_n;
            h.rec_n = rec_n;
        }
        h.valid = false;
    } else if (!h.valid || h.conv_n != conv_n || h.rec_n != rec_n) {
        return fail(ctx, K3XB_INVALID_STATE, "kda_block_held: no state of this shape held in the slot");
    }
    const auto state_at = [&](int i, uint16_t** conv, float** rec) {
        Carver c(static_cast<char*>(h.buf) + static_cast<size_t>(i) * state_bytes);
        *conv = c.take<uint16_t>(conv_n);
        *rec = c.take<float>(rec_n);
    };
    uint16_t *conv_in, *conv_out;
    float *rec_in, *rec_out;
    state_at(h.cur, &conv_in, &rec_in);
    state_at(h.cur ^ 1, &conv_out, &rec_out);
    const size_t xbytes = sizeof(float) * T * H;
    Sizer sz;
    sz.take<float>(static_cast<size_t>(T) * H);
    sz.take<float>(static_cast<size_t>(T) * H);
    sz.take<uint8_t>(k3xb_kda_trace_bytes(w, T, 1));
    void* base;
    if ((st = ensure_io(ctx, sz.used, &base))) return st;
    Carver c(base);
    float* x = c.take<float>(static_cast<size_t>(T) * H);
    float* out = c.take<float>(static_cast<size_t>(T) * H);
    void* trace = c.take<uint8_t>(k3xb_kda_trace_bytes(w, T, 1));
    K3XB_CUDA(ctx, cudaMemcpyAsync(x, x_host, xbytes, cudaMemcpyHostToDevice, ctx->stream));
    ctx->stats.h2d_bytes += xbytes;
    if (mode == K3XB_KDA_SEED) {
        K3XB_CUDA(ctx, cudaMemcpyAsync(conv_in, conv_host, conv_n * 2, cudaMemcpyHostToDevice, ctx->stream));
        K3XB_CUDA(ctx, cudaMemcpyAsync(rec_in, rec_host, rec_n * 4, cudaMemcpyHostToDevice, ctx->stream));
        ctx->stats.h2d_bytes += conv_n * 2 + rec_n * 4;
    }
    // the positions are a chain from the held state; its last node is the new state
    std::vector<int32_t> parent(T);
    for (uint32_t n = 0; n < T; ++n) parent[n] = static_cast<int32_t>(n) - 1;
    const int32_t last = static_cast<int32_t>(T) - 1;
    if ((st = k3xb_kda_block(ctx, w, H, x, parent.data(), T, 1, conv_in, rec_in, out, trace))) return st;
    if ((st = k3xb_kda_block_commit(ctx, w, trace, parent.data(), T, 1, &last, conv_in, rec_in, conv_out, rec_out)))
        return st;
    K3XB_CUDA(ctx, cudaMemcpyAsync(out_host, out, xbytes, cudaMemcpyDeviceToHost, ctx->stream));
    ctx->stats.d2h_bytes += xbytes;
    if (mode == K3XB_KDA_PUBLISH) {
        K3XB_CUDA(ctx, cudaMemcpyAsync(conv_host, conv_out, conv_n * 2, cudaMemcpyDeviceToHost, ctx->stream));
        K3XB_CUDA(ctx, cudaMemcpyAsync(rec_host, rec_out, rec_n * 4, cudaMemcpyDeviceToHost, ctx->stream));
        ctx->stats.d2h_bytes += conv_n * 2 + rec_n * 4;
    }
    if ((st = k3xb_sync(ctx))) return st;
    h.cur ^= 1;   // the new state is the one just written
    h.valid = true;
    return K3XB_OK;
}

int k3xb_attention_residual_norm(k3xb_ctx* ctx, const float* a, const float* delta, const float* block,
                                 const uint16_t* rnorm, const uint16_t* rproj, const uint16_t* post, uint32_t T,
                                 uint32_t H, float eps, float* prefix_out, float* out) {
    K3XB_ENTER(ctx);
    if (!a || !block || !rnorm || !rproj || !post || !T || !H || !out || (delta && !prefix_out))
        return fail(ctx, K3XB_INVALID_EXTENT, "attention residual arguments");
    if (!(eps > 0.0f)) return fail(ctx, K3XB_INVALID_EXTENT, "eps must be positive");
    return launch_attnres_norm(ctx, a, delta, block, rnorm, rproj, post, T, H, eps, prefix_out, out);
}

int k3xb_block_attention_residual(k3xb_ctx* ctx, const float* prefix, const float* sources, uint32_t S, uint32_t T,
                                  uint32_t H, const float* norm, const float* projection, float eps, float* out) {
    K3XB_ENTER(ctx);
    if (!prefix || (S && !sources) || !norm || !projection || !out || !T || !H)
        return fail(ctx, K3XB_INVALID_EXTENT, "block attention residual arguments");
    if (S >= kBlockAttnResMaxDepth)
        return fail(ctx, K3XB_INVALID_EXTENT, "block attention residual: at most 63 sources");
    if (T > 0x7fffffffu) return fail(ctx, K3XB_INVALID_EXTENT, "block attention residual: too many rows");
    if (!std::isfinite(eps) || eps < 0.0f) return fail(ctx, K3XB_INVALID_EXTENT, "eps must be finite and >= 0");
    PhaseScope ph(ctx, K3XB_PHASE_ATTN_RESIDUAL);
    return launch_block_attnres(ctx, prefix, sources, S, T, H, norm, projection, eps, out);
}

int k3xb_prepare_moe_route_host(k3xb_ctx* ctx, const float* a_host, const float* delta_host, const float* block_host,
                                uint32_t H, const uint16_t* rnorm, const uint16_t* rproj, const uint16_t* post, float eps,
                                const uint16_t* router, uint32_t E, float* prefix_host, float* hidden_host,
                                float* logits_host) {
    K3XB_ENTER(ctx);
    if (!a_host || !block_host || !H || !rnorm || !rproj || !post || !hidden_host || (delta_host && !prefix_host) ||
        (router && (!E || !logits_host)))
        return fail(ctx, K3XB_INVALID_EXTENT, "prepare moe route arguments");
    if (!(eps > 0.0f)) return fail(ctx, K3XB_INVALID_EXTENT, "eps must be positive");
    const uint32_t n_logits = router ? E : 0;
    Sizer sz;
    sz.take<float>(3 * size_t(H));   // a, delta, block (one upload each)
    sz.take<float>(H);               // the prefix (with delta)
    sz.take<float>(H);               // the prepared input
    sz.take<float>(n_logits ? n_logits : 1);
    void* base;
    int st;
    if ((st = ensure_scratch(ctx, sz.used, &base))) return st;
    Carver c(base);
    float* in = c.take<float>(3 * size_t(H));
    float* prefix = c.take<float>(H);
    float* hidden = c.take<float>(H);
    float* logits = c.take<float>(n_logits ? n_logits : 1);
    const size_t hbytes = sizeof(float) * H;
    K3XB_CUDA(ctx, cudaMemcpyAsync(in, a_host, hbytes, cudaMemcpyHostToDevice, ctx->stream));
    if (delta_host) K3XB_CUDA(ctx, cudaMemcpyAsync(in + H, delta_host, hbytes, cudaMemcpyHostToDevice, ctx->stream));
    K3XB_CUDA(ctx, cudaMemcpyAsync(in + 2 * size_t(H), block_host, hbytes, cudaMemcpyHostToDevice, ctx->stream));
    ctx->stats.h2d_bytes += (delta_host ? 3 : 2) * hbytes;
    {   // prepare_official_moe_input (official_moe.cpp:156-209); with delta the
        // first source is the prefix round_bf16(round_bf16(a) + delta) (official_layer.cpp:190-193)
        PhaseScope ph(ctx, K3XB_PHASE_ATTN_RESIDUAL);
        if ((st = launch_attnres_norm(ctx, in, delta_host ? in + H : nullptr, in + 2 * size_t(H), rnorm, rproj, post, 1,
                                      H, eps, delta_host ? prefix : nullptr, hidden)))
            return st;
    }
    if (router) {   // route_official_moe_logits' input (official_moe.cpp:211-245): FP64 sums in h order
        PhaseScope ph(ctx, K3XB_PHASE_ROUTE);
        if ((st = launch_router_logits(ctx, hidden, 1, H, router, E, logits))) return st;
    }
    K3XB_CUDA(ctx, cudaMemcpyAsync(hidden_host, hidden, hbytes, cudaMemcpyDeviceToHost, ctx->stream));
    if (delta_host) K3XB_CUDA(ctx, cudaMemcpyAsync(prefix_host, prefix, hbytes, cudaMemcpyDeviceToHost, ctx->stream));
    if (router)
        K3XB_CUDA(ctx, cudaMemcpyAsync(logits_host, logits, sizeof(float) * E, cudaMemcpyDeviceToHost, ctx->stream));
    ctx->stats.d2h_bytes += (delta_host ? 2 : 1) * hbytes + sizeof(float) * n_logits;
    if (router) ++ctx->stats.route_calls;
    return k3xb_sync(ctx);
}

int k3xb_layer_forward(k3xb_ctx* ctx, const k3xb_layer* L, const float* hidden_in, const float* block,
                       const int32_t* parent, uint32_t N, uint32_t S, const uint16_t* conv, const float* rec,
                       float* hidden_out, uint32_t* ids_out, void* trace) {
    K3XB_ENTER(ctx);
    int st = validate_full_layer(ctx, L);
    if (st) return st;
    if (!hidden_in || !block || !parent || !N || !S || !conv || !rec || !hidden_out)
        return fail(ctx, K3XB_INVALID_EXTENT, "layer arguments");
    KdaSchedule sch;
    if ((st = schedule_tree(ctx, parent, N, sch))) return st;
    const std::vector<int32_t> tables = kda_tables(parent, N, L->kda.conv_width, sch);
    // the layer's own region first, the topology tables after it
    const size_t own = layer_work_bytes(*L, N, S, trace == nullptr);
    void* base;
    if ((st = ensure_scratch(ctx, own + tables.size() * sizeof(int32_t) + 256, &base))) return st;
    int32_t* d_tables = reinterpret_cast<int32_t*>((reinterpret_cast<uintptr_t>(base) + own + 255) & ~uintptr_t(255));
    K3XB_CUDA(ctx, cudaMemcpyAsync(d_tables, tables.data(), tables.size() * sizeof(int32_t), cudaMemcpyHostToDevice,
                                   ctx->stream));
    return layer_forward_impl(ctx, *L, hidden_in, block, N, S, conv, rec, hidden_out, ids_out, trace, sch, d_tables);
}

// The verify step; with ep_E != 0 every layer's MoE is expert parallel
// (its descriptor holds this rank's slice of ep_E experts) and the step
// covers this rank's own sequences.
static int verify_step_impl(k3xb_ctx* ctx, const k3xb_verify_model* m, const k3xb_verify_io* io, uint32_t ep_E) {
    if (!m || !io || !m->layers || !m->layer || !m->vocab || !m->lm_head)
        return fail(ctx, K3XB_INVALID_EXTENT, "verify model");
    int st;
    const k3xb_layer& L0 = m->layer[0];
    for (uint32_t l = 0; l < m->layers; ++l) {
        if ((st = validate_full_layer(ctx, &m->layer[l]))) return st;
        const k3xb_layer& L = m->layer[l];
        if (L.hidden != L0.hidden || L.kda.heads != L0.kda.heads || L.kda.head_dim != L0.kda.head_dim ||
            L.kda.conv_width != L0.kda.conv_width)
            return fail(ctx, K3XB_INVALID_EXTENT, "verify layers must share hidden, heads, head_dim, conv_width");
    }
    const uint32_t S = io->sequences, p = io->drafts, N = p + 1, T = S * N, H = L0.hidden, V = m->vocab;
    if (!S || !io->conv || !io->recurrent || !io->accepted || !io->committed || !io->committed_count ||
        (p && !io->draft_tokens))
        return fail(ctx, K3XB_INVALID_EXTENT, "verify io");
    if (m->embedding ? !io->tokens : !io->hidden_in) return fail(ctx, K3XB_INVALID_EXTENT, "verify inputs");
    if (io->mode != K3XB_ACCEPT_GREEDY && io->mode != K3XB_ACCEPT_REJECTION)
        return fail(ctx, K3XB_INVALID_EXTENT, "acceptance mode");
    if (io->mode == K3XB_ACCEPT_REJECTION && ((p && !io->draft_logits) || !(io->temperature > 0.0f)))
        return fail(ctx, K3XB_INVALID_EXTENT, "rejection sampling needs draft logits and temperature > 0");
    if (H % 8) return fail(ctx, K3XB_INVALID_EXTENT, "LM head needs hidden % 8 == 0");
    std::vector<int32_t> parent(N);
    for (uint32_t i = 0; i < N; ++i) parent[i] = static_cast<int32_t>(i) - 1;
    KdaSchedule sch;
    if ((st = schedule_tree(ctx, parent.data(), N, sch))) return st;
    const uint32_t cw = L0.kda.conv_width, h = L0.kda.heads, d = L0.kda.head_dim, P = h * d;
    const std::vector<int32_t> tables = kda_tables(parent.data(), N, cw, sch);
    if (ep_E) {   // the exchange window for the widest layer, before anything is queued
        uint32_t Kmax = 0, Dmax = 0;
        for (uint32_t l = 0; l < m->layers; ++l) {
            Kmax = std::max(Kmax, m->layer[l].moe.top_k);
            Dmax = std::max(Dmax, expert_view(m->layer[l].moe).hidden);
        }
        if ((st = ep_reserve(ctx, T, Kmax, Dmax))) return st;
    }
    size_t own = 0;
    for (uint32_t l = 0; l < m->layers; ++l)
        own = std::max(own, layer_work_bytes(m->layer[l], N, S, false, ep_E));
    const size_t TH = static_cast<size_t>(T) * H, trace_bytes = k3xb_kda_trace_bytes(&L0.kda, N, S);
    Sizer sz;
    sz.take<uint8_t>(own);
    sz.take<int32_t>(tables.size());
    for (uint32_t l = 0; l < m->layers; ++l) sz.take<uint8_t>(trace_bytes, 1024);
    for (int i = 0; i < 3; ++i) sz.take<float>(TH);   // x0, ping, pong
    sz.take<uint16_t>(2 * TH, 1024);                   // LM-head operand terms
    if (!io->logits) sz.take<float>(static_cast<size_t>(T) * V);
    sz.take<uint32_t>(T);                              // greedy targets
    sz.take<double>(2 * static_cast<size_t>(T));       // rejection sums
    void* base;
    if ((st = ensure_scratch(ctx, sz.used, &base))) return st;
    Carver c(base);
    c.take<uint8_t>(own);
    int32_t* d_tables = c.take<int32_t>(tables.size());
    std::vector<void*> traces(m->layers);
    for (uint32_t l = 0; l < m->layers; ++l) traces[l] = c.take<uint8_t>(trace_bytes, 1024);
    float* x0 = c.take<float>(TH);
    float* buf[2] = {c.take<float>(TH), c.take<float>(TH)};
    uint16_t* xt = c.take<uint16_t>(2 * TH, 1024);
    float* logits = io->logits ? io->logits : c.take<float>(static_cast<size_t>(T) * V);
    uint32_t* targets = c.take<uint32_t>(T);
    double* pd = c.take<double>(T);
    double* qd = c.take<double>(T);
    K3XB_CUDA(ctx, cudaMemcpyAsync(d_tables, tables.data(), tables.size() * sizeof(int32_t), cudaMemcpyHostToDevice,
                                   ctx->stream));
    const float* x = io->hidden_in;
    if (m->embedding) {
        PhaseScope ph(ctx, K3XB_PHASE_EMBED);
        if ((st = launch_embed(ctx, io->tokens, m->embedding, V, T, H, x0))) return st;
        x = x0;
    }
    const float* block = io->block_source ? io->block_source : x;
    const size_t conv_stride = static_cast<size_t>(S) * 3 * (cw - 1) * P;
    const size_t rec_stride = static_cast<size_t>(S) * h * d * d;
    for (uint32_t l = 0; l < m->layers; ++l) {
        float* out = buf[l & 1u];
        if ((st = layer_forward_impl(ctx, m->layer[l], x, block, N, S, io->conv + l * conv_stride,
                                     io->recurrent + l * rec_stride, out, nullptr, traces[l], sch, d_tables, ep_E)))
            return st;
        x = out;
    }
    {
        PhaseScope ph(ctx, K3XB_PHASE_LM_HEAD);
        if (m->final_norm) {
            float* y = buf[m->layers & 1u];
            if ((st = launch_rms_norm(ctx, x, m->final_norm, T, H, m->final_eps, y))) return st;
            x = y;
        }
        // LM head: bf16 matvec semantics (official_moe.cpp:39-59), logits rounded to bf16
        if ((st = launch_split_terms(ctx, x, T, H, 1, xt))) return st;
        if ((st = launch_linear_terms(ctx, xt, 1, m->lm_head, T, V, H, 1, logits))) return st;
    }
    {
        PhaseScope ph(ctx, K3XB_PHASE_ACCEPT);
        if (io->mode == K3XB_ACCEPT_GREEDY) {
            st = launch_accept_greedy(ctx, logits, io->draft_tokens, S, p, V, targets, io->accepted,
                                      io->committed, io->committed_count);
        } else {
            st = launch_accept_rejection(ctx, logits, io->draft_logits, io->draft_tokens, S, p, V, io->temperature,
                                         io->seed, io->sequence_base, pd, qd, io->accepted, io->committed,
                                         io->committed_count);
        }
    }
    if (st) return st;
    ++ctx->stats.accept_calls;
    // commit every layer at node accepted[s] (model.cpp:1660-1664), on the device
    PhaseScope commit_phase(ctx, K3XB_PHASE_COMMIT);
    const int32_t* sched = d_tables + static_cast<size_t>(N) * (cw - 1);
    for (uint32_t l = 0; l < m->layers; ++l) {
        KdaTrace tr{};
        Carver t(traces[l]);
        layout_trace(t, T, P, h, &tr);
        const float* proj[3] = {tr.pq, tr.pk, tr.pv};
        uint16_t* conv = io->conv + l * conv_stride;
        float* rec = io->recurrent + l * rec_stride;
        if ((st = launch_conv_commit_linear(ctx, proj, conv, io->accepted, S, N, P, cw, conv))) return st;
        // in place: each warp reads its state rows before it writes them
        if ((st = launch_kda(ctx, rec, sched, sched + N, sched + 2 * N, N, N, S, h, d, tr.qn, tr.kn, tr.cv, tr.ld,
                             tr.be, nullptr, rec, sch.levels, reinterpret_cast<const int32_t*>(io->accepted))))
            return st;
    }
    return K3XB_OK;
}

int k3xb_verify_step(k3xb_ctx* ctx, const k3xb_verify_model* m, const k3xb_verify_io* io) {
    K3XB_ENTER(ctx);
    return verify_step_impl(ctx, m, io, 0);
}

int k3xb_ep_verify_step(k3xb_ctx* ctx, const k3xb_verify_model* m, const k3xb_verify_io* io,
                        uint32_t experts_total) {
    K3XB_ENTER(ctx);
    const int G = ep_world(ctx);
    if (G < 1) return fail(ctx, K3XB_INVALID_STATE, "expert parallelism not initialised (k3xb_ep_init)");
    if (!m || !m->layer || !m->layers) return fail(ctx, K3XB_INVALID_EXTENT, "verify model");
    if (!experts_total || experts_total % static_cast<uint32_t>(G) || experts_total > 1024)
        return fail(ctx, K3XB_INVALID_EXTENT, "experts_total must split evenly over the world (<= 1024)");
    for (uint32_t l = 0; l < m->layers; ++l) {
        const k3xb_moe_layer& M = m->layer[l].moe;
        if (M.engine != K3XB_ENGINE_MXF4) return fail(ctx, K3XB_INVALID_STATE, "expert parallelism runs the MXF4 engine");
        if (M.experts != experts_total / static_cast<uint32_t>(G))
            return fail(ctx, K3XB_INVALID_EXTENT, "every layer's experts must be experts_total / world (this rank's slice)");
        if (M.top_k > 32 || M.top_k > experts_total)
            return fail(ctx, K3XB_INVALID_EXTENT, "expert parallel route: top_k <= 32");
    }
    return verify_step_impl(ctx, m, io, experts_total);
}

int k3xb_ep_balance(const float* load, uint32_t E, uint32_t world, uint32_t* owner) {
    if (!load || !owner || !E || !world || E % world || E / world > 0xffffu) return K3XB_INVALID_EXTENT;
    std::vector<uint32_t> order(E);
    for (uint32_t e = 0; e < E; ++e) {
        if (!std::isfinite(load[e])) return K3XB_INVALID_EXTENT;
        order[e] = e;
    }
    std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) { return load[a] > load[b]; });
    for (uint32_t i = 0; i < E; ++i) {
        const uint32_t round = i / world, pos = i % world;
        const uint32_t rank = round % 2 == 0 ? pos : world - 1 - pos;
        owner[order[i]] = rank << 16 | round;
    }
    return K3XB_OK;
}

int k3xb_draft_greedy(k3xb_ctx* ctx, const k3xb_verify_model* m, const k3xb_draft_io* io) {
    K3XB_ENTER(ctx);
    if (!m || !io || !m->layers || !m->layer || !m->embedding)
        return fail(ctx, K3XB_INVALID_EXTENT, "draft model (needs its embedding)");
    const uint32_t S = io->sequences, p = io->drafts, K = io->draft_top_k;
    if (!S || !p || !io->anchors || !io->conv || !io->recurrent || !io->draft_tokens)
        return fail(ctx, K3XB_INVALID_EXTENT, "draft io");
    // the draft model: every MoE layer routed with draft_top_k experts
    std::unique_ptr<k3xb_layer[]> layers(new (std::nothrow) k3xb_layer[m->layers]);
    if (!layers) return fail(ctx, K3XB_BACKEND_UNAVAILABLE, "draft: out of host memory");
    for (uint32_t l = 0; l < m->layers; ++l) {
        layers[l] = m->layer[l];
        if (!K || K > layers[l].moe.top_k) return fail(ctx, K3XB_INVALID_EXTENT, "draft_top_k must be in [1, top_k]");
        layers[l].moe.top_k = K;
    }
    k3xb_verify_model dm = *m;
    dm.layer = layers.get();
    const k3xb_layer& L0 = layers[0];
    const size_t P = static_cast<size_t>(L0.kda.heads) * L0.kda.head_dim;
    const size_t conv_n = static_cast<size_t>(m->layers) * S * 3 * (L0.kda.conv_width ? L0.kda.conv_width - 1 : 0) * P;
    const size_t rec_n = static_cast<size_t>(m->layers) * S * L0.kda.heads * L0.kda.head_dim * L0.kda.head_dim;
    Sizer sz;
    sz.take<uint16_t>(conv_n);
    sz.take<float>(rec_n);
    sz.take<uint32_t>(4ull * S);
    void* base;
    int st = ensure_io(ctx, sz.used, &base);
    if (st) return st;
    Carver c(base);
    uint16_t* conv = c.take<uint16_t>(conv_n);
    float* rec = c.take<float>(rec_n);
    uint32_t* tok = c.take<uint32_t>(S);
    uint32_t* acc = c.take<uint32_t>(S);
    uint32_t* com = c.take<uint32_t>(S);
    uint32_t* cnt = c.take<uint32_t>(S);
    // the draft continues from the committed state on a copy of it
    K3XB_CUDA(ctx, cudaMemcpyAsync(conv, io->conv, conv_n * sizeof(uint16_t), cudaMemcpyDeviceToDevice, ctx->stream));
    K3XB_CUDA(ctx, cudaMemcpyAsync(rec, io->recurrent, rec_n * sizeof(float), cudaMemcpyDeviceToDevice, ctx->stream));
    K3XB_CUDA(ctx, cudaMemcpyAsync(tok, io->anchors, S * sizeof(uint32_t), cudaMemcpyDeviceToDevice, ctx->stream));
    k3xb_verify_io v{};
    v.sequences = S;
    v.drafts = 0;   // one position per sequence: a greedy decode step
    v.tokens = tok;
    v.conv = conv;
    v.recurrent = rec;
    v.mode = K3XB_ACCEPT_GREEDY;
    v.accepted = acc;
    v.committed = com;
    v.committed_count = cnt;
    for (uint32_t i = 0; i < p; ++i) {
        if ((st = k3xb_verify_step(ctx, &dm, &v))) return st;
        // committed[s][0] is the argmax after the fed token: draft i, and the next input
        K3XB_CUDA(ctx, cudaMemcpy2DAsync(io->draft_tokens + i, p * sizeof(uint32_t), com, sizeof(uint32_t),
                                         sizeof(uint32_t), S, cudaMemcpyDeviceToDevice, ctx->stream));
        K3XB_CUDA(ctx, cudaMemcpyAsync(tok, com, S * sizeof(uint32_t), cudaMemcpyDeviceToDevice, ctx->stream));
    }
    return K3XB_OK;
}

int k3xb_speculative_step(k3xb_ctx* ctx, const k3xb_verify_model* m, const k3xb_speculative_io* io) {
    K3XB_ENTER(ctx);
    if (!m || !io || !io->anchors || !io->conv || !io->recurrent || !io->draft_tokens || !io->accepted ||
        !io->committed || !io->committed_count || !io->sequences || !io->drafts)
        return fail(ctx, K3XB_INVALID_EXTENT, "speculative io");
    const uint32_t S = io->sequences, p = io->drafts;
    k3xb_draft_io d{S, p, io->draft_top_k, io->anchors, io->conv, io->recurrent, io->draft_tokens};
    int st = k3xb_draft_greedy(ctx, m, &d);
    if (st) return st;
    // anchor + drafts, per sequence (the drafter's own buffers are done with)
    void* base;
    if ((st = ensure_io(ctx, sizeof(uint32_t) * S * (p + 1), &base))) return st;
    uint32_t* tokens = static_cast<uint32_t*>(base);
    K3XB_CUDA(ctx, cudaMemcpy2DAsync(tokens, (p + 1) * sizeof(uint32_t), io->anchors, sizeof(uint32_t),
                                     sizeof(uint32_t), S, cudaMemcpyDeviceToDevice, ctx->stream));
    K3XB_CUDA(ctx, cudaMemcpy2DAsync(tokens + 1, (p + 1) * sizeof(uint32_t), io->draft_tokens, p * sizeof(uint32_t),
                                     p * sizeof(uint32_t), S, cudaMemcpyDeviceToDevice, ctx->stream));
    k3xb_verify_io v{};
    v.sequences = S;
    v.drafts = p;
    v.tokens = tokens;
    v.draft_tokens = io->draft_tokens;
    v.conv = io->conv;
    v.recurrent = io->recurrent;
    v.mode = K3XB_ACCEPT_GREEDY;
    v.logits = io->logits;
    v.accepted = io->accepted;
    v.committed = io->committed;
    v.committed_count = io->committed_count;
    if ((st = k3xb_verify_step(ctx, m, &v))) return st;
    return launch_next_anchor(ctx, io->committed, io->committed_count, S, p + 1, io->anchors);
}

int k3xb_ep_moe_layer_forward(k3xb_ctx* ctx, const k3xb_moe_layer* local, uint32_t E, const float* hidden,
                              uint32_t T, float* out, uint32_t* ids_out, float* contrib_out) {
    K3XB_ENTER(ctx);
    int st = validate_layer(ctx, local);
    if (st) return st;
    const int G = ep_world(ctx);
    if (G < 1) return fail(ctx, K3XB_INVALID_STATE, "expert parallelism not initialised (k3xb_ep_init)");
    if (local->engine != K3XB_ENGINE_MXF4) return fail(ctx, K3XB_INVALID_STATE, "expert parallelism runs the MXF4 engine");
    if (!E || E % static_cast<uint32_t>(G) || local->experts != E / static_cast<uint32_t>(G))
        return fail(ctx, K3XB_INVALID_EXTENT, "experts must split evenly: local.experts == experts_total / world");
    if (local->top_k > E || local->top_k > 32 || E > 1024 || local->top_k > 255)
        return fail(ctx, K3XB_INVALID_EXTENT, "route: need top_k <= 32 and experts <= 1024");
    if (!T || !hidden || !out) return fail(ctx, K3XB_INVALID_EXTENT, "ep forward arguments");
    if ((st = ep_reserve(ctx, T, local->top_k, expert_view(*local).hidden))) return st;
    const uint32_t K = local->top_k, H = local->hidden, Is = local->shared_inter;
    const bool shared = local->shared_gate != nullptr;
    // a LatentMoE layer sends, computes and returns latent rows (width D)
    const k3xb_moe_layer LE = expert_view(*local);
    const uint32_t D = LE.hidden;
    const size_t TD = static_cast<size_t>(T) * D, TH = static_cast<size_t>(T) * H;
    Sizer sz;
    sz.take<float>(static_cast<size_t>(T) * E);
    sz.take<uint32_t>(static_cast<size_t>(T) * K);
    sz.take<float>(static_cast<size_t>(T) * K);
    sz.take<float>(TH);
    sz.take<uint16_t>(2ull * T * H);
    sz.take<uint16_t>(2ull * T * (Is ? Is : 1));
    sz.take<uint8_t>(ep_scratch_bytes(G, T, K, D, local->experts), 1024);
    if (local->latent) {
        sz.take<float>(3 * TD);
        sz.take<float>(TH);
        sz.take<uint16_t>(2ull * T * (H > D ? H : D));
    }
    sz.used += mxf4_scratch_bytes(LE, static_cast<uint32_t>(G) * T);
    void* base;
    if ((st = ensure_scratch(ctx, sz.used, &base))) return st;
    Carver c(base);
    float* logits = c.take<float>(static_cast<size_t>(T) * E);
    uint32_t* ids = ids_out ? ids_out : c.take<uint32_t>(static_cast<size_t>(T) * K);
    if (ids_out) c.take<uint32_t>(static_cast<size_t>(T) * K);
    float* contrib = contrib_out ? contrib_out : c.take<float>(static_cast<size_t>(T) * K);
    if (contrib_out) c.take<float>(static_cast<size_t>(T) * K);
    float* shared_out = c.take<float>(static_cast<size_t>(T) * H);
    uint16_t* sxb = c.take<uint16_t>(2ull * T * H);
    uint16_t* sbd = c.take<uint16_t>(2ull * T * (Is ? Is : 1));
    void* region = c.take<uint8_t>(ep_scratch_bytes(G, T, K, D, local->experts), 1024);
    float *lat = nullptr, *mixed = nullptr, *normed = nullptr, *routed = nullptr;
    uint16_t* xt = nullptr;
    if (local->latent) {
        lat = c.take<float>(TD);
        mixed = c.take<float>(TD);
        normed = c.take<float>(TD);
        routed = c.take<float>(TH);
        xt = c.take<uint16_t>(2ull * T * (H > D ? H : D));
    }
    set_mxf4_scratch(ctx, reinterpret_cast<char*>(base) + c.used);
    if (shared) {   // side stream, as in the one-GPU layer
        K3XB_CUDA(ctx, cudaEventRecord(ctx->ev_fork, ctx->stream));
        K3XB_CUDA(ctx, cudaStreamWaitEvent(ctx->side_stream, ctx->ev_fork, 0));
        cudaStream_t main = ctx->stream;
        ctx->stream = ctx->side_stream;
        {
            PhaseScope ph(ctx, K3XB_PHASE_SHARED);
            st = launch_shared_tc(ctx, *local, hidden, T, sxb, sbd, shared_out);
        }
        ctx->stream = main;
        if (st) return st;
        K3XB_CUDA(ctx, cudaEventRecord(ctx->ev_join, ctx->side_stream));
    }
    {
        PhaseScope ph(ctx, K3XB_PHASE_ROUTE);
        if ((st = launch_router_logits(ctx, hidden, T, H, local->router, E, logits))) return st;
        if ((st = launch_topk(ctx, logits, local->correction, T, E, K, ids, contrib, nullptr, ctx->status_word)))
            return st;
    }
    if (!local->latent) {
        if (shared) K3XB_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, ctx->ev_join, 0));
        if ((st = ep_moe_forward(ctx, *local, E, hidden, T, ids, contrib, shared ? shared_out : nullptr, region,
                                 out, false)))
            return st;
    } else {   // official_moe.cpp:296, then the experts on latent rows, then :322-336
        {
            PhaseScope ph(ctx, K3XB_PHASE_LATENT);
            if ((st = launch_linear_bf16(ctx, hidden, local->routed_down, T, D, H, 1, xt, lat))) return st;
        }
        if ((st = ep_moe_forward(ctx, LE, E, lat, T, ids, contrib, nullptr, region, mixed, true))) return st;
        PhaseScope ph(ctx, K3XB_PHASE_LATENT);
        if ((st = launch_rms_norm(ctx, mixed, local->routed_norm, T, D, local->latent_eps, normed))) return st;
        if ((st = launch_linear_bf16(ctx, normed, local->routed_up, T, H, D, 1, xt, routed))) return st;
        if (shared) K3XB_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, ctx->ev_join, 0));
        st = shared ? launch_residual(ctx, routed, shared_out, TH, out) : launch_residual_round(ctx, routed, TH, out);
        if (st) return st;
    }
    ++ctx->stats.moe_layer_calls;
    return K3XB_OK;
}

}  // extern "C"
