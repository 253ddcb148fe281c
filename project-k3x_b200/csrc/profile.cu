// profile.cu — phase timing: NVTX ranges always, CUDA event pairs when
// profiling is on (see profile.cuh). C ABI: k3xb_set_profiling,
// k3xb_get_profile, k3xb_phase_name.
#include <vector>

#include "profile.cuh"

namespace k3xb {
namespace {

constexpr int kMaxPending = 4096;

const char* const kNames[] = {"route",         "plan",          "expert_prep",   "expert_gateup", "expert_down",
                              "shared",        "combine",       "ep_dispatch",   "ep_exchange",   "ep_return",
                              "attn_residual", "kda_project",   "kda_conv",      "kda_recurrence", "kda_output",
                              "embed",         "lm_head",       "accept",        "commit",        "latent"};
static_assert(sizeof(kNames) / sizeof(kNames[0]) == K3XB_PHASE_COUNT, "one name per phase");

struct Profiler {
    std::vector<cudaEvent_t> start, stop;   // event pairs, created on first use
    std::vector<int> phase;                 // phase of each pending pair; -1 = not usable
    int pending = 0;
    bool on = false;
    double ms[K3XB_PHASE_COUNT] = {};
    uint64_t calls[K3XB_PHASE_COUNT] = {};
    uint64_t dropped = 0;

    void clear() {
        pending = 0;
        dropped = 0;
        for (int i = 0; i < K3XB_PHASE_COUNT; ++i) {
            ms[i] = 0.0;
            calls[i] = 0;
        }
    }
    // A free pair, or -1.
    int take() {
        if (pending >= kMaxPending) return -1;
        if (pending == static_cast<int>(start.size())) {
            cudaEvent_t a = nullptr, b = nullptr;
            if (cudaEventCreate(&a) != cudaSuccess || cudaEventCreate(&b) != cudaSuccess) {
                cudaGetLastError();
                if (a) cudaEventDestroy(a);
                return -1;
            }
            start.push_back(a);
            stop.push_back(b);
            phase.push_back(-1);
        }
        return pending++;
    }
};

Profiler* profiler_of(k3xb_ctx* ctx) { return static_cast<Profiler*>(ctx->profiler); }

}  // namespace

const char* phase_name(int p) { return p >= 0 && p < K3XB_PHASE_COUNT ? kNames[p] : nullptr; }

PhaseScope::PhaseScope(k3xb_ctx* ctx, int phase) : ctx_(ctx), stream_(ctx->stream) {
    nvtxRangePushA(phase_name(phase));
    Profiler* p = profiler_of(ctx);
    if (!p || !p->on) return;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream_, &cs) != cudaSuccess) {
        cudaGetLastError();
        return;
    }
    if (cs != cudaStreamCaptureStatusNone) return;
    slot_ = p->take();
    if (slot_ < 0) {
        ++p->dropped;
        return;
    }
    p->phase[slot_] = cudaEventRecord(p->start[slot_], stream_) == cudaSuccess ? phase : -1;
}

void PhaseScope::end() {
    if (!open_) return;
    open_ = false;
    if (slot_ >= 0) {
        Profiler* p = profiler_of(ctx_);
        if (p->phase[slot_] >= 0 && cudaEventRecord(p->stop[slot_], stream_) != cudaSuccess) p->phase[slot_] = -1;
    }
    nvtxRangePop();
}

void release_profiler(k3xb_ctx* ctx) {
    Profiler* p = profiler_of(ctx);
    if (!p) return;
    for (size_t i = 0; i < p->start.size(); ++i) {
        cudaEventDestroy(p->start[i]);
        cudaEventDestroy(p->stop[i]);
    }
    delete p;
    ctx->profiler = nullptr;
}

}  // namespace k3xb

using namespace k3xb;

int k3xb_set_profiling(k3xb_ctx* ctx, int enable) {
    K3XB_ENTER(ctx);
    if (!ctx->profiler) {
        if (!enable) return K3XB_OK;
        ctx->profiler = new (std::nothrow) Profiler();
        if (!ctx->profiler) return fail(ctx, K3XB_BACKEND_UNAVAILABLE, "profiler: out of host memory");
    }
    Profiler* p = profiler_of(ctx);
    // pairs still in flight are waited for before they can be recorded again
    for (int i = 0; i < p->pending; ++i)
        if (p->phase[i] >= 0) cudaEventSynchronize(p->stop[i]);
    p->clear();
    p->on = enable != 0;
    return K3XB_OK;
}

int k3xb_get_profile(k3xb_ctx* ctx, k3xb_phase_time* out, uint64_t* dropped) {
    if (!ctx || !out) return K3XB_INVALID_EXTENT;
    Profiler* p = profiler_of(ctx);
    if (p) {
        for (int i = 0; i < p->pending; ++i) {
            const int ph = p->phase[i];
            if (ph < 0) continue;
            float ms = 0.0f;
            if (cudaEventSynchronize(p->stop[i]) != cudaSuccess ||
                cudaEventElapsedTime(&ms, p->start[i], p->stop[i]) != cudaSuccess) {
                cudaGetLastError();
                ++p->dropped;
                continue;
            }
            p->ms[ph] += ms;
            ++p->calls[ph];
        }
        p->pending = 0;
    }
    for (int i = 0; i < K3XB_PHASE_COUNT; ++i) {
        out[i].device_ms = p ? p->ms[i] : 0.0;
        out[i].calls = p ? p->calls[i] : 0;
    }
    if (dropped) *dropped = p ? p->dropped : 0;
    return K3XB_OK;
}

const char* k3xb_phase_name(int phase) { return phase_name(phase); }
