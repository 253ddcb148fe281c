// resident.cu — the context's resident weight table (resident.hpp) on the
// device: cudaMalloc'd entries, host->device copies on the context's stream,
// and the tcgen05 scale re-layout of experts_tc.cu. C ABI:
// k3xb_set_resident_capacity, k3xb_acquire_weight,
// k3xb_acquire_expert_stack, k3xb_release_resident.
#include "kernels.cuh"
#include "resident.hpp"

namespace k3xb {
namespace {

class CudaArena final : public DeviceArena {
public:
    explicit CudaArena(k3xb_ctx* ctx) : ctx_(ctx) {}
    int allocate(size_t bytes, void** out) override {
        *out = nullptr;
        if (cudaMalloc(out, bytes) != cudaSuccess) {
            cudaGetLastError();
            *out = nullptr;
            return K3XB_BACKEND_UNAVAILABLE;
        }
        return K3XB_OK;
    }
    void release(void* p) noexcept override {
        if (p) cudaFree(p);
    }
    int upload(void* dst, const void* src, size_t bytes) override {
        if (!bytes) return K3XB_OK;
        if (cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx_->stream) != cudaSuccess)
            return K3XB_BACKEND_UNAVAILABLE;
        return K3XB_OK;
    }
    int relayout_scales(const void* scales, uint64_t rows, uint64_t cols, void* out) override {
        return prepare_mxfp4_scales(ctx_, static_cast<const uint8_t*>(scales), rows, cols,
                                    static_cast<uint8_t*>(out));
    }

private:
    k3xb_ctx* ctx_;
};

struct Resident {
    explicit Resident(k3xb_ctx* ctx) : arena(ctx), table(&arena) {}
    CudaArena arena;
    ResidentTable table;
};

Resident* resident_of(k3xb_ctx* ctx) {
    if (!ctx->resident) ctx->resident = new (std::nothrow) Resident(ctx);
    return static_cast<Resident*>(ctx->resident);
}

}  // namespace

void release_resident(k3xb_ctx* ctx) {
    if (!ctx->resident) return;
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    delete static_cast<Resident*>(ctx->resident);
    ctx->resident = nullptr;
}

void resident_stats(const k3xb_ctx* ctx, k3xb_stats* out) {
    if (!ctx->resident) return;
    const ResidentCounters& c = static_cast<const Resident*>(ctx->resident)->table.counters();
    out->weight_cache_hits = c.hits;
    out->weight_cache_misses = c.misses;
    out->weight_cache_bypasses = c.bypasses;
    out->resident_weight_bytes = c.resident_bytes;
    out->peak_resident_weight_bytes = c.peak_resident_bytes;
    out->weight_h2d_bytes = c.uploaded_bytes;
}

}  // namespace k3xb

using namespace k3xb;

int k3xb_set_resident_capacity(k3xb_ctx* ctx, uint64_t bytes) {
    K3XB_ENTER(ctx);
    Resident* r = resident_of(ctx);
    if (!r) return fail(ctx, K3XB_BACKEND_UNAVAILABLE, "resident table: out of host memory");
    r->table.set_capacity(bytes);
    return K3XB_OK;
}

int k3xb_acquire_weight(k3xb_ctx* ctx, uint64_t tensor_id, int32_t representation, uint64_t rows, uint64_t cols,
                        uint64_t group_size, const void* primary, size_t primary_bytes, const void* secondary,
                        size_t secondary_bytes, k3xb_resident* out) {
    K3XB_ENTER(ctx);
    if (!out) return fail(ctx, K3XB_INVALID_EXTENT, "acquire_weight: null result");
    Resident* r = resident_of(ctx);
    if (!r) return fail(ctx, K3XB_BACKEND_UNAVAILABLE, "resident table: out of host memory");
    const char* why = "";
    const int st = r->table.acquire(ResidentKey{tensor_id, representation, rows, cols, group_size}, primary,
                                    primary_bytes, secondary, secondary_bytes, out, &why);
    if (st) return fail(ctx, st, why);
    ctx->stats.h2d_bytes += out->uploaded_bytes;
    return K3XB_OK;
}

int k3xb_acquire_expert_stack(k3xb_ctx* ctx, uint64_t stack_id, uint32_t experts, uint32_t hidden, uint32_t inter,
                              const k3xb_mxfp4_expert_host* host, k3xb_resident_stack* out) {
    K3XB_ENTER(ctx);
    if (!out) return fail(ctx, K3XB_INVALID_EXTENT, "acquire_expert_stack: null result");
    Resident* r = resident_of(ctx);
    if (!r) return fail(ctx, K3XB_BACKEND_UNAVAILABLE, "resident table: out of host memory");
    const char* why = "";
    const int st = r->table.acquire_stack(stack_id, experts, hidden, inter, host, out, &why);
    if (st) return fail(ctx, st, why);
    ctx->stats.h2d_bytes += out->uploaded_bytes;
    return K3XB_OK;
}

int k3xb_release_resident(k3xb_ctx* ctx) {
    K3XB_ENTER(ctx);
    if (!ctx->resident) return K3XB_OK;
    if (const int st = stream_wait(ctx)) return st;
    static_cast<Resident*>(ctx->resident)->table.clear();   // keeps the capacity and counters
    return K3XB_OK;
}
