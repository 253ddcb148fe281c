// A scripted stand-in for the part of libk3xb's C ABI that the
// ComputeBackend adapter calls, for protocol tests on the CPU only
// (tests/cpp/adapter_protocol_check.cpp). It computes nothing of the path:
// outputs are finite placeholders. It checks what the adapter hands it:
// payload sizes against their keys, non-null arrays, and the held KDA
// slots' seed-before-continue rule, so an adapter bug shows up as a status.
#include <cstdint>
#include <cstdio>
#include <cstring>

#include "k3xb.h"

struct k3xb_ctx {
    bool held[K3XB_KDA_HELD_SLOTS] = {};
    char error[128] = {};
};

namespace {

int fail(k3xb_ctx* ctx, int st, const char* why) {
    std::snprintf(ctx->error, sizeof ctx->error, "%s", why);
    return st;
}

void fill(float* out, size_t n, float v) {
    for (size_t i = 0; i < n; ++i) out[i] = v;
}

}  // namespace

extern "C" {

int k3xb_create(int, k3xb_ctx** out) {
    *out = new k3xb_ctx();
    return K3XB_OK;
}

int k3xb_destroy(k3xb_ctx* ctx) {
    delete ctx;
    return K3XB_OK;
}

int k3xb_last_error(const k3xb_ctx* ctx, char* buf, size_t len) {
    if (!ctx || !buf || !len) return K3XB_INVALID_EXTENT;
    std::snprintf(buf, len, "%s", ctx->error);
    return K3XB_OK;
}

int k3xb_get_stats(const k3xb_ctx* ctx, k3xb_stats* out) {
    if (!ctx || !out) return K3XB_INVALID_EXTENT;
    *out = k3xb_stats{};
    return K3XB_OK;
}

int k3xb_set_resident_capacity(k3xb_ctx* ctx, uint64_t) { return ctx ? K3XB_OK : K3XB_INVALID_EXTENT; }

int k3xb_acquire_weight(k3xb_ctx* ctx, uint64_t id, int32_t repr, uint64_t rows, uint64_t cols, uint64_t group,
                        const void* primary, size_t pbytes, const void* secondary, size_t sbytes, k3xb_resident* out) {
    if (!ctx || !out || !id || !rows || !cols || !primary) return K3XB_INVALID_EXTENT;
    const bool ok = repr == K3XB_WEIGHT_F32    ? pbytes == rows * cols * 4 && !secondary
                    : repr == K3XB_WEIGHT_BF16 ? pbytes == rows * cols * 2 && !secondary
                    : repr == K3XB_WEIGHT_MXFP4
                        ? group && secondary && pbytes == rows * cols / 2 && sbytes == rows * cols / group
                        : false;
    if (!ok) return fail(ctx, K3XB_INVALID_EXTENT, "fake acquire_weight: payload does not match its key");
    *out = k3xb_resident{K3XB_RESIDENT_ADMITTED, primary, secondary, secondary, pbytes + sbytes};
    return K3XB_OK;
}

int k3xb_acquire_expert_stack(k3xb_ctx* ctx, uint64_t id, uint32_t experts, uint32_t hidden, uint32_t inter,
                              const k3xb_mxfp4_expert_host* host, k3xb_resident_stack* out) {
    if (!ctx || !out || !host || !id || !experts || hidden % 128 || inter % 128) return K3XB_INVALID_EXTENT;
    *out = k3xb_resident_stack{K3XB_RESIDENT_ADMITTED, host->gate_packed, host->gate_scales, host->up_packed,
                               host->up_scales, host->down_packed, host->down_scales, host->gate_scales,
                               host->up_scales, host->down_scales, 0};
    return K3XB_OK;
}

int k3xb_expert_grid_host(k3xb_ctx* ctx, const k3xb_moe_layer* layer, const uint32_t* ids, uint32_t n,
                          const float* x, uint32_t T, float* out) {
    if (!ctx || !layer || !ids || !n || !x || !T || !out) return K3XB_INVALID_EXTENT;
    fill(out, static_cast<size_t>(n) * T * (layer->latent ? layer->latent : layer->hidden), 0.0f);
    return K3XB_OK;
}

int k3xb_kda_block_host(k3xb_ctx* ctx, const k3xb_kda_layer* w, uint32_t H, const float* x, uint32_t T,
                        uint16_t* conv, float* rec, float* out) {
    if (!ctx || !w || !H || !x || !T || !conv || !rec || !out) return K3XB_INVALID_EXTENT;
    for (size_t i = 0; i < static_cast<size_t>(T) * H; ++i) out[i] = 0.5f * x[i];
    return K3XB_OK;
}

int k3xb_kda_block_held(k3xb_ctx* ctx, const k3xb_kda_layer* w, uint32_t H, const float* x, uint32_t T,
                        uint32_t slot, int32_t mode, uint16_t* conv, float* rec, float* out) {
    if (!ctx || !w || !H || !x || !T || !out || slot >= K3XB_KDA_HELD_SLOTS) return K3XB_INVALID_EXTENT;
    if (mode == K3XB_KDA_SEED) {
        if (!conv || !rec) return fail(ctx, K3XB_INVALID_EXTENT, "fake kda_block_held: a seed brings its state");
        ctx->held[slot] = true;
    } else if (!ctx->held[slot]) {
        return fail(ctx, K3XB_INVALID_STATE, "fake kda_block_held: nothing held in the slot");
    }
    if (mode == K3XB_KDA_PUBLISH) {
        if (!conv || !rec) return fail(ctx, K3XB_INVALID_EXTENT, "fake kda_block_held: publish needs the arrays");
        const size_t P = static_cast<size_t>(w->heads) * w->head_dim;
        std::memset(conv, 0, 3 * (w->conv_width - 1) * P * sizeof(uint16_t));
        fill(rec, P * w->head_dim, 0.0f);
    }
    for (size_t i = 0; i < static_cast<size_t>(T) * H; ++i) out[i] = 0.5f * x[i];
    return K3XB_OK;
}

int k3xb_official_moe_ffn_host(k3xb_ctx* ctx, const k3xb_moe_layer* tail, const k3xb_moe_layer* slots, uint32_t K,
                               const float* contributions, const float* hidden, const float* prefix, float* out) {
    if (!ctx || !tail || !slots || !K || !contributions || !hidden || !prefix || !out) return K3XB_INVALID_EXTENT;
    for (uint32_t k = 0; k < K; ++k)
        if (slots[k].experts != 1 || !slots[k].gate_packed || !slots[k].down_scales)
            return fail(ctx, K3XB_INVALID_MXFP4, "fake official_moe_ffn_host: a slot is not one expert");
    std::memcpy(out, prefix, sizeof(float) * tail->hidden);
    return K3XB_OK;
}

int k3xb_prepare_moe_route_host(k3xb_ctx* ctx, const float* a, const float* delta, const float* block, uint32_t H,
                                const uint16_t* rnorm, const uint16_t* rproj, const uint16_t* post, float eps,
                                const uint16_t* router, uint32_t E, float* prefix_out, float* hidden_out,
                                float* logits_out) {
    if (!ctx || !a || !block || !H || !rnorm || !rproj || !post || !(eps > 0.0f) || !hidden_out ||
        (delta && !prefix_out) || (router && (!E || !logits_out)))
        return K3XB_INVALID_EXTENT;
    for (uint32_t i = 0; i < H; ++i) {
        hidden_out[i] = a[i];
        if (delta) prefix_out[i] = a[i] + delta[i];
    }
    if (router)
        for (uint32_t e = 0; e < E; ++e) logits_out[e] = 0.01f * static_cast<float>(e % 7);
    return K3XB_OK;
}

int k3xb_dense_matvec_host(k3xb_ctx* ctx, const float* W, uint32_t rows, uint32_t cols, const float* x, float* y) {
    if (!ctx || !W || !rows || !cols || !x || !y) return K3XB_INVALID_EXTENT;
    fill(y, rows, 0.0f);
    return K3XB_OK;
}

int k3xb_dense_situ_mlp_host(k3xb_ctx* ctx, const float* g, const float* u, const float* d, uint32_t inter,
                             uint32_t cols, uint32_t out_rows, const float* x, float beta, float, float* y) {
    if (!ctx || !g || !u || !d || !inter || !cols || !out_rows || !x || !(beta > 0.0f) || !y)
        return K3XB_INVALID_EXTENT;
    fill(y, out_rows, 0.0f);
    return K3XB_OK;
}

int k3xb_mxfp4_matvec_host(k3xb_ctx* ctx, const uint8_t* packed, const uint8_t* scales, uint32_t rows, uint32_t cols,
                           const float* x, float* y) {
    if (!ctx || !packed || !scales || !rows || !cols || !x || !y) return K3XB_INVALID_EXTENT;
    fill(y, rows, 0.0f);
    return K3XB_OK;
}

int k3xb_resident_moe_layer_host(k3xb_ctx* ctx, uint32_t H, uint32_t, uint32_t, uint32_t, const float*, const float*,
                                 const float*, const float*, const float*, const float*,
                                 const k3xb_mxfp4_expert* experts, uint32_t K, const float* c, float, float, float,
                                 const float* x, float* y) {
    if (!ctx || !H || !experts || !K || !c || !x || !y) return K3XB_INVALID_EXTENT;
    fill(y, H, 0.0f);
    return K3XB_OK;
}

}  // extern "C"
