// ref_b200.cpp — the reference's own layer driver over this library's
// ComputeBackend.
//
// TEST INFRASTRUCTURE ONLY. oracle/Makefile compiles this file with the
// reference's unmodified official_layer_cuda (runtime/src/official_layer.cpp:
// 246-500) and the CPU pieces it calls (attention residual, RMSNorm, MoE
// input preparation and routing: official_layer.cpp, official_moe.cpp,
// ops.cpp), read in place from the reference checkout, together with the
// B200Backend adapter (project-k3x_b200/adapter/backend_b200.cpp), linked
// against libk3xb.so, into oracle/_ref/libk3x_ref_b200.so. It shows the
// drop-in: the reference's caller, unchanged, runs a whole official layer
// with its KDA block (official_kda: host-roundtrip state, or device_seed then
// device_publish across two calls) and its LatentMoE
// FFN on the B200: official_mxfp4_moe_ffn after host route preparation, or
// prepare_official_moe_route + official_mxfp4_moe_ffn_prepared after device
// route preparation. The GPU test compares the result with
// official_layer_cpu's golden output.
// Nothing here is reference source: it only marshals plain C arrays into
// the reference's C++ API and back.
#include "k3x/official_layer.hpp"
#include "k3x/official_two_layer.hpp"

#include <algorithm>
#include <array>
#include <cstdint>
#include <cstdio>
#include <optional>
#include <span>
#include <vector>

#include "backend_b200.hpp"
#include "ref_shim.hpp"

namespace {

std::span<const std::uint16_t> w16(const std::uint16_t* p, std::size_t n) { return {p, n}; }
std::span<const std::byte> bytes(const std::uint8_t* p, std::size_t n) {
    return {reinterpret_cast<const std::byte*>(p), n};
}

void message(char* err, std::size_t len, const std::string& m) {
    if (err && len) std::snprintf(err, len, "%s", m.c_str());
}

// The reference's OfficialLayerCudaWeights over a layer's plain arrays,
// every tensor with its own non-zero id (the device path keeps weights
// resident by id; ids start at `first_id`). `experts` is what w.moe.experts
// points into.
struct Norms6 {
    const std::uint16_t* v[6];
};
Norms6 norms6(const std::uint16_t* a, const std::uint16_t* b, const std::uint16_t* c, const std::uint16_t* d,
              const std::uint16_t* e, const std::uint16_t* f) {
    return {{a, b, c, d, e, f}};
}

struct LayerViews {
    std::vector<k3x::OfficialExpertView> experts;
    k3x::OfficialLayerCudaWeights w{};
    LayerViews(const LayerViews&) = delete;   // w.moe.experts points into `experts`
    LayerViews& operator=(const LayerViews&) = delete;

    LayerViews(const k3xr_kda_weights& kwr, const k3xr_moe_layer& mwr, Norms6 n, std::uint64_t first_id) {
        const k3xr_kda_weights* kw = &kwr;
        const k3xr_moe_layer* mw = &mwr;
        const std::size_t H = kw->hidden, h = kw->heads, d = kw->head_dim, P = h * d, W = kw->conv_width;
        const std::size_t E = mw->experts, I = mw->inter, D = mw->latent, S = mw->shared_inter;
        const std::uint16_t *self_residual_norm = n.v[0], *self_residual_proj = n.v[1], *input_norm = n.v[2],
                            *moe_residual_norm = n.v[3], *moe_residual_proj = n.v[4], *post_norm = n.v[5];
        std::uint64_t next_id = first_id;
        const auto mat = [&](const std::uint16_t* p, std::size_t rows, std::size_t cols) {
            return k3x::Bf16WeightView{w16(p, rows * cols), rows, cols, next_id++};
        };
        const auto vec = [&](const std::uint16_t* p, std::size_t n) { return k3x::Bf16VectorView{w16(p, n), next_id++}; };
        const auto dense = [&](const float* p, std::size_t rows, std::size_t cols) {
            return k3x::DenseWeightView{next_id++, {p, rows * cols}, rows, cols};
        };
        const auto dvec = [&](const float* p, std::size_t n) { return k3x::DenseVectorView{next_id++, {p, n}}; };

        experts.assign(E, {});
        for (std::size_t e = 0; e < E; ++e) {
            experts[e].expert_id = static_cast<std::uint32_t>(e);
            experts[e].weights.gate = {next_id++, bytes(mw->gate_packed + e * I * D / 2, I * D / 2),
                                       bytes(mw->gate_scales + e * I * D / 32, I * D / 32), I, D, 32};
            experts[e].weights.up = {next_id++, bytes(mw->up_packed + e * I * D / 2, I * D / 2),
                                     bytes(mw->up_scales + e * I * D / 32, I * D / 32), I, D, 32};
            experts[e].weights.down = {next_id++, bytes(mw->down_packed + e * D * I / 2, D * I / 2),
                                       bytes(mw->down_scales + e * D * I / 32, D * I / 32), D, I, 32};
        }
        w.self_residual_norm = vec(self_residual_norm, H);
        w.self_residual_proj = mat(self_residual_proj, 1, H);
        w.input_norm = vec(input_norm, H);
        w.kda = k3x::OfficialKdaCudaView{mat(kw->q_proj, P, H),   mat(kw->k_proj, P, H),   mat(kw->v_proj, P, H),
                                         dense(kw->q_conv, P, W), dense(kw->k_conv, P, W), dense(kw->v_conv, P, W),
                                         mat(kw->f_a_proj, d, H), mat(kw->f_b_proj, P, d), dvec(kw->a_log, d),
                                         dvec(kw->dt_bias, P),    mat(kw->b_proj, h, H),   mat(kw->g_proj, P, H),
                                         dvec(kw->o_norm, d),     mat(kw->o_proj, H, P)};
        // the host-side route preparation's weights (official_moe.cpp:156-269)
        w.moe.residual_norm = vec(moe_residual_norm, H);
        w.moe.residual_proj = mat(moe_residual_proj, 1, H);
        w.moe.post_norm = vec(post_norm, H);
        w.moe.router = mat(mw->router, E, H);
        w.moe.correction = {mw->correction, E};
        w.moe.routed_down = mat(mw->routed_down, D, H);
        w.moe.routed_norm = vec(mw->routed_norm, D);
        w.moe.routed_up = mat(mw->routed_up, H, D);
        w.moe.shared = {mat(mw->shared_gate, S, H), mat(mw->shared_up, S, H), mat(mw->shared_down, H, S)};
        w.moe.experts = experts;
        // the FFN the backend runs shares the tensors (and their ids)
        w.moe_ffn = {w.moe.routed_down, w.moe.routed_norm, w.moe.routed_up, w.moe.shared};
    }
};

}  // namespace

extern "C" {

// official_layer_cuda(B200Backend) over T positions of one layer with a
// LatentMoE (SwiGLU: situ_glu with beta 2^64, no linear bound), the
// arguments of k3xr_official_layer plus the device, the route preparation
// (0 host, 1 device) and kda_split: 0 for one call that brings the KDA state
// and takes it back, else two calls, positions [0, kda_split) with
// device_seed and the rest with device_publish from the state the device
// kept. The KDA state arrays are
// updated in place; out [T][H] and ids [T][top_k]. Returns the k3x::ErrorCode
// value; err receives the message.
int k3xr_official_layer_b200(int device, int device_route, std::size_t kda_split, const k3xr_kda_weights* kw,
                             const k3xr_moe_layer* mw,
                             const std::uint16_t* self_residual_norm, const std::uint16_t* self_residual_proj,
                             const std::uint16_t* input_norm, const std::uint16_t* moe_residual_norm,
                             const std::uint16_t* moe_residual_proj, const std::uint16_t* post_norm, float eps,
                             const float* hidden_in, const float* block, std::size_t T, std::uint16_t* conv_q,
                             std::uint16_t* conv_k, std::uint16_t* conv_v, float* recurrent, float* out,
                             std::uint32_t* ids, char* err, std::size_t err_len) {
    using k3x::ErrorCode;
    const std::size_t H = kw->hidden, h = kw->heads, d = kw->head_dim, P = h * d, W = kw->conv_width;
    const std::size_t E = mw->experts, I = mw->inter, D = mw->latent, S = mw->shared_inter;
    if (!D || mw->activation != 0 || mw->hidden != H || !S) return static_cast<int>(ErrorCode::invalid_state);

    k3x::BackendOptions options{};
    options.kind = k3x::BackendKind::cuda_custom;
    auto made = k3x::make_b200_backend(options, device);
    if (!made) {
        message(err, err_len, made.message());
        return static_cast<int>(made.error());
    }
    k3x::ComputeBackend& backend = *made.value();

    LayerViews views(*kw, *mw, norms6(self_residual_norm, self_residual_proj, input_norm, moe_residual_norm,
                                      moe_residual_proj, post_norm), 1);
    const k3x::OfficialLayerCudaWeights& w = views.w;

    const std::size_t hist = (W - 1) * P;
    const k3x::OfficialKdaState state{std::vector<std::uint16_t>(conv_q, conv_q + hist),
                                      std::vector<std::uint16_t>(conv_k, conv_k + hist),
                                      std::vector<std::uint16_t>(conv_v, conv_v + hist),
                                      std::vector<float>(recurrent, recurrent + h * d * d)};
    const k3x::OfficialKdaConfig config{H, h, d, W, eps, kw->gate_lower_bound};
    std::vector<k3x::OfficialLayerInput> inputs(T);
    for (std::size_t t = 0; t < T; ++t)
        inputs[t] = {std::vector<float>(hidden_in + t * H, hidden_in + (t + 1) * H),
                     std::vector<float>(block + t * H, block + (t + 1) * H)};
    const auto route = device_route ? k3x::OfficialMoeRoutePreparationMode::device
                                    : k3x::OfficialMoeRoutePreparationMode::host;
    const auto run = [&](std::size_t t0, std::size_t t1, const k3x::OfficialKdaState& from,
                         k3x::OfficialKdaStateControl control) {
        const std::vector<k3x::OfficialLayerInput> part(inputs.begin() + static_cast<std::ptrdiff_t>(t0),
                                                        inputs.begin() + static_cast<std::ptrdiff_t>(t1));
        return k3x::official_layer_cuda(backend, part, w, from, config, mw->top_k, 0x1p64F, std::nullopt, 1,
                                        k3x::ProfilePhase::decode, control, route);
    };
    std::vector<k3x::OfficialLayerCudaStepResult> steps;
    k3x::OfficialKdaState final_state;
    if (!kda_split || kda_split >= T) {   // one call, the state brought and taken back
        auto r = run(0, T, state, {});
        if (!r) {
            message(err, err_len, r.message());
            return static_cast<int>(r.error());
        }
        steps = std::move(r.value().steps);
        final_state = std::move(r.value().kda_state);
    } else {   // two calls: the first seeds the device-held state, the second continues it and publishes
        auto a = run(0, kda_split, state, {k3x::OfficialKdaStateMode::device_seed, {}});
        if (!a) {
            message(err, err_len, "device_seed: " + a.message());
            return static_cast<int>(a.error());
        }
        auto b = run(kda_split, T, k3x::OfficialKdaState{},
                     {k3x::OfficialKdaStateMode::device_publish, a.value().kda_device_state});
        if (!b) {
            message(err, err_len, "device_publish: " + b.message());
            return static_cast<int>(b.error());
        }
        steps = std::move(a.value().steps);
        for (auto& s : b.value().steps) steps.push_back(std::move(s));
        final_state = std::move(b.value().kda_state);
    }
    for (std::size_t t = 0; t < T; ++t) {
        const auto& step = steps[t];
        std::copy(step.output.begin(), step.output.end(), out + t * H);
        std::copy(step.route.expert_ids.begin(), step.route.expert_ids.end(), ids + t * mw->top_k);
    }
    const auto& s = final_state;
    std::copy(s.conv_q.begin(), s.conv_q.end(), conv_q);
    std::copy(s.conv_k.begin(), s.conv_k.end(), conv_k);
    std::copy(s.conv_v.begin(), s.conv_v.end(), conv_v);
    std::copy(s.recurrent_v_first.begin(), s.recurrent_v_first.end(), recurrent);
    return 0;
}

// official_two_layer_cuda (official_two_layer.cpp:102-414) over
// B200Backend: two positions, position-major through layers 1 and 2, each
// layer's KDA state seeded on the device at position 0 and published at
// position 1 (device_seed / device_publish). host_round_trip mode: each
// layer an official_layer_cuda with device route preparation;
// device_closure: official_layer_front / _tail, layer 1's output held for
// layer 2's front. The arguments of k3xr_official_two_layer plus the device
// and the mode; the state arrays receive the final states, out [2][H], ids
// [2 positions][2 layers][top_k].
int k3xr_official_two_layer_b200(int device, int device_closure, const k3xr_kda_weights* const kw[2],
                                 const k3xr_moe_layer* const mw[2],
                                 const std::uint16_t* const norms[2][6], float eps, const float* hidden_in,
                                 const float* block, std::uint16_t* const conv_q[2], std::uint16_t* const conv_k[2],
                                 std::uint16_t* const conv_v[2], float* const recurrent[2], float* out,
                                 std::uint32_t* ids, char* err, std::size_t err_len) {
    using k3x::ErrorCode;
    const std::size_t H = kw[0]->hidden, h = kw[0]->heads, d = kw[0]->head_dim, P = h * d, W = kw[0]->conv_width;
    for (int l = 0; l < 2; ++l)
        if (!mw[l]->latent || mw[l]->activation != 0 || mw[l]->hidden != H || kw[l]->hidden != H ||
            !mw[l]->shared_inter || mw[l]->top_k != mw[0]->top_k)
            return static_cast<int>(ErrorCode::invalid_state);
    k3x::BackendOptions options{};
    options.kind = k3x::BackendKind::cuda_custom;
    auto made = k3x::make_b200_backend(options, device);
    if (!made) {
        message(err, err_len, made.message());
        return static_cast<int>(made.error());
    }
    const auto norms_of = [&](int l) {
        return norms6(norms[l][0], norms[l][1], norms[l][2], norms[l][3], norms[l][4], norms[l][5]);
    };
    LayerViews l1(*kw[0], *mw[0], norms_of(0), 1), l2(*kw[1], *mw[1], norms_of(1), 1000000);
    const std::array<k3x::OfficialTwoLayerCudaWeights, 2> layers{{{1, l1.w}, {2, l2.w}}};
    const std::size_t hist = (W - 1) * P;
    std::array<k3x::OfficialKdaState, 2> states;
    for (int l = 0; l < 2; ++l)
        states[l] = {std::vector<std::uint16_t>(conv_q[l], conv_q[l] + hist),
                     std::vector<std::uint16_t>(conv_k[l], conv_k[l] + hist),
                     std::vector<std::uint16_t>(conv_v[l], conv_v[l] + hist),
                     std::vector<float>(recurrent[l], recurrent[l] + h * d * d)};
    std::vector<k3x::OfficialLayerInput> inputs(2);
    for (std::size_t t = 0; t < 2; ++t)
        inputs[t] = {std::vector<float>(hidden_in + t * H, hidden_in + (t + 1) * H),
                     std::vector<float>(block + t * H, block + (t + 1) * H)};
    const k3x::OfficialKdaConfig config{H, h, d, W, eps, kw[0]->gate_lower_bound};
    auto r = k3x::official_two_layer_cuda(*made.value(), inputs, layers, states, config, mw[0]->top_k, 0x1p64F,
                                          std::nullopt, k3x::ProfilePhase::decode,
                                          device_closure ? k3x::OfficialTwoLayerCudaMode::device_closure
                                                         : k3x::OfficialTwoLayerCudaMode::host_round_trip,
                                          nullptr, nullptr);
    if (!r) {
        message(err, err_len, r.message());
        return static_cast<int>(r.error());
    }
    for (std::size_t t = 0; t < 2; ++t) std::copy(r.value().outputs[t].begin(), r.value().outputs[t].end(), out + t * H);
    // routes [position][layer][top_k], from the steps (position-major)
    for (const auto& step : r.value().steps)
        std::copy(step.route.expert_ids.begin(), step.route.expert_ids.end(),
                  ids + (step.position * 2 + (step.layer_id - 1)) * mw[0]->top_k);
    for (int l = 0; l < 2; ++l) {
        const auto& s = r.value().final_states[l];
        std::copy(s.conv_q.begin(), s.conv_q.end(), conv_q[l]);
        std::copy(s.conv_k.begin(), s.conv_k.end(), conv_k[l]);
        std::copy(s.conv_v.begin(), s.conv_v.end(), conv_v[l]);
        std::copy(s.recurrent_v_first.begin(), s.recurrent_v_first.end(), recurrent[l]);
    }
    return 0;
}

}  // extern "C"
