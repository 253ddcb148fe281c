// The adapter's token and slot rules against the reference's own drivers,
// on the CPU: official_layer_cuda (host and device route preparation, the
// KDA state seeded and published across two calls) and
// official_two_layer_cuda (host_round_trip and device_closure), unchanged
// reference code, run over B200Backend linked with a scripted C ABI
// (fake_k3xb.cpp, placeholder arithmetic). The drivers check every token,
// publication flag and output size they get back, so a run that succeeds
// means the adapter keeps the protocol; the numbers are not looked at.
#include <cstdio>
#include <vector>

#include "backend_b200.hpp"
#include "k3x/official_layer.hpp"
#include "k3x/official_two_layer.hpp"

#define CHECK(cond)                                                              \
    do {                                                                         \
        if (!(cond)) {                                                           \
            std::fprintf(stderr, "check failed: %s (line %d)\n", #cond, __LINE__); \
            return 1;                                                            \
        }                                                                        \
    } while (0)

namespace {

using namespace k3x;

constexpr std::size_t H = 128, h = 2, d = 64, W = 4, P = h * d, E = 8, K = 2, I = 128, D = 128, S = 128;

// One layer's weights (zeros; MXFP4 scales 1.0) and the reference's views of
// them, every tensor with its own id from `id`.
struct Layer {
    std::vector<std::uint16_t> bf16_h, bf16_d, proj_h, qkv, fa, fb, bp, gp, op, router, rdown, rup, sgate, sup, sdown;
    std::vector<float> conv, alog, dtb, onorm, corr;
    std::vector<std::byte> packed, scales, dpacked, dscales;
    std::vector<OfficialExpertView> experts;
    OfficialLayerCudaWeights w{};
    Layer(const Layer&) = delete;

    explicit Layer(std::uint64_t id)
        : bf16_h(H, 0x3f80), bf16_d(D, 0x3f80), proj_h(H), qkv(P * H), fa(d * H), fb(P * d), bp(h * H), gp(P * H),
          op(H * P), router(E * H), rdown(D * H), rup(H * D), sgate(S * H), sup(S * H), sdown(H * S), conv(P * W),
          alog(d), dtb(P), onorm(d, 1.0F), corr(E), packed(I * D / 2), scales(I * D / 32, std::byte{127}),
          dpacked(D * I / 2), dscales(D * I / 32, std::byte{127}) {
        const auto mat = [&](const std::vector<std::uint16_t>& v, std::size_t r, std::size_t c) {
            return Bf16WeightView{v, r, c, id++};
        };
        const auto vec = [&](const std::vector<std::uint16_t>& v) { return Bf16VectorView{v, id++}; };
        experts.resize(E);
        for (std::size_t e = 0; e < E; ++e) {
            experts[e].expert_id = static_cast<std::uint32_t>(e);
            experts[e].weights.gate = {id++, packed, scales, I, D, 32};
            experts[e].weights.up = {id++, packed, scales, I, D, 32};
            experts[e].weights.down = {id++, dpacked, dscales, D, I, 32};
        }
        w.self_residual_norm = vec(bf16_h);
        w.self_residual_proj = mat(proj_h, 1, H);
        w.input_norm = vec(bf16_h);
        w.kda = {mat(qkv, P, H), mat(qkv, P, H), mat(qkv, P, H), {id++, conv, P, W}, {id++, conv, P, W},
                 {id++, conv, P, W}, mat(fa, d, H), mat(fb, P, d), {id++, alog}, {id++, dtb}, mat(bp, h, H),
                 mat(gp, P, H), {id++, onorm}, mat(op, H, P)};
        w.moe.residual_norm = vec(bf16_h);
        w.moe.residual_proj = mat(proj_h, 1, H);
        w.moe.post_norm = vec(bf16_h);
        w.moe.router = mat(router, E, H);
        w.moe.correction = corr;
        w.moe.routed_down = mat(rdown, D, H);
        w.moe.routed_norm = vec(bf16_d);
        w.moe.routed_up = mat(rup, H, D);
        w.moe.shared = {mat(sgate, S, H), mat(sup, S, H), mat(sdown, H, S)};
        w.moe.experts = experts;
        w.moe_ffn = {w.moe.routed_down, w.moe.routed_norm, w.moe.routed_up, w.moe.shared};
    }
};

OfficialKdaState zero_state() {
    return {std::vector<std::uint16_t>((W - 1) * P), std::vector<std::uint16_t>((W - 1) * P),
            std::vector<std::uint16_t>((W - 1) * P), std::vector<float>(h * d * d)};
}

std::vector<OfficialLayerInput> inputs(std::size_t T) {
    std::vector<OfficialLayerInput> in(T);
    for (std::size_t t = 0; t < T; ++t) in[t] = {std::vector<float>(H, 0.25F * (t + 1)), std::vector<float>(H, 0.5F)};
    return in;
}

int layer_driver(ComputeBackend& b, const Layer& L) {
    const OfficialKdaConfig cfg{H, h, d, W, 1e-6F, -5.0F};
    const auto in = inputs(5);
    for (const auto route : {OfficialMoeRoutePreparationMode::host, OfficialMoeRoutePreparationMode::device}) {
        auto r = official_layer_cuda(b, in, L.w, zero_state(), cfg, K, 0x1p64F, std::nullopt, 1,
                                     ProfilePhase::decode, {}, route);
        if (!r) std::fprintf(stderr, "official_layer_cuda: %s\n", r.message().c_str());
        CHECK(r && r.value().steps.size() == 5 && r.value().kda_state_published);
        for (const auto& s : r.value().steps) CHECK(s.output.size() == H && s.route.expert_ids.size() == K);
        // the state kept on the device across two calls
        const std::vector<OfficialLayerInput> first(in.begin(), in.begin() + 2), rest(in.begin() + 2, in.end());
        auto a = official_layer_cuda(b, first, L.w, zero_state(), cfg, K, 0x1p64F, std::nullopt, 1,
                                     ProfilePhase::decode, {OfficialKdaStateMode::device_seed, {}}, route);
        CHECK(a && a.value().kda_device_state.owner && !a.value().kda_state_published);
        auto c = official_layer_cuda(b, rest, L.w, OfficialKdaState{}, cfg, K, 0x1p64F, std::nullopt, 1,
                                     ProfilePhase::decode,
                                     {OfficialKdaStateMode::device_publish, a.value().kda_device_state}, route);
        if (!c) std::fprintf(stderr, "device_publish: %s\n", c.message().c_str());
        CHECK(c && c.value().kda_state_published && c.value().kda_state.recurrent_v_first.size() == h * d * d);
        // that state was consumed: the old token is refused
        CHECK(b.discard_official_kda_device_state(a.value().kda_device_state).error() == ErrorCode::invalid_state);
    }
    return 0;
}

int two_layer_driver(ComputeBackend& b, const Layer& l1, const Layer& l2) {
    const OfficialKdaConfig cfg{H, h, d, W, 1e-6F, -5.0F};
    const std::vector<OfficialTwoLayerCudaWeights> layers{{1, l1.w}, {2, l2.w}};
    const std::vector<OfficialKdaState> states{zero_state(), zero_state()};
    for (int round = 0; round < 2; ++round)   // twice: nothing leaks from one run into the next
        for (const auto mode : {OfficialTwoLayerCudaMode::host_round_trip, OfficialTwoLayerCudaMode::device_closure}) {
            auto r = official_two_layer_cuda(b, inputs(2), layers, states, cfg, K, 0x1p64F, std::nullopt,
                                             ProfilePhase::decode, mode, nullptr, nullptr);
            if (!r) std::fprintf(stderr, "official_two_layer_cuda: %s\n", r.message().c_str());
            CHECK(r && r.value().executed && r.value().steps.size() == 4);
            CHECK(r.value().outputs[0].size() == H && r.value().outputs[1].size() == H);
            CHECK(r.value().final_states[0].recurrent_v_first.size() == h * d * d &&
                  r.value().final_states[1].recurrent_v_first.size() == h * d * d);
        }
    return 0;
}

}  // namespace

int main() {
    BackendOptions o{};
    o.kind = BackendKind::cuda_custom;
    auto made = make_b200_backend(o, 0);   // the scripted C ABI always gives a context
    if (!made) {
        std::fprintf(stderr, "make_b200_backend failed\n");
        return 1;
    }
    const Layer l1(1), l2(1000000);
    if (layer_driver(*made.value(), l1) || two_layer_driver(*made.value(), l1, l2)) return 1;
    std::printf("adapter protocol ok\n");
    return 0;
}
