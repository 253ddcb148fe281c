// Host-side checks of B200Backend (project-k3x_b200/adapter/backend_b200.cpp)
// compiled against the reference's own ComputeBackend header: every method
// reaches libk3xb or returns backend_unavailable (no CPU fallback), the
// reference's argument checks come first, and statuses pass through by
// value. A context of NULL
// stands for "no GPU": every C ABI call then returns INVALID_EXTENT, which
// shows the call reached the library.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "backend_b200.hpp"

#define CHECK(cond)                                                              \
    do {                                                                         \
        if (!(cond)) {                                                           \
            std::fprintf(stderr, "check failed: %s (line %d)\n", #cond, __LINE__); \
            return 1;                                                            \
        }                                                                        \
    } while (0)

namespace {

using namespace k3x;

// One expert's views over host buffers (rows x cols MXFP4, group 32).
struct ExpertBuffers {
    std::vector<std::byte> gp, gs, up, us, dp, ds;
    Mxfp4MlpView view{};
    ExpertBuffers(std::size_t H, std::size_t I, std::uint64_t id)
        : gp(I * H / 2), gs(I * H / 32), up(I * H / 2), us(I * H / 32), dp(H * I / 2), ds(H * I / 32) {
        view.gate = {id, gp, gs, I, H, 32};
        view.up = {id + 1, up, us, I, H, 32};
        view.down = {id + 2, dp, ds, H, I, 32};
    }
};

int factory() {
    BackendOptions o{};
    o.kind = BackendKind::cuda_custom;
    auto b = make_b200_backend(o, 0);
    if (b) {   // a B200 is present
        CHECK(b.value()->kind() == BackendKind::cuda_custom);
    } else {
        CHECK(b.error() == ErrorCode::backend_unavailable || b.error() == ErrorCode::unsupported_architecture);
    }
    return 0;
}

int unsupported_is_unavailable() {
    BackendOptions o{};
    auto b = wrap_b200_context(o, nullptr);
    CHECK(b->kind() == BackendKind::cuda_custom && !b->device_name().empty());
    CHECK(b->runtime_stats().weight_cache_hits == 0 && b->memory_stats().current_device_bytes == 0);
    const std::vector<float> x(128, 1.0F);
    // weights without a tensor id cannot stay resident: backend_unavailable, never a CPU product
    std::vector<std::byte> pk1(64), sc1(4);
    auto mv = b->mxfp4_matvec(x, Mxfp4WeightView{0, pk1, sc1, 1, 128, 32}, 0, ProfilePhase::decode);
    CHECK(!mv && mv.error() == ErrorCode::backend_unavailable);
    auto mt = b->mxfp4_matvec(x, Mxfp4WeightView{9, pk1, sc1, 1, 128, 32}, 0, ProfilePhase::decode);
    CHECK(!mt && mt.error() == ErrorCode::invalid_extent);   // tracked: the C ABI
    auto mb = b->mxfp4_matvec(x, Mxfp4WeightView{9, pk1, sc1, 2, 128, 32}, 0, ProfilePhase::decode);
    CHECK(!mb && mb.error() == ErrorCode::invalid_mxfp4);    // mxfp4_matmul's size check
    auto d = b->dense_matvec(x, DenseWeightView{0, x, 1, 128}, 0, ProfilePhase::decode);
    CHECK(!d && d.error() == ErrorCode::backend_unavailable);
    // a tracked dense weight is on the path: the C ABI (NULL context -> invalid_extent)
    auto dt = b->dense_matvec(x, DenseWeightView{1, x, 1, 128}, 0, ProfilePhase::decode);
    CHECK(!dt && dt.error() == ErrorCode::invalid_extent);
    // the CPU backend's shape check (backend_cpu.cpp:368-377) comes first
    auto ds = b->dense_matvec(std::span<const float>(x).first(100), DenseWeightView{1, x, 1, 128}, 0,
                              ProfilePhase::decode);
    CHECK(!ds && ds.error() == ErrorCode::invalid_extent);
    // on the path: reaches the C ABI (NULL context -> invalid_extent)
    ExpertBuffers e(128, 128, 10);
    const std::vector<Mxfp4MlpView> experts{e.view};
    auto g = b->mxfp4_situ_mlp_group(x, experts, 1.0e6F, std::nullopt, 0, ProfilePhase::decode);
    CHECK(!g && g.error() == ErrorCode::invalid_extent);
    const std::vector<float> c{1.0F};
    auto m = b->mxfp4_situ_moe(x, experts, c, 1.0e6F, std::nullopt, 0, ProfilePhase::decode);
    CHECK(!m && m.error() == ErrorCode::invalid_extent);
    // device KDA state modes run here too
    OfficialKdaStateControl ctl{};
    ctl.mode = OfficialKdaStateMode::device_seed;
    auto k = b->official_kda(x, OfficialKdaCudaView{}, OfficialKdaCudaStateView{}, OfficialKdaCudaConfig{}, 1,
                             ProfilePhase::decode, ctl);
    CHECK(!k && k.error() == ErrorCode::invalid_extent);
    return 0;
}

int resident_layer_checks() {
    BackendOptions o{};
    auto b = wrap_b200_context(o, nullptr);
    const std::vector<float> x(128, 1.0F);
    auto d = b->dense_matvec(x, DenseWeightView{0, x, 1, 128}, 0, ProfilePhase::decode);
    CHECK(!d && d.error() == ErrorCode::backend_unavailable);
    auto r = b->resident_mxfp4_moe_layer(x, ResidentMoeLayerView{}, {}, {}, 1e-6F, 1.0F, std::nullopt, 0,
                                         ProfilePhase::decode);
    CHECK(!r && r.error() == ErrorCode::invalid_mxfp4);   // the CPU backend's checks (backend_cpu.cpp:442-500)
    // a well-formed resident layer reaches the C ABI (NULL context -> invalid_extent)
    const std::size_t H = 128, D = 64, I = 64, S = 64;
    std::vector<float> rd(D * H), rn(D, 1.0F), ru(H * D), sg(S * H), su(S * H), sd(H * S);
    ResidentMoeLayerView rv{{1, rd, D, H}, {2, rn}, {3, ru, H, D}, {{4, sg, S, H}, {5, su, S, H}, {6, sd, H, S}}};
    ExpertBuffers e1(D, I, 10);
    const std::vector<Mxfp4MlpView> one{e1.view};
    const std::vector<float> c1{1.0F};
    auto rr = b->resident_mxfp4_moe_layer(x, rv, one, c1, 1e-6F, 4.0F, std::nullopt, 0, ProfilePhase::decode);
    CHECK(!rr && rr.error() == ErrorCode::invalid_extent);
    ResidentMoeLayerView dup = rv;
    dup.routed_up.tensor_id = 1;   // a tensor id twice
    auto rdup = b->resident_mxfp4_moe_layer(x, dup, one, c1, 1e-6F, 4.0F, std::nullopt, 0, ProfilePhase::decode);
    CHECK(!rdup && rdup.error() == ErrorCode::invalid_mxfp4);
    return 0;
}

int argument_checks() {
    BackendOptions o{};
    auto b = wrap_b200_context(o, nullptr);
    const std::vector<float> x(128, 1.0F);
    ExpertBuffers e(128, 128, 10), f(128, 128, 20);
    const std::vector<Mxfp4MlpView> one{e.view}, two{e.view, f.view}, dup{e.view, e.view};
    const std::vector<float> c1{1.0F}, c2{0.5F, 0.5F}, bad{NAN};
    const auto P = ProfilePhase::decode;
    // contributions must match the experts and be finite (backend_cpu.cpp:270-280)
    CHECK(b->mxfp4_situ_moe(x, two, c1, 1.0F, std::nullopt, 0, P).error() == ErrorCode::invalid_mxfp4);
    CHECK(b->mxfp4_situ_moe(x, one, bad, 1.0F, std::nullopt, 0, P).error() == ErrorCode::invalid_mxfp4);
    // SiTU parameters (backend_cpu.cpp:200-208)
    CHECK(b->mxfp4_situ_mlp_group(x, one, 0.0F, std::nullopt, 0, P).error() == ErrorCode::invalid_mxfp4);
    CHECK(b->mxfp4_situ_mlp_group(x, one, 1.0F, -1.0F, 0, P).error() == ErrorCode::invalid_mxfp4);
    // input width, token counts, distinct tensor ids in a grid
    CHECK(b->mxfp4_situ_mlp_group(std::span<const float>(x).first(64), one, 1.0F, std::nullopt, 0, P).error() ==
          ErrorCode::invalid_mxfp4);
    CHECK(b->mxfp4_situ_mlp_grid(x, 0, one, 1.0F, std::nullopt, 0, P).error() == ErrorCode::invalid_mxfp4);
    CHECK(b->mxfp4_situ_mlp_grid(x, 1, dup, 1.0F, std::nullopt, 0, P).error() == ErrorCode::invalid_mxfp4);
    CHECK(b->mxfp4_situ_mlp_batch(x, 2, e.view, 1.0F, std::nullopt, 0, P).error() == ErrorCode::invalid_mxfp4);
    // malformed MXFP4 views
    ExpertBuffers g(128, 128, 30);
    g.view.down.group_size = 16;
    CHECK(b->mxfp4_situ_mlp_group(x, std::vector<Mxfp4MlpView>{g.view}, 1.0F, std::nullopt, 0, P).error() ==
          ErrorCode::invalid_mxfp4);
    // shapes the tcgen05 tiles cannot take run on the CUDA-core engine: the call reaches the C ABI
    ExpertBuffers h(96, 128, 40);
    const std::vector<float> x96(96, 1.0F);
    CHECK(b->mxfp4_situ_mlp_group(x96, std::vector<Mxfp4MlpView>{h.view}, 1.0F, std::nullopt, 0, P).error() ==
          ErrorCode::invalid_extent);
    // prefetch tokens
    CHECK(b->mxfp4_situ_mlp_group_prepared(x, Mxfp4PrefetchToken{99, 0}, 1.0F, std::nullopt, 0, P).error() ==
          ErrorCode::invalid_state);
    // KDA, host-roundtrip: config and state extents (official_kda.cpp:150-180)
    OfficialKdaCudaConfig cfg{128, 2, 64, 4, 1e-5F, -5.0F};
    const std::vector<std::uint16_t> hist(3 * 128);
    const std::vector<float> rec(2 * 64 * 64);
    OfficialKdaCudaStateView st{hist, hist, hist, rec};
    const std::vector<float> x3(3 * 128, 0.0F);
    CHECK(b->official_kda(std::span<const float>(x3).first(100), OfficialKdaCudaView{}, st, cfg, 0, P).error() ==
          ErrorCode::invalid_extent);
    OfficialKdaCudaConfig pos = cfg;
    pos.gate_lower_bound = 1.0F;
    CHECK(b->official_kda(x3, OfficialKdaCudaView{}, st, pos, 0, P).error() == ErrorCode::invalid_extent);
    OfficialKdaCudaStateView short_state{std::span<const std::uint16_t>(hist).first(10), hist, hist, rec};
    CHECK(b->official_kda(x3, OfficialKdaCudaView{}, short_state, cfg, 0, P).error() == ErrorCode::invalid_extent);
    // weight views of the wrong shape
    CHECK(b->official_kda(x3, OfficialKdaCudaView{}, st, cfg, 0, P).error() == ErrorCode::invalid_extent);
    // the state modes' rules (backend_cuda.cu:2564-2625, :2691-2702)
    const auto kda = [&](OfficialKdaStateMode mode, const OfficialKdaCudaStateView& s, std::uint32_t layer,
                         OfficialKdaDeviceStateToken token = {}) {
        return b->official_kda(x3, OfficialKdaCudaView{}, s, cfg, layer, P, OfficialKdaStateControl{mode, token}).error();
    };
    using M = OfficialKdaStateMode;
    const OfficialKdaCudaStateView empty{};
    CHECK(kda(M::device_continue, st, 1) == ErrorCode::invalid_extent);            // a continuation brings no state
    CHECK(kda(M::device_seed, empty, 1) == ErrorCode::invalid_extent);             // a seed brings one
    CHECK(kda(M::host_roundtrip, empty, 1) == ErrorCode::invalid_extent);
    CHECK(kda(M::device_seed, st, 1, {5, 6}) == ErrorCode::invalid_extent);        // a seed takes no token
    CHECK(kda(M::device_seed, st, 3) == ErrorCode::invalid_state);                 // slots for layers 1 and 2 only
    CHECK(kda(M::device_continue, empty, 1, {5, 6}) == ErrorCode::invalid_state);  // nothing kept
    CHECK(kda(M::device_publish, empty, 2, {5, 6}) == ErrorCode::invalid_state);
    CHECK(b->discard_official_kda_device_state({5, 6}).error() == ErrorCode::invalid_state);
    // a seed that passes the rules reaches the weight checks (empty views: invalid_extent)
    CHECK(kda(M::device_seed, st, 1) == ErrorCode::invalid_extent);
    return 0;
}

// The official LatentMoE FFN's views: H hidden, D latent (= the experts'
// width and output width unless `dout` differs), I expert inter, S shared.
struct OfficialFfn {
    std::vector<std::uint16_t> down, norm, up, sg, su, sd;
    ExpertBuffers e1, e2;
    OfficialMoeFfnView view{};
    std::vector<Mxfp4MlpView> experts;
    OfficialFfn(std::size_t H, std::size_t D, std::size_t I, std::size_t S)
        : down(D * H), norm(D), up(H * D), sg(S * H), su(S * H), sd(H * S), e1(D, I, 200), e2(D, I, 210) {
        view.routed_down = {down, D, H, 100};
        view.routed_norm = {norm, 101};
        view.routed_up = {up, H, D, 102};
        view.shared = {{sg, S, H, 103}, {su, S, H, 104}, {sd, H, S, 105}};
        experts = {e1.view, e2.view};
    }
};

int official_ffn() {
    const auto P = ProfilePhase::decode;
    const std::vector<float> x(128, 0.5F), prefix(128, 0.25F), c{0.75F, 0.25F};
    const std::vector<std::uint32_t> ids{3, 9};
    BackendOptions o{};
    {   // on the path: reaches the C ABI (NULL context -> invalid_extent)
        auto b = wrap_b200_context(o, nullptr);
        OfficialFfn f(128, 128, 128, 128);
        auto r = b->official_mxfp4_moe_ffn(x, prefix, f.view, f.experts, ids, c, 1e-6F, 1.0F, std::nullopt, 0, P);
        CHECK(!r && r.error() == ErrorCode::invalid_extent);
        // latent 96 (a multiple of 32, not of 128): the CUDA-core engine, still the C ABI
        OfficialFfn g(128, 96, 64, 128);
        r = b->official_mxfp4_moe_ffn(x, prefix, g.view, g.experts, ids, c, 1e-6F, 1.0F, std::nullopt, 0, P);
        CHECK(!r && r.error() == ErrorCode::invalid_extent);
        // hidden not a multiple of 8: not this library's shape, so backend_unavailable (no CPU fallback)
        const std::vector<float> x12(12, 0.5F), p12(12, 0.25F);
        OfficialFfn h(12, 32, 32, 32);
        r = b->official_mxfp4_moe_ffn(x12, p12, h.view, h.experts, ids, c, 1e-6F, 1.0F, std::nullopt, 0, P);
        CHECK(!r && r.error() == ErrorCode::backend_unavailable);
    }
    auto b = wrap_b200_context(o, nullptr);
    OfficialFfn f(128, 128, 128, 128);
    const auto call = [&](std::span<const float> hx, std::span<const float> px, const OfficialMoeFfnView& v,
                          std::span<const Mxfp4MlpView> ex, std::span<const std::uint32_t> ix,
                          std::span<const float> cx, float eps = 1e-6F) {
        return b->official_mxfp4_moe_ffn(hx, px, v, ex, ix, cx, eps, 1.0F, std::nullopt, 0, P).error();
    };
    // the reference's checks (backend_cuda.cu:3770-3875): all invalid_mxfp4
    CHECK(call(x, std::span<const float>(prefix).first(64), f.view, f.experts, ids, c) == ErrorCode::invalid_mxfp4);
    CHECK(call(x, prefix, f.view, f.experts, std::span<const std::uint32_t>(ids).first(1), c) ==
          ErrorCode::invalid_mxfp4);
    CHECK(call(x, prefix, f.view, f.experts, ids, c, 0.0F) == ErrorCode::invalid_mxfp4);
    const std::vector<std::uint32_t> same{3, 3};
    CHECK(call(x, prefix, f.view, f.experts, same, c) == ErrorCode::invalid_mxfp4);       // repeated expert
    const std::vector<float> neg{1.25F, -0.25F}, off{0.5F, 0.25F};
    CHECK(call(x, prefix, f.view, f.experts, ids, neg) == ErrorCode::invalid_mxfp4);      // contribution <= 0
    CHECK(call(x, prefix, f.view, f.experts, ids, off) == ErrorCode::invalid_mxfp4);      // sum != 1
    OfficialMoeFfnView shared_id = f.view;
    shared_id.shared.up.tensor_id = 100;                                                // a tensor id twice
    CHECK(call(x, prefix, shared_id, f.experts, ids, c) == ErrorCode::invalid_mxfp4);
    OfficialMoeFfnView narrow = f.view;
    narrow.routed_norm.values = std::span<const std::uint16_t>(f.norm).first(64);       // routed width
    CHECK(call(x, prefix, narrow, f.experts, ids, c) == ErrorCode::invalid_mxfp4);
    // a routed width other than the latent width is not this library's shape
    OfficialFfn w(128, 128, 128, 128);
    const std::vector<std::uint16_t> norm64(64), up64(128 * 64);
    ExpertBuffers n1(128, 128, 320), n2(128, 128, 330);
    std::vector<std::byte> dp1(64 * 128 / 2), ds1(64 * 128 / 32), dp2(64 * 128 / 2), ds2(64 * 128 / 32);
    n1.view.down = {322, dp1, ds1, 64, 128, 32};
    n2.view.down = {332, dp2, ds2, 64, 128, 32};
    OfficialMoeFfnView v64 = w.view;
    v64.routed_norm = {norm64, 101};
    v64.routed_up = {up64, 128, 64, 102};
    const std::vector<Mxfp4MlpView> e64{n1.view, n2.view};
    CHECK(call(x, prefix, v64, e64, ids, c) == ErrorCode::backend_unavailable);

    // prepared routes (backend_cuda.cu:3478-3716): nothing prepared yet
    auto none = b->official_mxfp4_moe_ffn_prepared(OfficialMoePreparedToken{1, 1}, f.view, f.experts, ids, c, 1e-6F,
                                                   1.0F, std::nullopt, 0, P);
    CHECK(!none && none.error() == ErrorCode::invalid_mxfp4);
    CHECK(b->discard_official_moe_prepared(OfficialMoePreparedToken{1, 1}).error() == ErrorCode::invalid_state);
    // the preparation's checks: invalid_extent
    std::vector<std::uint16_t> rn(128), rp(128), pn(128), rt(8 * 128);
    OfficialMoeRoutePrepareView pv{{rn, 401}, {rp, 1, 128, 402}, {pn, 403}, {rt, 8, 128, 404}};
    const auto prep = [&](std::span<const float> px, std::span<const float> bx, const OfficialMoeRoutePrepareView& v,
                          float eps = 1e-6F) { return b->prepare_official_moe_route(px, bx, v, eps, 0, P).error(); };
    CHECK(prep(prefix, std::span<const float>(x).first(64), pv) == ErrorCode::invalid_extent);
    CHECK(prep(prefix, x, pv, -1.0F) == ErrorCode::invalid_extent);
    OfficialMoeRoutePrepareView twice = pv;
    twice.router.tensor_id = 401;
    CHECK(prep(prefix, x, twice) == ErrorCode::invalid_extent);
    OfficialMoeRoutePrepareView narrow_proj = pv;
    narrow_proj.residual_proj.cols = 64;
    CHECK(prep(prefix, x, narrow_proj) == ErrorCode::invalid_extent);
    rt[5] = 0x7f80;   // an infinite router word
    CHECK(prep(prefix, x, pv) == ErrorCode::invalid_extent);

    // a layer's front and tail (backend_cuda.cu:3161-3476)
    std::vector<std::uint16_t> sn(128), sp(128), in(128);
    OfficialLayerFrontWeights fw{{sn, 501}, {sp, 1, 128, 502}, {in, 503}, OfficialKdaCudaView{}, pv};
    const OfficialKdaCudaConfig kc{128, 2, 64, 4, 1e-5F, -5.0F};
    const auto front = [&](std::span<const float> hx, std::span<const float> bx, OfficialLayerHiddenToken tok,
                           std::uint32_t layer, OfficialKdaStateMode mode) {
        return b->official_layer_front(hx, bx, tok, fw, OfficialKdaCudaStateView{}, kc, layer, P,
                                       OfficialKdaStateControl{mode, {}})
            .error();
    };
    using M = OfficialKdaStateMode;
    const OfficialLayerHiddenToken tok{7, 1, 1, 128, 0};
    CHECK(front(x, prefix, tok, 1, M::device_seed) == ErrorCode::invalid_extent);      // host rows and a token
    CHECK(front({}, {}, {}, 1, M::device_seed) == ErrorCode::invalid_extent);          // neither
    CHECK(front(x, prefix, {}, 2, M::device_seed) == ErrorCode::invalid_extent);       // host rows: layer 1 only
    CHECK(front(x, prefix, {}, 1, M::host_roundtrip) == ErrorCode::invalid_extent);    // device state modes only
    CHECK(front(x, prefix, {}, 3, M::device_seed) == ErrorCode::invalid_extent);
    CHECK(front({}, {}, tok, 2, M::device_continue) == ErrorCode::invalid_state);      // not this backend's token
    CHECK(b->official_layer_tail(OfficialMoePreparedToken{1, 1}, f.view, f.experts, ids, c, 1e-6F, 1.0F,
                                 std::nullopt, 1, P, true)
              .error() == ErrorCode::invalid_state);                                   // nothing prepared
    CHECK(b->discard_official_layer_hidden(tok).error() == ErrorCode::invalid_state);
    return 0;
}

}  // namespace

int main() {
    if (factory() || unsupported_is_unavailable() || resident_layer_checks() || argument_checks() || official_ffn())
        return 1;
    std::printf("backend adapter ok\n");
    return 0;
}
