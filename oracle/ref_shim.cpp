// ref_shim.cpp — extern "C" entry points over the reference's own CPU code.
//
// TEST INFRASTRUCTURE ONLY. oracle/Makefile compiles this file together with
// the reference's unmodified sources (runtime/src/{ops,official_moe,
// official_kda,official_layer,official_two_layer,expert_major,speculative,
// routing_policy,profile}.cpp, read in place from the reference checkout) into
// oracle/_ref/libk3x_ref.so. Tests use it to pin the C restatement
// (k3x_oracle.c); bench.py uses it as the timed CPU reference arm. Nothing
// here is reference source: every function below only marshals plain C
// arrays into the reference's C++ API and back.
#include "k3x/backend.hpp"
#include "k3x/expert_major.hpp"
#include "k3x/official_kda.hpp"
#include "k3x/official_layer.hpp"
#include "k3x/official_two_layer.hpp"
#include "k3x/official_moe.hpp"
#include "k3x/routing_policy.hpp"
#include "k3x/ops.hpp"
#include "k3x/speculative.hpp"
#include "ref_shim.hpp"

#include <algorithm>
#include <atomic>
#include <bit>
#include <cstdint>
#include <cstring>
#include <optional>
#include <span>
#include <thread>
#include <vector>

namespace {

using k3x::ErrorCode;

template <typename T>
int code(const k3x::Result<T>& r) {
    return r ? 0 : static_cast<int>(r.error());
}

std::span<const std::byte> bytes(const std::uint8_t* p, std::size_t n) {
    return {reinterpret_cast<const std::byte*>(p), n};
}

// Rounding helper used where the reference's own (file-local) round_bf16
// is applied by a composed step; same bit formula.
float round_bf16(float value) {
    auto bits = std::bit_cast<std::uint32_t>(value);
    if ((bits & 0x7f800000U) == 0x7f800000U) {
        if (bits & 0x007fffffU) bits |= 0x00400000U;
        return std::bit_cast<float>(bits & 0xffff0000U);
    }
    bits += 0x7fffU + ((bits >> 16U) & 1U);
    return std::bit_cast<float>(bits & 0xffff0000U);
}

std::optional<float> linear(float linear_beta) {
    return linear_beta > 0.0F ? std::optional<float>(linear_beta) : std::nullopt;
}

}  // namespace

extern "C" {


int k3xr_decode_mxfp4(const std::uint8_t* packed, const std::uint8_t* scales,
                      std::size_t rows, std::size_t cols, std::size_t group,
                      float* out) {
    auto r = k3x::decode_mxfp4(bytes(packed, rows * cols / 2),
                               bytes(scales, rows * cols / group), rows, cols, group);
    if (r) std::copy(r.value().begin(), r.value().end(), out);
    return code(r);
}

int k3xr_mxfp4_matmul(const float* x, const std::uint8_t* packed,
                      const std::uint8_t* scales, std::size_t rows,
                      std::size_t cols, std::size_t group, float* out) {
    auto r = k3x::mxfp4_matmul({x, cols}, bytes(packed, rows * cols / 2),
                               bytes(scales, rows * cols / group), rows, cols, group);
    if (r) std::copy(r.value().begin(), r.value().end(), out);
    return code(r);
}

void k3xr_situ_glu(float* out, const float* gate, const float* up, std::size_t n,
                   float beta, float linear_beta) {
    k3x::situ_glu({out, n}, {gate, n}, {up, n}, beta, linear(linear_beta));
}

// rms_norm (ops.cpp:10-18) with float weights: the key of the model's block
// attention residual (model.cpp:63-67, :652-655).
void k3xr_rms_norm(float* out, const float* x, const float* weight, std::size_t n, float eps) {
    k3x::rms_norm({out, n}, {x, n}, {weight, n}, eps);
}

// prepare_official_moe_input (official_moe.cpp:156-209): attention residual
// of {block, prefix} then RMSNorm with post_norm; only the three weights it
// reads are set.
int k3xr_prepare_moe_input(const float* prefix, const float* block, const std::uint16_t* residual_norm,
                           const std::uint16_t* residual_proj, const std::uint16_t* post_norm, std::size_t n,
                           float eps, float* out) {
    k3x::OfficialMoeWeights w{};
    w.residual_norm.values = {residual_norm, n};
    w.residual_proj.values = {residual_proj, n};
    w.residual_proj.rows = 1;
    w.residual_proj.cols = n;
    w.post_norm.values = {post_norm, n};
    const k3x::OfficialMoeInput input{std::vector<float>(prefix, prefix + n), std::vector<float>(block, block + n)};
    auto r = k3x::prepare_official_moe_input(input, w, eps);
    if (!r) return code(r);
    std::copy(r.value().begin(), r.value().end(), out);
    return 0;
}

// select_routing (routing_policy.cpp:31-159) with the outputs flattened.
int k3xr_select_routing(const float* scores, const float* bias, std::size_t experts, std::size_t natural_k,
                        int mode, std::size_t fixed_k, float mass_target, float minimum_gap,
                        std::size_t quality_floor_k, std::uint32_t* full_order, std::uint32_t* expert_ids,
                        float* weights, std::size_t* selected_k, float* stats, int* escalated) {
    k3x::RoutingPolicyConfig config{};
    config.mode = mode == 1 ? k3x::RoutingMode::fixed
                            : mode == 2 ? k3x::RoutingMode::adaptive : k3x::RoutingMode::natural;
    config.fixed_k = fixed_k;
    config.mass_target = mass_target;
    config.minimum_boundary_gap = minimum_gap;
    config.quality_floor_k = quality_floor_k;
    auto r = k3x::select_routing({scores, experts}, {bias, experts}, natural_k, config);
    if (!r) return code(r);
    const auto& d = r.value();
    if (full_order)
        for (std::size_t i = 0; i < d.full_order.size(); ++i) full_order[i] = static_cast<std::uint32_t>(d.full_order[i]);
    for (std::size_t i = 0; i < d.selected_k; ++i) {
        expert_ids[i] = static_cast<std::uint32_t>(d.expert_ids[i]);
        weights[i] = d.normalized_weights[i];
    }
    *selected_k = d.selected_k;
    stats[0] = d.normalized_entropy;
    stats[1] = d.entropy_effective_support;
    stats[2] = d.selected_cumulative_mass;
    stats[3] = d.boundary_confidence;
    *escalated = d.quality_floor_escalated ? 1 : 0;
    return 0;
}

int k3xr_route_official_moe(const float* hidden, const std::uint16_t* router,
                            std::size_t experts, std::size_t hidden_size,
                            const float* correction, std::size_t top_k,
                            std::uint32_t* ids, float* contributions, float* scores) {
    k3x::Bf16WeightView view{{router, experts * hidden_size}, experts, hidden_size, 0};
    auto r = k3x::route_official_moe({hidden, hidden_size}, view,
                                     {correction, experts}, top_k);
    if (r) {
        std::copy(r.value().expert_ids.begin(), r.value().expert_ids.end(), ids);
        std::copy(r.value().contributions.begin(), r.value().contributions.end(),
                  contributions);
        if (scores) std::copy(r.value().scores.begin(), r.value().scores.end(), scores);
    }
    return code(r);
}

int k3xr_route_official_moe_logits(const float* logits, const float* correction,
                                   std::size_t experts, std::size_t top_k,
                                   std::uint32_t* ids, float* contributions,
                                   float* scores) {
    auto r = k3x::route_official_moe_logits({logits, experts}, {correction, experts}, top_k);
    if (r) {
        std::copy(r.value().expert_ids.begin(), r.value().expert_ids.end(), ids);
        std::copy(r.value().contributions.begin(), r.value().contributions.end(),
                  contributions);
        if (scores) std::copy(r.value().scores.begin(), r.value().scores.end(), scores);
    }
    return code(r);
}

// Routes are given per token as (ids, contributions) of width counts[t].
int k3xr_expert_major_plan(const std::uint32_t* ids, const float* contributions,
                           const std::uint32_t* counts, std::size_t tokens,
                           std::uint32_t* group_expert, std::uint32_t* group_offset,
                           std::uint32_t* assign_token, std::uint32_t* assign_slot,
                           float* assign_contrib, std::size_t* group_count) {
    std::vector<k3x::ExpertMajorTokenRoute> routes(tokens);
    std::size_t at = 0;
    for (std::size_t t = 0; t < tokens; ++t) {
        routes[t].expert_ids.assign(ids + at, ids + at + counts[t]);
        routes[t].contributions.assign(contributions + at, contributions + at + counts[t]);
        at += counts[t];
    }
    auto r = k3x::build_expert_major_plan(routes);
    if (!r) return code(r);
    std::size_t pos = 0;
    const auto& plan = r.value();
    for (std::size_t g = 0; g < plan.groups.size(); ++g) {
        group_expert[g] = plan.groups[g].expert_id;
        group_offset[g] = static_cast<std::uint32_t>(pos);
        for (const auto& a : plan.groups[g].assignments) {
            assign_token[pos] = static_cast<std::uint32_t>(a.token_index);
            assign_slot[pos] = static_cast<std::uint32_t>(a.router_slot);
            assign_contrib[pos] = a.contribution;
            ++pos;
        }
    }
    group_offset[plan.groups.size()] = static_cast<std::uint32_t>(pos);
    *group_count = plan.groups.size();
    return 0;
}

int k3xr_verify_greedy_target_block(std::uint32_t anchor, const std::uint32_t* drafts,
                                    std::size_t count, std::size_t max_draft,
                                    std::size_t vocab, const std::uint32_t* targets,
                                    std::size_t* accepted, std::uint32_t* committed,
                                    std::size_t* committed_count, int* all_accepted) {
    k3x::DraftProposal proposal{anchor, std::vector<std::uint32_t>(drafts, drafts + count)};
    auto r = k3x::verify_greedy_target_block(proposal, max_draft, vocab,
                                             {targets, count + 1});
    if (!r) return code(r);
    *accepted = r.value().accepted_draft_tokens;
    *committed_count = r.value().committed_tokens.size();
    std::copy(r.value().committed_tokens.begin(), r.value().committed_tokens.end(), committed);
    *all_accepted = r.value().all_draft_tokens_accepted ? 1 : 0;
    return 0;
}

typedef int (*k3xr_target_step_fn)(void* user, std::uint32_t input, std::uint32_t* output);

int k3xr_verify_greedy_draft(std::uint32_t anchor, const std::uint32_t* drafts,
                             std::size_t count, std::size_t max_draft, std::size_t vocab,
                             k3xr_target_step_fn step, void* user, std::size_t* accepted,
                             std::uint32_t* committed, std::size_t* committed_count,
                             int* all_accepted) {
    k3x::DraftProposal proposal{anchor, std::vector<std::uint32_t>(drafts, drafts + count)};
    k3x::GreedyTargetStep target;
    if (step) {
        target = [step, user](std::uint32_t input) {
            std::uint32_t out = 0;
            int status = step(user, input, &out);
            if (status) return k3x::Result<std::uint32_t>::failure(static_cast<ErrorCode>(status));
            return k3x::Result<std::uint32_t>::success(out);
        };
    }
    auto r = k3x::verify_greedy_draft(proposal, max_draft, vocab, target);
    if (!r) return code(r);
    *accepted = r.value().accepted_draft_tokens;
    *committed_count = r.value().committed_tokens.size();
    std::copy(r.value().committed_tokens.begin(), r.value().committed_tokens.end(), committed);
    *all_accepted = r.value().all_draft_tokens_accepted ? 1 : 0;
    return 0;
}

// One routed expert through the reference primitives used by expert_ffn
// (official_moe.cpp:82-103): mxfp4_matmul, situ_glu, mxfp4_matmul, bf16 round.
static int expert_ffn(const k3xr_moe_layer& L, std::size_t e, const float* x, float* y) {
    const std::size_t H = L.hidden, I = L.inter;
    auto gate = k3x::mxfp4_matmul({x, H}, bytes(L.gate_packed + e * I * H / 2, I * H / 2),
                                  bytes(L.gate_scales + e * I * H / 32, I * H / 32), I, H, 32);
    auto up = k3x::mxfp4_matmul({x, H}, bytes(L.up_packed + e * I * H / 2, I * H / 2),
                                bytes(L.up_scales + e * I * H / 32, I * H / 32), I, H, 32);
    if (!gate) return code(gate);
    if (!up) return code(up);
    std::vector<float> act(I);
    if (L.activation == 1)
        k3x::situ_glu(act, gate.value(), up.value(), L.situ_beta, linear(L.situ_linear_beta));
    else
        k3x::situ_glu(act, gate.value(), up.value(), 0x1p64F, std::nullopt);
    auto down = k3x::mxfp4_matmul(act, bytes(L.down_packed + e * H * I / 2, H * I / 2),
                                  bytes(L.down_scales + e * H * I / 32, H * I / 32), H, I, 32);
    if (!down) return code(down);
    for (std::size_t i = 0; i < H; ++i) y[i] = round_bf16(down.value()[i]);
    return 0;
}

static int bf16_matvec(const float* x, const std::uint16_t* w, std::size_t rows,
                       std::size_t cols, float* out) {
    for (std::size_t r = 0; r < rows; ++r) {
        double sum = 0.0;
        for (std::size_t c = 0; c < cols; ++c)
            sum += static_cast<double>(k3x::decode_bf16_word(w[r * cols + c])) * x[c];
        out[r] = round_bf16(static_cast<float>(sum));
    }
    return 0;
}

// Scratch of one plain-MoE position.
struct MoeBufs {
    std::vector<float> y, mixed, shared, g, u, a;
    explicit MoeBufs(const k3xr_moe_layer& L)
        : y(L.top_k * L.hidden), mixed(L.hidden), shared(L.hidden), g(L.shared_inter), u(L.shared_inter),
          a(L.shared_inter) {}
};

// One position of the plain (hidden-space) MoE: the reference's routing,
// expert primitives and slot-ordered combine rule (official_moe.cpp:271-344
// without the latent projections); out = round_bf16(round_bf16(mix) + shared).
// With route_only the experts are not run.
static int plain_moe_position(const k3xr_moe_layer& L, const float* x, std::uint32_t* ids, float* con,
                              bool route_only, float* out, MoeBufs& b) {
    const std::size_t H = L.hidden, K = L.top_k;
    int st = k3xr_route_official_moe(x, L.router, L.experts, H, L.correction, K, ids, con, nullptr);
    if (st || route_only) return st;
    for (std::size_t s = 0; s < K && !st; ++s) st = expert_ffn(L, ids[s], x, b.y.data() + s * H);
    if (st) return st;
    std::fill(b.mixed.begin(), b.mixed.end(), 0.0F);
    for (std::size_t s = 0; s < K; ++s)
        for (std::size_t i = 0; i < H; ++i) b.mixed[i] += con[s] * b.y[s * H + i];
    for (auto& v : b.mixed) v = round_bf16(v);
    if (L.shared_gate) {
        bf16_matvec(x, L.shared_gate, L.shared_inter, H, b.g.data());
        bf16_matvec(x, L.shared_up, L.shared_inter, H, b.u.data());
        if (L.activation == 1)
            k3x::situ_glu(b.a, b.g, b.u, L.situ_beta, linear(L.situ_linear_beta));
        else
            k3x::situ_glu(b.a, b.g, b.u, 0x1p64F, std::nullopt);
        bf16_matvec(b.a.data(), L.shared_down, H, L.shared_inter, b.shared.data());
    } else {
        std::fill(b.shared.begin(), b.shared.end(), 0.0F);
    }
    for (std::size_t i = 0; i < H; ++i) out[i] = round_bf16(b.mixed[i] + b.shared[i]);
    return 0;
}

// Plain (hidden-space) MoE layer composed of the reference's routing,
// expert primitives and its slot-ordered combine rule
// (official_moe.cpp:271-344 without the latent projections). Tokens
// [token_begin, token_end) are processed with up to `threads` workers.
int k3xr_moe_layer_forward(const k3xr_moe_layer* layer, const float* hidden,
                           std::size_t token_begin, std::size_t token_end,
                           float* out, std::uint32_t* ids, float* contributions,
                           int threads) {
    const auto& L = *layer;
    const std::size_t H = L.hidden, K = L.top_k;
    std::atomic<std::size_t> next{token_begin};
    std::atomic<int> status{0};
    auto worker = [&]() {
        MoeBufs b(L);
        for (;;) {
            std::size_t t = next.fetch_add(1);
            if (t >= token_end || status.load()) break;
            const int st = plain_moe_position(L, hidden + t * H, ids + t * K, contributions + t * K, false,
                                              out + t * H, b);
            if (st) { status.store(st); break; }
        }
    };
    if (threads < 1) threads = 1;
    std::vector<std::thread> pool;
    for (int i = 1; i < threads; ++i) pool.emplace_back(worker);
    worker();
    for (auto& th : pool) th.join();
    return status.load();
}

// official_moe_cpu itself (official_moe.cpp:271-344, LatentMoE) for T
// positions: each position's input is {prefix, block}, its hidden row the
// reference's prepare_official_moe_input (with residual_norm/proj and
// post_norm), its route route_official_moe on that row. out [T][H] is the
// reference's `output` (with the prefix residual); ids/contributions [T][k].
}  // extern "C"

namespace {

std::span<const std::uint16_t> w16(const std::uint16_t* p, std::size_t n) { return {p, n}; }

// The reference's OfficialMoeWeights over a LatentMoE layer's arrays;
// `experts` receives the per-expert views it points into.
k3x::OfficialMoeWeights official_moe_weights(const k3xr_moe_layer& L, const std::uint16_t* residual_norm,
                                             const std::uint16_t* residual_proj, const std::uint16_t* post_norm,
                                             std::vector<k3x::OfficialExpertView>& experts) {
    const std::size_t H = L.hidden, I = L.inter, D = L.latent, E = L.experts;
    experts.assign(E, {});
    for (std::size_t e = 0; e < E; ++e) {
        experts[e].expert_id = static_cast<std::uint32_t>(e);
        experts[e].weights.gate = {e * 3 + 1, bytes(L.gate_packed + e * I * D / 2, I * D / 2),
                                   bytes(L.gate_scales + e * I * D / 32, I * D / 32), I, D, 32};
        experts[e].weights.up = {e * 3 + 2, bytes(L.up_packed + e * I * D / 2, I * D / 2),
                                 bytes(L.up_scales + e * I * D / 32, I * D / 32), I, D, 32};
        experts[e].weights.down = {e * 3 + 3, bytes(L.down_packed + e * D * I / 2, D * I / 2),
                                   bytes(L.down_scales + e * D * I / 32, D * I / 32), D, I, 32};
    }
    k3x::OfficialMoeWeights w{};
    w.residual_norm = {w16(residual_norm, H), 1};
    w.residual_proj = {w16(residual_proj, H), 1, H, 2};
    w.post_norm = {w16(post_norm, H), 3};
    w.router = {w16(L.router, E * H), E, H, 4};
    w.correction = {L.correction, E};
    w.routed_down = {w16(L.routed_down, D * H), D, H, 5};
    w.routed_norm = {w16(L.routed_norm, D), 6};
    w.routed_up = {w16(L.routed_up, H * D), H, D, 7};
    if (L.shared_gate) {
        w.shared.gate = {w16(L.shared_gate, L.shared_inter * H), L.shared_inter, H, 8};
        w.shared.up = {w16(L.shared_up, L.shared_inter * H), L.shared_inter, H, 9};
        w.shared.down = {w16(L.shared_down, H * L.shared_inter), H, L.shared_inter, 10};
    }
    w.experts = experts;
    return w;
}

}  // namespace

extern "C" {

int k3xr_official_moe(const k3xr_moe_layer* layer, const float* prefix, const float* block,
                      const std::uint16_t* residual_norm, const std::uint16_t* residual_proj,
                      const std::uint16_t* post_norm, float eps, std::size_t T, float* out,
                      std::uint32_t* ids, float* contributions) {
    const auto& L = *layer;
    const std::size_t H = L.hidden;
    if (!L.latent || L.activation != 0) return static_cast<int>(ErrorCode::invalid_state);
    std::vector<k3x::OfficialExpertView> experts;
    const k3x::OfficialMoeWeights w = official_moe_weights(L, residual_norm, residual_proj, post_norm, experts);
    for (std::size_t t = 0; t < T; ++t) {
        k3x::OfficialMoeInput in{std::vector<float>(prefix + t * H, prefix + (t + 1) * H),
                                 std::vector<float>(block + t * H, block + (t + 1) * H)};
        auto hidden = k3x::prepare_official_moe_input(in, w, eps);
        if (!hidden) return code(hidden);
        auto route = k3x::route_official_moe(hidden.value(), w.router, w.correction, L.top_k);
        if (!route) return code(route);
        auto r = k3x::official_moe_cpu(in, w, route.value(), eps, 0x1p64F, std::nullopt);
        if (!r) return code(r);
        std::copy(r.value().output.begin(), r.value().output.end(), out + t * H);
        std::copy(route.value().expert_ids.begin(), route.value().expert_ids.end(), ids + t * L.top_k);
        std::copy(route.value().contributions.begin(), route.value().contributions.end(),
                  contributions + t * L.top_k);
    }
    return 0;
}


// official_kda_cpu over `tokens` positions; state arrays are updated in place.
int k3xr_official_kda_cpu(const k3xr_kda_weights* w, const float* hidden,
                          std::size_t tokens, std::uint16_t* conv_q,
                          std::uint16_t* conv_k, std::uint16_t* conv_v,
                          float* recurrent, float* out) {
    const std::size_t H = w->hidden, h = w->heads, d = w->head_dim, P = h * d;
    const std::size_t W = w->conv_width;
    k3x::OfficialKdaConfig config{H, h, d, W, w->eps, w->gate_lower_bound};
    auto mat = [](const std::uint16_t* p, std::size_t rows, std::size_t cols) {
        return k3x::Bf16WeightView{{p, rows * cols}, rows, cols, 0};
    };
    k3x::OfficialKdaWeightsView view{
        mat(w->q_proj, P, H), mat(w->k_proj, P, H), mat(w->v_proj, P, H),
        {w->q_conv, P * W}, {w->k_conv, P * W}, {w->v_conv, P * W},
        mat(w->f_a_proj, d, H), mat(w->f_b_proj, P, d),
        {w->a_log, d}, {w->dt_bias, P},
        mat(w->b_proj, h, H), mat(w->g_proj, P, H),
        {w->o_norm, d}, mat(w->o_proj, H, P)};
    const std::size_t hist = (W - 1) * P;
    k3x::OfficialKdaState state{
        std::vector<std::uint16_t>(conv_q, conv_q + hist),
        std::vector<std::uint16_t>(conv_k, conv_k + hist),
        std::vector<std::uint16_t>(conv_v, conv_v + hist),
        std::vector<float>(recurrent, recurrent + h * d * d)};
    auto r = k3x::official_kda_cpu({hidden, tokens * H}, view, state, config);
    if (!r) return code(r);
    const auto& s = r.value().state;
    std::copy(s.conv_q.begin(), s.conv_q.end(), conv_q);
    std::copy(s.conv_k.begin(), s.conv_k.end(), conv_k);
    std::copy(s.conv_v.begin(), s.conv_v.end(), conv_v);
    std::copy(s.recurrent_v_first.begin(), s.recurrent_v_first.end(), recurrent);
    std::copy(r.value().output.begin(), r.value().output.end(), out);
    return 0;
}

// One KDA + plain-MoE layer for S independent sequences of T positions,
// through the reference's own functions in official_layer_cpu's order
// (official_layer.cpp:134-244, with the plain hidden-space MoE of the
// BASELINE configs in place of official_moe_cpu's LatentMoE): per position
// prepare_official_moe_input (attention residual + input norm), then
// official_kda_cpu over the sequence's positions, then per position the
// prefix round_bf16(round_bf16(hidden) + kda), the MoE input (the same
// preparation with the MoE norms), route_official_moe, the experts through
// mxfp4_matmul / situ_glu, the slot-ordered combine and the shared expert,
// and out = round_bf16(round_bf16(prefix) + combined). norms: self_residual_
// norm, self_residual_proj, input_norm, moe_residual_norm, moe_residual_proj,
// post_norm ([H] bf16 words each). Arrays are per sequence: hidden_in, block,
// out [S][T][H]; conv [S][3][(W-1)*P] and recurrent [S][h][d][d] hold the
// initial states and receive the final ones; ids [S][T][k]. Sequences are
// shared out over `threads` workers. With route_only the routed experts and
// the rest of the MoE are skipped (ids are still the route): the caller can
// then build only the experts a sample needs before it runs the layer.
int k3xr_plain_layer(const k3xr_kda_weights* kw, const k3xr_moe_layer* mw, const std::uint16_t* const norms[6],
                     float rms_eps, std::size_t S, std::size_t T, const float* hidden_in, const float* block,
                     std::uint16_t* conv, float* recurrent, float* out, std::uint32_t* ids, int route_only,
                     int threads) {
    const std::size_t H = kw->hidden, h = kw->heads, d = kw->head_dim, P = h * d, W = kw->conv_width;
    const std::size_t K = mw->top_k, hist = (W - 1) * P;
    if (mw->latent || mw->hidden != H) return static_cast<int>(ErrorCode::invalid_state);
    std::atomic<std::size_t> next{0};
    std::atomic<int> status{0};
    auto worker = [&]() {
        MoeBufs b(*mw);
        std::vector<float> xin(T * H), kda(T * H), prefix(H), moe_in(H), con(K), combined(H);
        for (;;) {
            const std::size_t sq = next.fetch_add(1);
            if (sq >= S || status.load()) break;
            const float* hin = hidden_in + sq * T * H;
            const float* blk = block + sq * T * H;
            int st = 0;
            for (std::size_t t = 0; t < T && !st; ++t)
                st = k3xr_prepare_moe_input(hin + t * H, blk + t * H, norms[0], norms[1], norms[2], H, rms_eps,
                                            xin.data() + t * H);
            std::uint16_t* cv = conv + sq * 3 * hist;
            if (!st)
                st = k3xr_official_kda_cpu(kw, xin.data(), T, cv, cv + hist, cv + 2 * hist,
                                           recurrent + sq * h * d * d, kda.data());
            for (std::size_t t = 0; t < T && !st; ++t) {
                for (std::size_t i = 0; i < H; ++i)
                    prefix[i] = round_bf16(round_bf16(hin[t * H + i]) + kda[t * H + i]);
                st = k3xr_prepare_moe_input(prefix.data(), blk + t * H, norms[3], norms[4], norms[5], H, rms_eps,
                                            moe_in.data());
                if (!st)
                    st = plain_moe_position(*mw, moe_in.data(), ids + (sq * T + t) * K, con.data(), route_only != 0,
                                            combined.data(), b);
                if (!st && !route_only)
                    for (std::size_t i = 0; i < H; ++i)
                        out[(sq * T + t) * H + i] = round_bf16(round_bf16(prefix[i]) + combined[i]);
            }
            if (st) { status.store(st); break; }
        }
    };
    if (threads < 1) threads = 1;
    std::vector<std::thread> pool;
    for (int i = 1; i < threads; ++i) pool.emplace_back(worker);
    worker();
    for (auto& th : pool) th.join();
    return status.load();
}

// official_layer_cpu itself (official_layer.cpp:134-244: attention
// residual + input norm, official_kda_cpu over the positions, then per
// position the prefix, the MoE input preparation, route_official_moe and
// official_moe_cpu with LatentMoE) for T positions of one sequence. The
// KDA state arrays hold the initial state and receive the final one;
// out [T][H] is each position's layer output, ids [T][k] its route.
}  // extern "C"

namespace {

// The reference's OfficialLayerWeights over one layer's arrays; `norms`
// are self_residual_norm, self_residual_proj, input_norm,
// moe_residual_norm, moe_residual_proj, post_norm ([H] bf16 words each).
k3x::OfficialLayerWeights official_layer_weights(const k3xr_kda_weights& kw, const k3xr_moe_layer& mw,
                                                 const std::uint16_t* const norms[6],
                                                 std::vector<k3x::OfficialExpertView>& experts) {
    const std::size_t H = kw.hidden, h = kw.heads, d = kw.head_dim, P = h * d, W = kw.conv_width;
    auto mat = [](const std::uint16_t* p, std::size_t rows, std::size_t cols) {
        return k3x::Bf16WeightView{{p, rows * cols}, rows, cols, 0};
    };
    return k3x::OfficialLayerWeights{
        {w16(norms[0], H), 11}, {w16(norms[1], H), 1, H, 12}, {w16(norms[2], H), 13},
        k3x::OfficialKdaWeightsView{
            mat(kw.q_proj, P, H), mat(kw.k_proj, P, H), mat(kw.v_proj, P, H),
            {kw.q_conv, P * W}, {kw.k_conv, P * W}, {kw.v_conv, P * W},
            mat(kw.f_a_proj, d, H), mat(kw.f_b_proj, P, d), {kw.a_log, d}, {kw.dt_bias, P},
            mat(kw.b_proj, h, H), mat(kw.g_proj, P, H), {kw.o_norm, d}, mat(kw.o_proj, H, P)},
        official_moe_weights(mw, norms[3], norms[4], norms[5], experts)};
}

}  // namespace

extern "C" {

int k3xr_official_layer(const k3xr_kda_weights* kw, const k3xr_moe_layer* mw,
                        const std::uint16_t* self_residual_norm, const std::uint16_t* self_residual_proj,
                        const std::uint16_t* input_norm, const std::uint16_t* moe_residual_norm,
                        const std::uint16_t* moe_residual_proj, const std::uint16_t* post_norm, float eps,
                        const float* hidden_in, const float* block, std::size_t T, std::uint16_t* conv_q,
                        std::uint16_t* conv_k, std::uint16_t* conv_v, float* recurrent, float* out,
                        std::uint32_t* ids) {
    const std::size_t H = kw->hidden, h = kw->heads, d = kw->head_dim, P = h * d, W = kw->conv_width;
    if (!mw->latent || mw->activation != 0 || mw->hidden != H) return static_cast<int>(ErrorCode::invalid_state);
    std::vector<k3x::OfficialExpertView> experts;
    const std::uint16_t* const norms[6] = {self_residual_norm, self_residual_proj, input_norm,
                                           moe_residual_norm,  moe_residual_proj,  post_norm};
    const k3x::OfficialLayerWeights w = official_layer_weights(*kw, *mw, norms, experts);
    const k3x::OfficialKdaConfig config{H, h, d, W, eps, kw->gate_lower_bound};
    const std::size_t hist = (W - 1) * P;
    const k3x::OfficialKdaState state{std::vector<std::uint16_t>(conv_q, conv_q + hist),
                                      std::vector<std::uint16_t>(conv_k, conv_k + hist),
                                      std::vector<std::uint16_t>(conv_v, conv_v + hist),
                                      std::vector<float>(recurrent, recurrent + h * d * d)};
    std::vector<k3x::OfficialLayerInput> inputs(T);
    for (std::size_t t = 0; t < T; ++t)
        inputs[t] = {std::vector<float>(hidden_in + t * H, hidden_in + (t + 1) * H),
                     std::vector<float>(block + t * H, block + (t + 1) * H)};
    auto r = k3x::official_layer_cpu(inputs, w, state, config, mw->top_k, 0x1p64F, std::nullopt);
    if (!r) return code(r);
    for (std::size_t t = 0; t < T; ++t) {
        const auto& step = r.value().steps[t];
        std::copy(step.moe.output.begin(), step.moe.output.end(), out + t * H);
        std::copy(step.route.expert_ids.begin(), step.route.expert_ids.end(), ids + t * mw->top_k);
    }
    const auto& s2 = r.value().kda.state;
    std::copy(s2.conv_q.begin(), s2.conv_q.end(), conv_q);
    std::copy(s2.conv_k.begin(), s2.conv_k.end(), conv_k);
    std::copy(s2.conv_v.begin(), s2.conv_v.end(), conv_v);
    std::copy(s2.recurrent_v_first.begin(), s2.recurrent_v_first.end(), recurrent);
    return 0;
}

// official_two_layer_cpu itself (official_two_layer.cpp:16-70): two
// positions, position-major through layers 1 and 2, each layer with its own
// KDA state, the block source unchanged between layers. Per layer l:
// kw[l], mw[l], norms[l][6] as for k3xr_official_layer; conv_*[l] and
// recurrent[l] hold the initial state and receive the final one. out [2][H].
int k3xr_official_two_layer(const k3xr_kda_weights* const kw[2], const k3xr_moe_layer* const mw[2],
                            const std::uint16_t* const norms[2][6], float eps, const float* hidden_in,
                            const float* block, std::uint16_t* const conv_q[2], std::uint16_t* const conv_k[2],
                            std::uint16_t* const conv_v[2], float* const recurrent[2], float* out) {
    const std::size_t H = kw[0]->hidden, h = kw[0]->heads, d = kw[0]->head_dim, P = h * d, W = kw[0]->conv_width;
    std::vector<k3x::OfficialExpertView> experts[2];
    std::vector<k3x::OfficialTwoLayerWeights> layers;
    std::vector<k3x::OfficialKdaState> states;
    const std::size_t hist = (W - 1) * P;
    for (int l = 0; l < 2; ++l) {
        if (!mw[l]->latent || mw[l]->activation != 0 || kw[l]->hidden != H || mw[l]->top_k != mw[0]->top_k)
            return static_cast<int>(ErrorCode::invalid_state);
        layers.push_back({static_cast<std::uint32_t>(l + 1), official_layer_weights(*kw[l], *mw[l], norms[l], experts[l])});
        states.push_back({std::vector<std::uint16_t>(conv_q[l], conv_q[l] + hist),
                          std::vector<std::uint16_t>(conv_k[l], conv_k[l] + hist),
                          std::vector<std::uint16_t>(conv_v[l], conv_v[l] + hist),
                          std::vector<float>(recurrent[l], recurrent[l] + h * d * d)});
    }
    std::vector<k3x::OfficialLayerInput> inputs(2);
    for (std::size_t t = 0; t < 2; ++t)
        inputs[t] = {std::vector<float>(hidden_in + t * H, hidden_in + (t + 1) * H),
                     std::vector<float>(block + t * H, block + (t + 1) * H)};
    const k3x::OfficialKdaConfig config{H, h, d, W, eps, kw[0]->gate_lower_bound};
    auto r = k3x::official_two_layer_cpu(inputs, layers, states, config, mw[0]->top_k, 0x1p64F, std::nullopt);
    if (!r) return code(r);
    for (std::size_t t = 0; t < 2; ++t) std::copy(r.value().outputs[t].begin(), r.value().outputs[t].end(), out + t * H);
    for (int l = 0; l < 2; ++l) {
        const auto& s = r.value().final_states[l];
        std::copy(s.conv_q.begin(), s.conv_q.end(), conv_q[l]);
        std::copy(s.conv_k.begin(), s.conv_k.end(), conv_k[l]);
        std::copy(s.conv_v.begin(), s.conv_v.end(), conv_v[l]);
        std::copy(s.recurrent_v_first.begin(), s.recurrent_v_first.end(), recurrent[l]);
    }
    return 0;
}

// The reference CPU backend's dense_matvec (backend_cpu.cpp:23-47) and
// dense_situ_mlp (:107-122) through make_cpu_backend. y [rows] / [out_rows].
int k3xr_dense_matvec(const float* W, std::size_t rows, std::size_t cols, const float* x, float* y) {
    auto backend = k3x::make_cpu_backend();
    auto r = backend->dense_matvec({x, cols}, k3x::DenseWeightView{1, {W, rows * cols}, rows, cols}, 0,
                                   k3x::ProfilePhase::decode);
    if (r) std::copy(r.value().begin(), r.value().end(), y);
    return code(r);
}

int k3xr_dense_situ_mlp(const float* gate, const float* up, const float* down, std::size_t inter, std::size_t cols,
                        std::size_t out_rows, const float* x, float beta, float linear_beta, float* y) {
    auto backend = k3x::make_cpu_backend();
    const k3x::DenseMlpView w{{1, {gate, inter * cols}, inter, cols},
                              {2, {up, inter * cols}, inter, cols},
                              {3, {down, out_rows * inter}, out_rows, inter}};
    auto r = backend->dense_situ_mlp({x, cols}, w, beta, linear(linear_beta), 0, k3x::ProfilePhase::decode);
    if (r) std::copy(r.value().begin(), r.value().end(), y);
    return code(r);
}

// The reference CPU backend's resident_mxfp4_moe_layer (backend_cpu.cpp:
// 305-339) for one position: f32 projections routed_down [D][H], routed_norm
// [D], routed_up [H][D], shared gate/up [S][H] and down [H][S]; K experts
// gate/up [I][D], down [D][I] (MXFP4, group 32, stacked per expert). y [H].
int k3xr_resident_moe_layer(std::size_t H, std::size_t D, std::size_t I, std::size_t S, const float* routed_down,
                            const float* routed_norm, const float* routed_up, const float* shared_gate,
                            const float* shared_up, const float* shared_down, const std::uint8_t* gate_packed,
                            const std::uint8_t* gate_scales, const std::uint8_t* up_packed,
                            const std::uint8_t* up_scales, const std::uint8_t* down_packed,
                            const std::uint8_t* down_scales, std::size_t K, const float* contributions, float eps,
                            float beta, float linear_beta, const float* x, float* y) {
    auto backend = k3x::make_cpu_backend();
    std::uint64_t id = 1;
    const k3x::ResidentMoeLayerView w{{id++, {routed_down, D * H}, D, H},
                                      {id++, {routed_norm, D}},
                                      {id++, {routed_up, H * D}, H, D},
                                      {{id++, {shared_gate, S * H}, S, H},
                                       {id++, {shared_up, S * H}, S, H},
                                       {id++, {shared_down, H * S}, H, S}}};
    std::vector<k3x::Mxfp4MlpView> experts(K);
    for (std::size_t k = 0; k < K; ++k) {
        experts[k].gate = {id++, bytes(gate_packed + k * I * D / 2, I * D / 2), bytes(gate_scales + k * I * D / 32, I * D / 32),
                           I, D, 32};
        experts[k].up = {id++, bytes(up_packed + k * I * D / 2, I * D / 2), bytes(up_scales + k * I * D / 32, I * D / 32),
                         I, D, 32};
        experts[k].down = {id++, bytes(down_packed + k * D * I / 2, D * I / 2),
                           bytes(down_scales + k * D * I / 32, D * I / 32), D, I, 32};
    }
    auto r = backend->resident_mxfp4_moe_layer({x, H}, w, experts, {contributions, K}, eps, beta, linear(linear_beta), 0,
                                               k3x::ProfilePhase::decode);
    if (r) std::copy(r.value().output.begin(), r.value().output.end(), y);
    return code(r);
}

}  // extern "C"
