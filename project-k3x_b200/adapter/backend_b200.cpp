// backend_b200.cpp — B200Backend: k3x::ComputeBackend over the C ABI of
// libk3xb (see backend_b200.hpp for the method split).
#include "backend_b200.hpp"

#include <atomic>
#include <cmath>
#include <cstring>
#include <map>
#include <string>
#include <unordered_set>
#include <utility>
#include <vector>

namespace k3x {
namespace {

// The C ABI's status values are the values of k3x::ErrorCode
// (runtime/include/k3x/status.hpp:9-30), so a status converts by value.
static_assert(static_cast<int>(ErrorCode::ok) == K3XB_OK);
static_assert(static_cast<int>(ErrorCode::invalid_extent) == K3XB_INVALID_EXTENT);
static_assert(static_cast<int>(ErrorCode::invalid_mxfp4) == K3XB_INVALID_MXFP4);
static_assert(static_cast<int>(ErrorCode::invalid_state) == K3XB_INVALID_STATE);
static_assert(static_cast<int>(ErrorCode::backend_unavailable) == K3XB_BACKEND_UNAVAILABLE);
static_assert(static_cast<int>(ErrorCode::unsupported_architecture) == K3XB_UNSUPPORTED_ARCHITECTURE);

template <class T>
Result<T> unavailable(const char* what) {
    return Result<T>::failure(ErrorCode::backend_unavailable, what);
}

const std::uint8_t* bytes_of(std::span<const std::byte> s) {
    return reinterpret_cast<const std::uint8_t*>(s.data());
}

// One MXFP4 matrix of `rows` x `cols`, group 32 (the engine's block size).
bool valid_matrix(const Mxfp4WeightView& w, std::size_t rows, std::size_t cols) {
    return w.tensor_id != 0 && w.rows == rows && w.cols == cols && w.group_size == 32 && cols % 32 == 0 &&
           w.packed.size() == rows * cols / 2 && w.scales.size() == rows * cols / 32;
}

// Same dimensions for every expert, as the reference's grid checks
// (backend_cpu.cpp:215-234): gate/up [I][H], down [H][I].
bool valid_experts(std::span<const Mxfp4MlpView> experts, std::size_t* H, std::size_t* I) {
    if (experts.empty()) return false;
    *H = experts.front().gate.cols;
    *I = experts.front().gate.rows;
    for (const auto& e : experts)
        if (!valid_matrix(e.gate, *I, *H) || !valid_matrix(e.up, *I, *H) || !valid_matrix(e.down, *H, *I))
            return false;
    return *H > 0 && *I > 0;
}

bool valid_activation(float beta, std::optional<float> linear) {
    return std::isfinite(beta) && beta > 0.0F && (!linear || (std::isfinite(*linear) && *linear > 0.0F));
}

class B200Backend final : public ComputeBackend {
public:
    B200Backend(const BackendOptions& options, k3xb_ctx* ctx) : options_(options), ctx_(ctx) {
        if (ctx_ && options_.cuda_weights == CudaWeightMode::resident && options_.cuda_resident_bytes)
            k3xb_set_resident_capacity(ctx_, options_.cuda_resident_bytes);
    }
    ~B200Backend() override {
        if (ctx_) k3xb_destroy(ctx_);
    }
    B200Backend(const B200Backend&) = delete;
    B200Backend& operator=(const B200Backend&) = delete;

    BackendKind kind() const noexcept override { return BackendKind::cuda_custom; }
    const BackendOptions& options() const noexcept override { return options_; }
    std::string_view device_name() const noexcept override { return "NVIDIA B200 (libk3xb, sm_100a)"; }

    BackendRuntimeStats runtime_stats() const noexcept override {
        BackendRuntimeStats r{};
        k3xb_stats s{};
        if (ctx_ && k3xb_get_stats(ctx_, &s) == K3XB_OK) {
            r.weight_cache_hits += s.weight_cache_hits;
            r.weight_cache_misses += s.weight_cache_misses;
            r.weight_cache_bypasses += s.weight_cache_bypasses;
            r.resident_weight_bytes += s.resident_weight_bytes;
            r.peak_resident_weight_bytes += s.peak_resident_weight_bytes;
            r.weight_h2d_bytes += s.weight_h2d_bytes;
            r.activation_h2d_bytes += s.h2d_bytes - s.weight_h2d_bytes;
            r.device_to_host_bytes += s.d2h_bytes;
            r.scratch_bytes += s.scratch_bytes;
            r.peak_scratch_bytes += s.peak_scratch_bytes;
        }
        r.batched_expert_ffn_calls += grid_calls_;
        r.batched_expert_ffn_tokens += grid_tokens_;
        r.fused_moe_calls += moe_calls_;
        r.official_kda_calls += kda_calls_;
        return r;
    }

    BackendMemoryStats memory_stats() const noexcept override {
        BackendMemoryStats m{};
        k3xb_stats s{};
        if (ctx_ && k3xb_get_stats(ctx_, &s) == K3XB_OK) {
            m.current_device_bytes += s.resident_weight_bytes + s.scratch_bytes;
            m.peak_device_bytes += s.peak_resident_weight_bytes + s.peak_scratch_bytes;
        }
        return m;
    }

    // ---- f32 dense products (k3xb_dense_matvec_host, k3xb_dense_situ_mlp_host)
    // The CPU backend's checks (backend_cpu.cpp:368-377, :404-410,
    // invalid_extent) and its arithmetic bit for bit (one FP64 chain per row
    // in column order). A weight is kept resident by its tensor id; one
    // without an id (0) cannot be: backend_unavailable (backend.hpp:357-362).
    Result<std::vector<float>> dense_matvec(std::span<const float> input, DenseWeightView weight,
                                            std::uint32_t /*layer*/, ProfilePhase /*phase*/) override {
        if (!valid_dense(input, weight)) return Result<std::vector<float>>::failure(ErrorCode::invalid_extent);
        if (!weight.tensor_id || !weight.rows)
            return unavailable<std::vector<float>>("dense_matvec: a weight without a tensor id");
        ErrorCode st = ErrorCode::ok;
        const float* W = dense_resident(weight, &st);
        if (!W) return Result<std::vector<float>>::failure(st, last_error());
        std::vector<float> y(weight.rows);
        const int rc = k3xb_dense_matvec_host(ctx_, W, static_cast<std::uint32_t>(weight.rows),
                                              static_cast<std::uint32_t>(weight.cols), input.data(), y.data());
        if (rc != K3XB_OK) return Result<std::vector<float>>::failure(static_cast<ErrorCode>(rc), last_error());
        return Result<std::vector<float>>::success(std::move(y));
    }
    // single MXFP4 products (k3xb_mxfp4_matvec_host): mxfp4_matmul's checks
    // (ops.cpp:32-60, invalid_mxfp4) and arithmetic bit for bit
    Result<std::vector<float>> mxfp4_matvec(std::span<const float> input, Mxfp4WeightView weight,
                                            std::uint32_t /*layer*/, ProfilePhase /*phase*/) override {
        if (input.size() != weight.cols || !weight.rows || !weight.cols || !weight.group_size ||
            weight.cols % weight.group_size || weight.cols % 2 || weight.packed.size() != weight.rows * weight.cols / 2 ||
            weight.scales.size() != weight.rows * weight.cols / weight.group_size)
            return Result<std::vector<float>>::failure(ErrorCode::invalid_mxfp4);
        if (!weight.tensor_id || weight.group_size != 32)   // nothing to keep it resident by, or not group 32
            return unavailable<std::vector<float>>("mxfp4_matvec: no tensor id, or a group other than 32");
        k3xb_resident r{};
        const ErrorCode st = mxfp4_resident(weight, &r);
        if (st != ErrorCode::ok) return Result<std::vector<float>>::failure(st, last_error());
        std::vector<float> y(weight.rows);
        const int rc = k3xb_mxfp4_matvec_host(ctx_, static_cast<const std::uint8_t*>(r.primary),
                                              static_cast<const std::uint8_t*>(r.secondary),
                                              static_cast<std::uint32_t>(weight.rows),
                                              static_cast<std::uint32_t>(weight.cols), input.data(), y.data());
        if (rc != K3XB_OK) return Result<std::vector<float>>::failure(static_cast<ErrorCode>(rc), last_error());
        return Result<std::vector<float>>::success(std::move(y));
    }
    Result<std::vector<std::vector<float>>> dense_matvec_group(std::span<const float> input,
                                                               std::span<const DenseWeightView> weights,
                                                               std::uint32_t layer, ProfilePhase phase) override {
        using R = Result<std::vector<std::vector<float>>>;
        for (const auto& w : weights)   // backend_cpu.cpp:61-80: every weight checked first
            if (!valid_dense(input, w)) return R::failure(ErrorCode::invalid_extent);
        std::vector<std::vector<float>> out;
        out.reserve(weights.size());
        for (const auto& w : weights) {
            auto y = dense_matvec(input, w, layer, phase);
            if (!y) return R::failure(y.error(), y.message());
            out.push_back(std::move(y.value()));
        }
        return R::success(std::move(out));
    }
    Result<std::vector<std::vector<float>>> mxfp4_matvec_group(std::span<const float> input,
                                                               std::span<const Mxfp4WeightView> weights,
                                                               std::uint32_t layer, ProfilePhase phase) override {
        using R = Result<std::vector<std::vector<float>>>;
        std::vector<std::vector<float>> out;
        out.reserve(weights.size());
        for (const auto& w : weights) {
            auto y = mxfp4_matvec(input, w, layer, phase);
            if (!y) return R::failure(y.error(), y.message());
            out.push_back(std::move(y.value()));
        }
        return R::success(std::move(out));
    }
    Result<std::vector<float>> dense_situ_mlp(std::span<const float> input, DenseMlpView weights, float situ_beta,
                                              std::optional<float> situ_linear, std::uint32_t /*layer*/,
                                              ProfilePhase /*phase*/) override {
        const auto& g = weights.gate;
        if (!valid_dense(input, g) || !valid_dense(input, weights.up) || !g.rows || g.rows != weights.up.rows ||
            weights.down.cols != g.rows || weights.down.values.size() != weights.down.rows * weights.down.cols)
            return Result<std::vector<float>>::failure(ErrorCode::invalid_extent);
        if (!g.tensor_id || !weights.up.tensor_id || !weights.down.tensor_id || !weights.down.rows ||
            !valid_activation(situ_beta, situ_linear))
            return unavailable<std::vector<float>>("dense_situ_mlp: untracked weights or SiTU parameters");
        ErrorCode st = ErrorCode::ok;
        const float* G = dense_resident(g, &st);
        const float* U = G ? dense_resident(weights.up, &st) : nullptr;
        const float* D = U ? dense_resident(weights.down, &st) : nullptr;
        if (!D) return Result<std::vector<float>>::failure(st, last_error());
        std::vector<float> y(weights.down.rows);
        const int rc = k3xb_dense_situ_mlp_host(ctx_, G, U, D, static_cast<std::uint32_t>(g.rows),
                                                static_cast<std::uint32_t>(g.cols),
                                                static_cast<std::uint32_t>(weights.down.rows), input.data(),
                                                situ_beta, situ_linear ? *situ_linear : 0.0F, y.data());
        if (rc != K3XB_OK) return Result<std::vector<float>>::failure(static_cast<ErrorCode>(rc), last_error());
        return Result<std::vector<float>>::success(std::move(y));
    }

    // The resident layer (backend_cpu.cpp:305-339): f32 projections, the
    // experts' unrounded outputs mixed in float, with the CPU backend's checks
    // (:442-500, invalid_mxfp4); k3xb_resident_moe_layer_host runs it with
    // the CPU backend's products and norm bit for bit.
    Result<ResidentMoeLayerResult> resident_mxfp4_moe_layer(std::span<const float> input, ResidentMoeLayerView w,
                                                            std::span<const Mxfp4MlpView> experts,
                                                            std::span<const float> contributions, float epsilon,
                                                            float beta, std::optional<float> linear,
                                                            std::uint32_t /*layer*/, ProfilePhase /*phase*/) override {
        using R = Result<ResidentMoeLayerResult>;
        const auto& sh = w.shared;
        const bool mlp_ok = valid_dense(input, sh.gate) && valid_dense(input, sh.up) && sh.gate.rows &&
                            sh.gate.rows == sh.up.rows && sh.down.cols == sh.gate.rows && sh.down.rows &&
                            sh.down.values.size() == sh.down.rows * sh.down.cols;
        if (input.empty() || experts.empty() || experts.size() != contributions.size() || !std::isfinite(epsilon) ||
            epsilon <= 0.0F || !valid_activation(beta, linear) || !finite(input) || !finite(contributions) ||
            !finite(w.routed_down.values) || !finite(w.routed_norm.values) || !finite(w.routed_up.values) ||
            !finite(sh.gate.values) || !finite(sh.up.values) || !finite(sh.down.values) ||
            !valid_dense(input, w.routed_down) || !mlp_ok)
            return R::failure(ErrorCode::invalid_mxfp4);
        const std::size_t H = input.size(), D = w.routed_down.rows, Dout = experts.front().down.rows,
                          I = experts.front().gate.rows, S = sh.gate.rows;
        if (!D || !Dout || w.routed_norm.values.size() != Dout || w.routed_up.cols != Dout || !w.routed_up.rows ||
            w.routed_up.values.size() != w.routed_up.rows * w.routed_up.cols || w.routed_up.rows != H ||
            sh.down.rows != H)
            return R::failure(ErrorCode::invalid_mxfp4);
        std::unordered_set<std::uint64_t> tensors;
        const auto fresh = [&tensors](std::uint64_t id) { return id && tensors.insert(id).second; };
        if (!fresh(w.routed_down.tensor_id) || !fresh(w.routed_norm.tensor_id) || !fresh(w.routed_up.tensor_id) ||
            !fresh(sh.gate.tensor_id) || !fresh(sh.up.tensor_id) || !fresh(sh.down.tensor_id))
            return R::failure(ErrorCode::invalid_mxfp4);
        for (const auto& e : experts)
            if (!valid_matrix(e.gate, I, D) || !valid_matrix(e.up, I, D) || !valid_matrix(e.down, Dout, I) ||
                !fresh(e.gate.tensor_id) || !fresh(e.up.tensor_id) || !fresh(e.down.tensor_id))
                return R::failure(ErrorCode::invalid_mxfp4);
        if (Dout != D)   // a routed width other than the latent width: not this library's shape
            return unavailable<ResidentMoeLayerResult>("resident MoE layer shape is not on the B200 path");
        ErrorCode st = ErrorCode::ok;
        const auto f32 = [&](std::uint64_t id, std::span<const float> v, std::size_t rows, std::size_t cols) {
            return st == ErrorCode::ok ? static_cast<const float*>(
                                             resident(id, K3XB_WEIGHT_F32, rows, cols, v.data(), v.size() * 4, &st))
                                       : nullptr;
        };
        const float* rd = f32(w.routed_down.tensor_id, w.routed_down.values, D, H);
        const float* rn = f32(w.routed_norm.tensor_id, w.routed_norm.values, 1, D);
        const float* ru = f32(w.routed_up.tensor_id, w.routed_up.values, H, D);
        const float* sg = f32(sh.gate.tensor_id, sh.gate.values, S, H);
        const float* su = f32(sh.up.tensor_id, sh.up.values, S, H);
        const float* sd = f32(sh.down.tensor_id, sh.down.values, H, S);
        if (st != ErrorCode::ok) return R::failure(st, last_error());
        std::vector<k3xb_mxfp4_expert> dev(experts.size());
        for (std::size_t k = 0; k < experts.size(); ++k) {
            k3xb_resident g{}, u{}, d{};
            if ((st = mxfp4_resident(experts[k].gate, &g)) != ErrorCode::ok ||
                (st = mxfp4_resident(experts[k].up, &u)) != ErrorCode::ok ||
                (st = mxfp4_resident(experts[k].down, &d)) != ErrorCode::ok)
                return R::failure(st, last_error());
            dev[k] = {static_cast<const std::uint8_t*>(g.primary), static_cast<const std::uint8_t*>(g.secondary),
                      static_cast<const std::uint8_t*>(u.primary), static_cast<const std::uint8_t*>(u.secondary),
                      static_cast<const std::uint8_t*>(d.primary), static_cast<const std::uint8_t*>(d.secondary)};
        }
        ResidentMoeLayerResult out;
        out.output.resize(H);
        const int rc = k3xb_resident_moe_layer_host(
            ctx_, static_cast<std::uint32_t>(H), static_cast<std::uint32_t>(D), static_cast<std::uint32_t>(I),
            static_cast<std::uint32_t>(S), rd, rn, ru, sg, su, sd, dev.data(), static_cast<std::uint32_t>(dev.size()),
            contributions.data(), epsilon, beta, linear ? *linear : 0.0F, input.data(), out.output.data());
        if (rc != K3XB_OK) return R::failure(static_cast<ErrorCode>(rc), last_error());
        out.executed = true;
        ++moe_calls_;
        return R::success(std::move(out));
    }

    // ---- the official LatentMoE FFN of one position (k3xb_official_moe_ffn_host)
    // A direct call ends a prepared route still held (backend_cuda.cu:3724-3732).
    Result<OfficialMoeFfnResult> official_mxfp4_moe_ffn(std::span<const float> hidden, std::span<const float> prefix,
                                                        OfficialMoeFfnView w, std::span<const Mxfp4MlpView> experts,
                                                        std::span<const std::uint32_t> ids,
                                                        std::span<const float> contributions, float epsilon,
                                                        float beta, std::optional<float> linear,
                                                        std::uint32_t layer, ProfilePhase phase) override {
        end_prepared();
        if (hidden.empty() || hidden.size() != prefix.size() || !finite(hidden) || !finite(prefix))
            return Result<OfficialMoeFfnResult>::failure(ErrorCode::invalid_mxfp4);
        return official_ffn(hidden, prefix, false, w, experts, ids, contributions, epsilon, beta, linear, layer,
                            phase);
    }

    // ---- device route preparation (k3xb_prepare_moe_route_host) -----------
    // prepare_official_moe_route with the checks of backend_cuda.cu:3478-3570
    // (invalid_extent): the MoE input and its router logits computed on the
    // device. The prepared input and the prefix are kept (on the host, a few
    // KB) for the one official_mxfp4_moe_ffn_prepared that may consume them;
    // a new preparation or a direct FFN call ends the old one.
    Result<OfficialMoeRoutePrepareResult> prepare_official_moe_route(std::span<const float> prefix,
                                                                     std::span<const float> block,
                                                                     OfficialMoeRoutePrepareView w, float epsilon,
                                                                     std::uint32_t layer, ProfilePhase) override {
        const std::size_t H = prefix.size();
        if (!H || block.size() != H || !finite(prefix) || !finite(block))
            return Result<OfficialMoeRoutePrepareResult>::failure(ErrorCode::invalid_extent);
        return prepare_route(prefix, {}, block, w, epsilon, layer, 2);
    }

    // Consumes the prepared route of the same layer (backend_cuda.cu:3738-3748, :3779-3784).
    // Consumes the prepared route of the same layer (backend_cuda.cu:3738-3748, :3779-3784).
    Result<OfficialMoeFfnResult> official_mxfp4_moe_ffn_prepared(OfficialMoePreparedToken token, OfficialMoeFfnView w,
                                                                 std::span<const Mxfp4MlpView> experts,
                                                                 std::span<const std::uint32_t> ids,
                                                                 std::span<const float> contributions, float epsilon,
                                                                 float beta, std::optional<float> linear,
                                                                 std::uint32_t layer, ProfilePhase phase) override {
        if (!prepared_.active || token.owner != owner_ || token.generation != prepared_.generation ||
            prepared_.layer != layer)
            return Result<OfficialMoeFfnResult>::failure(ErrorCode::invalid_mxfp4);
        const std::vector<float> hidden = prepared_.hidden, prefix = prepared_.prefix;
        return official_ffn(hidden, prefix, true, w, experts, ids, contributions, epsilon, beta, linear, layer,
                            phase);
    }

    Result<bool> discard_official_moe_prepared(OfficialMoePreparedToken token) override {
        if (!prepared_.active || token.owner != owner_ || token.generation != prepared_.generation)
            return Result<bool>::failure(ErrorCode::invalid_state);
        end_prepared();
        return Result<bool>::success(true);
    }

    // ---- a layer's front and tail with its hidden rows held between them
    // (official_layer_front / _tail / discard_official_layer_hidden,
    // backend_cuda.cu:3161-3476: the device_closure mode of
    // official_two_layer_cuda). Two hidden slots (free, live, prepared) with
    // the reference's token rules; the rows a slot holds (hidden input and
    // block source, a few KB) stay in the adapter between calls, the compute
    // runs on the device.
    Result<OfficialLayerFrontResult> official_layer_front(std::span<const float> host_hidden,
                                                          std::span<const float> host_block,
                                                          OfficialLayerHiddenToken in, OfficialLayerFrontWeights w,
                                                          OfficialKdaCudaStateView state, OfficialKdaCudaConfig config,
                                                          std::uint32_t layer, ProfilePhase phase,
                                                          OfficialKdaStateControl control) override {
        using R = Result<OfficialLayerFrontResult>;
        using Mode = OfficialKdaStateMode;
        const std::size_t H = config.hidden_size;
        const bool host_input = !host_hidden.empty() || !host_block.empty();
        const bool token_input = in.owner || in.generation || in.producing_layer || in.width || in.slot;
        if (layer < 1 || layer > 2 || !H || H > SIZE_MAX / 16 || host_input == token_input ||
            (control.mode != Mode::device_seed && control.mode != Mode::device_continue &&
             control.mode != Mode::device_publish) ||
            (host_input && (layer != 1 || host_hidden.size() != H || host_block.size() != H || !finite(host_hidden) ||
                            !finite(host_block))) ||
            !w.self_residual_norm.tensor_id || w.self_residual_norm.values.size() != H ||
            !w.input_norm.tensor_id || w.input_norm.values.size() != H)
            return R::failure(ErrorCode::invalid_extent);
        if (prepared_.active) return R::failure(ErrorCode::invalid_state);
        std::uint32_t slot = 2;
        if (host_input) {
            for (const HiddenSlot& s : hidden_slots_)
                if (s.state != HiddenSlot::kFree) return R::failure(ErrorCode::invalid_state);
            slot = 0;
        } else {
            if (in.owner != owner_ || !in.generation || in.slot >= 2 || in.producing_layer + 1 != layer ||
                in.width != H)
                return R::failure(ErrorCode::invalid_state);
            slot = in.slot;
            const HiddenSlot& s = hidden_slots_[slot];
            if (s.state != HiddenSlot::kLive || s.generation != in.generation ||
                s.producing_layer != in.producing_layer || s.width != in.width ||
                hidden_slots_[1 - slot].state != HiddenSlot::kFree)
                return R::failure(ErrorCode::invalid_state);
        }
        // the self-attention residual's weights: distinct ids, well-formed bf16 (backend_cuda.cu:3271-3318)
        const Bf16WeightView self_views[] = {{w.self_residual_norm.values, 1, H, w.self_residual_norm.tensor_id},
                                             w.self_residual_proj,
                                             {w.input_norm.values, 1, H, w.input_norm.tensor_id}};
        std::unordered_set<std::uint64_t> tensors;
        for (const auto& v : self_views)
            if (!tensors.insert(v.tensor_id).second || !v.tensor_id || v.rows != 1 || v.cols != H ||
                v.values.size() != H || !scan_bf16(v.tensor_id, v.values))
                return R::failure(ErrorCode::invalid_extent);
        ErrorCode st = ErrorCode::ok;
        const std::uint16_t* dev[3];
        for (int i = 0; i < 3; ++i)
            if (!(dev[i] = static_cast<const std::uint16_t*>(resident(self_views[i].tensor_id, K3XB_WEIGHT_BF16, 1, H,
                                                                      self_views[i].values.data(), H * 2, &st))))
                return R::failure(st, last_error());
        HiddenSlot& hs = hidden_slots_[slot];
        if (host_input) {
            hs.hidden.assign(host_hidden.begin(), host_hidden.end());
            hs.block.assign(host_block.begin(), host_block.end());
        }
        hs.state = HiddenSlot::kPrepared;
        // the KDA input: attention residual over (hidden, block), input norm (official_layer.cpp:159-172)
        std::vector<float> normalized(H);
        const int rc = k3xb_prepare_moe_route_host(ctx_, hs.hidden.data(), nullptr, hs.block.data(),
                                                   static_cast<std::uint32_t>(H), dev[0], dev[1], dev[2],
                                                   config.rms_norm_epsilon, nullptr, 0, nullptr, normalized.data(),
                                                   nullptr);
        if (rc != K3XB_OK) {
            hs.state = HiddenSlot::kFree;
            return R::failure(static_cast<ErrorCode>(rc), last_error());
        }
        auto kda = official_kda(normalized, w.kda, state, config, layer, phase, control);
        if (!kda) {
            hs.state = HiddenSlot::kFree;
            return R::failure(kda.error(), kda.message());
        }
        // the prefix round_bf16(round_bf16(hidden) + kda) and its MoE route (official_layer.cpp:190-205)
        auto route = prepare_route(hs.hidden, kda.value().output, hs.block, w.moe, config.rms_norm_epsilon, layer,
                                   slot);
        if (!route) {
            if (kda.value().device_state.owner) (void)discard_official_kda_device_state(kda.value().device_state);
            hs.state = HiddenSlot::kFree;
            return R::failure(route.error(), route.message());
        }
        OfficialLayerFrontResult out;
        out.executed = true;
        out.kda = std::move(kda.value());
        out.kda.output.clear();   // the KDA output stays with the layer (the reference keeps it on the device)
        out.route = std::move(route.value());
        return R::success(std::move(out));
    }

    Result<OfficialLayerTailResult> official_layer_tail(OfficialMoePreparedToken prepared, OfficialMoeFfnView w,
                                                        std::span<const Mxfp4MlpView> experts,
                                                        std::span<const std::uint32_t> ids,
                                                        std::span<const float> contributions, float epsilon,
                                                        float beta, std::optional<float> linear, std::uint32_t layer,
                                                        ProfilePhase phase, bool retain_hidden) override {
        using R = Result<OfficialLayerTailResult>;
        if (!prepared_.active || prepared_.hidden_slot >= 2 || prepared.owner != owner_ ||
            prepared.generation != prepared_.generation || prepared_.layer != layer)
            return R::failure(ErrorCode::invalid_state);
        const std::uint32_t source = prepared_.hidden_slot, target = 1 - source;
        if (hidden_slots_[source].state != HiddenSlot::kPrepared ||
            (retain_hidden && hidden_slots_[target].state != HiddenSlot::kFree))
            return R::failure(ErrorCode::invalid_state);
        auto moe = official_mxfp4_moe_ffn_prepared(prepared, w, experts, ids, contributions, epsilon, beta, linear,
                                                   layer, phase);
        if (!moe) {
            if (prepared_.active && prepared.generation == prepared_.generation) {
                end_prepared();
            } else {
                hidden_slots_[source].state = HiddenSlot::kFree;
                prepared_.hidden_slot = 2;
            }
            return R::failure(moe.error(), moe.message());
        }
        hidden_slots_[source].state = HiddenSlot::kFree;
        OfficialLayerTailResult out;
        out.executed = true;
        out.selected_expert_ids = std::move(moe.value().selected_expert_ids);
        if (retain_hidden) {   // the output is the next layer's hidden input; the block source carries over
            if (!++hidden_generation_) ++hidden_generation_;
            HiddenSlot& t = hidden_slots_[target];
            t.hidden = std::move(moe.value().output);
            t.block = hidden_slots_[source].block;
            t.generation = hidden_generation_;
            t.producing_layer = layer;
            t.width = t.hidden.size();
            t.state = HiddenSlot::kLive;
            out.hidden = {owner_, hidden_generation_, layer, t.width, target};
        } else {
            out.output = std::move(moe.value().output);
        }
        prepared_.hidden_slot = 2;
        return R::success(std::move(out));
    }

    Result<bool> discard_official_layer_hidden(OfficialLayerHiddenToken token) override {
        if (token.owner != owner_ || token.slot >= 2) return Result<bool>::failure(ErrorCode::invalid_state);
        HiddenSlot& s = hidden_slots_[token.slot];
        if (s.state != HiddenSlot::kLive || s.generation != token.generation ||
            s.producing_layer != token.producing_layer || s.width != token.width)
            return Result<bool>::failure(ErrorCode::invalid_state);
        s.state = HiddenSlot::kFree;
        return Result<bool>::success(true);
    }

private:
    // A prepared route ends (a discard, a new preparation, a direct FFN
    // call); the hidden slot it held is freed (backend_cuda.cu:3594-3603).
    void end_prepared() {
        if (prepared_.active && prepared_.hidden_slot < 2) hidden_slots_[prepared_.hidden_slot].state = HiddenSlot::kFree;
        prepared_.hidden_slot = 2;
        prepared_.active = false;
    }

    // bf16 words with an all-ones exponent are refused; each tensor id is scanned at its first use
    bool scan_bf16(std::uint64_t id, std::span<const std::uint16_t> values) {
        if (scanned_.count(id)) return true;
        for (const std::uint16_t word : values)
            if ((word & 0x7f80U) == 0x7f80U) return false;
        scanned_.insert(id);
        return true;
    }

    // prepare_official_moe_route's checks (backend_cuda.cu:3478-3570,
    // invalid_extent) and work: from the prefix `a`, or with `delta` from the
    // prefix round_bf16(round_bf16(a) + delta); `hidden_slot` is the layer
    // hidden slot the route holds (2: none).
    Result<OfficialMoeRoutePrepareResult> prepare_route(std::span<const float> a, std::span<const float> delta,
                                                        std::span<const float> block,
                                                        const OfficialMoeRoutePrepareView& w, float epsilon,
                                                        std::uint32_t layer, std::uint32_t hidden_slot) {
        using R = Result<OfficialMoeRoutePrepareResult>;
        const std::size_t H = a.size();
        const auto valid_bf16 = [](const Bf16WeightView& v, std::size_t rows, std::size_t cols) {
            return v.tensor_id && v.rows == rows && v.cols == cols && rows && cols && rows <= SIZE_MAX / cols &&
                   v.values.size() == rows * cols;
        };
        if ((!delta.empty() && delta.size() != H) || !std::isfinite(epsilon) ||
            epsilon <= 0.0F || !w.residual_norm.tensor_id || w.residual_norm.values.size() != H ||

            !valid_bf16(w.residual_proj, 1, H) || !w.post_norm.tensor_id || w.post_norm.values.size() != H ||
            !valid_bf16(w.router, w.router.rows, H))
            return R::failure(ErrorCode::invalid_extent);
        std::unordered_set<std::uint64_t> tensors;
        for (const std::uint64_t id : {w.residual_norm.tensor_id, w.residual_proj.tensor_id, w.post_norm.tensor_id,
                                       w.router.tensor_id})
            if (!tensors.insert(id).second) return R::failure(ErrorCode::invalid_extent);
        if (!scan_bf16(w.residual_norm.tensor_id, w.residual_norm.values) ||
            !scan_bf16(w.residual_proj.tensor_id, w.residual_proj.values) ||
            !scan_bf16(w.post_norm.tensor_id, w.post_norm.values) || !scan_bf16(w.router.tensor_id, w.router.values))
            return R::failure(ErrorCode::invalid_extent);
        ErrorCode st = ErrorCode::ok;
        const auto bf16 = [&](std::uint64_t id, std::span<const std::uint16_t> v, std::size_t rows, std::size_t cols) {
            return static_cast<const std::uint16_t*>(
                resident(id, K3XB_WEIGHT_BF16, rows, cols, v.data(), v.size() * 2, &st));
        };
        const std::size_t E = w.router.rows;
        const std::uint16_t* rnorm = bf16(w.residual_norm.tensor_id, w.residual_norm.values, 1, H);
        const std::uint16_t* rproj = bf16(w.residual_proj.tensor_id, w.residual_proj.values, 1, H);
        const std::uint16_t* post = bf16(w.post_norm.tensor_id, w.post_norm.values, 1, H);
        const std::uint16_t* router = bf16(w.router.tensor_id, w.router.values, E, H);
        if (st != ErrorCode::ok) return R::failure(st, last_error());
        end_prepared();
        std::vector<float> hidden(H), prefix(delta.empty() ? 0 : H);
        OfficialMoeRoutePrepareResult out;
        out.router_logits.resize(E);
        const int rc = k3xb_prepare_moe_route_host(ctx_, a.data(), delta.empty() ? nullptr : delta.data(), block.data(),
                                                   static_cast<std::uint32_t>(H), rnorm, rproj, post, epsilon, router,
                                                   static_cast<std::uint32_t>(E), prefix.empty() ? nullptr : prefix.data(),
                                                   hidden.data(), out.router_logits.data());
        if (rc != K3XB_OK) return R::failure(static_cast<ErrorCode>(rc), last_error());
        if (!finite(out.router_logits)) return R::failure(ErrorCode::backend_unavailable, "non-finite router logits");
        if (!++prepared_.generation) ++prepared_.generation;
        prepared_.layer = layer;
        if (delta.empty()) prepared_.prefix.assign(a.begin(), a.end());
        else prepared_.prefix = std::move(prefix);
        prepared_.hidden = std::move(hidden);
        prepared_.hidden_slot = hidden_slot;
        prepared_.active = true;
        out.executed = true;
        out.prepared = {owner_, prepared_.generation};
        return R::success(std::move(out));
    }


    // backend_cpu.cpp:368-377
    static bool valid_dense(std::span<const float> input, const DenseWeightView& w) {
        if (input.size() != w.cols || w.rows > w.values.size() || (w.cols != 0 && w.rows > w.values.size() / w.cols))
            return false;
        return w.values.size() == w.rows * w.cols;
    }

    // One MXFP4 matrix resident by its tensor id (its scales checked for 0xFF at admission).
    ErrorCode mxfp4_resident(const Mxfp4WeightView& w, k3xb_resident* r) {
        const int rc = k3xb_acquire_weight(ctx_, w.tensor_id, K3XB_WEIGHT_MXFP4, w.rows, w.cols, w.group_size,
                                           w.packed.data(), w.packed.size(), w.scales.data(), w.scales.size(), r);
        if (rc != K3XB_OK) return static_cast<ErrorCode>(rc);
        return r->disposition == K3XB_RESIDENT_BYPASS ? ErrorCode::backend_unavailable : ErrorCode::ok;
    }

    const float* dense_resident(const DenseWeightView& w, ErrorCode* st) {
        return static_cast<const float*>(
            resident(w.tensor_id, K3XB_WEIGHT_F32, w.rows, w.cols, w.values.data(), w.values.size() * 4, st));
    }

    static bool finite(std::span<const float> v) {
        for (const float x : v)
            if (!std::isfinite(x)) return false;
        return true;
    }

    // Checks of backend_cuda.cu:3770-3875 (same failures, invalid_mxfp4);
    // then each bf16 projection resident by tensor id, each routed expert a
    // resident stack of one, and the tail on the device. `prepared`: the
    // inputs are a prepared route's, consumed once the checks pass.
    Result<OfficialMoeFfnResult> official_ffn(std::span<const float> hidden, std::span<const float> prefix,
                                              bool prepared, OfficialMoeFfnView w,
                                              std::span<const Mxfp4MlpView> experts,
                                              std::span<const std::uint32_t> ids,
                                              std::span<const float> contributions, float epsilon, float beta,
                                              std::optional<float> linear, std::uint32_t /*layer*/, ProfilePhase /*phase*/) {
        using R = Result<OfficialMoeFfnResult>;
        const auto valid_bf16 = [](const Bf16WeightView& v) {
            return v.tensor_id && v.rows && v.cols && v.rows <= SIZE_MAX / v.cols && v.values.size() == v.rows * v.cols;
        };
        if (experts.empty() || experts.size() > 65535 ||
            experts.size() != ids.size() || experts.size() != contributions.size() ||
            !finite(contributions) || !std::isfinite(epsilon) || epsilon <= 0.0F ||
            !valid_activation(beta, linear) || !valid_bf16(w.routed_down) || !valid_bf16(w.routed_up) ||
            !valid_bf16(w.shared.gate) || !valid_bf16(w.shared.up) || !valid_bf16(w.shared.down) ||
            !w.routed_norm.tensor_id || w.routed_norm.values.empty())
            return R::failure(ErrorCode::invalid_mxfp4);
        const std::size_t H = hidden.size(), D = w.routed_down.rows, Dout = experts.front().down.rows,
                          I = experts.front().gate.rows, Is = w.shared.gate.rows;
        if (w.routed_down.cols != H || w.routed_norm.values.size() != Dout || w.routed_up.rows != H ||
            w.routed_up.cols != Dout || w.shared.gate.cols != H || w.shared.up.rows != Is || w.shared.up.cols != H ||
            w.shared.down.rows != H || w.shared.down.cols != Is)
            return R::failure(ErrorCode::invalid_mxfp4);
        std::unordered_set<std::uint64_t> tensors;
        const auto fresh = [&tensors](std::uint64_t id) { return id && tensors.insert(id).second; };
        if (!fresh(w.routed_down.tensor_id) || !fresh(w.routed_norm.tensor_id) || !fresh(w.routed_up.tensor_id) ||
            !fresh(w.shared.gate.tensor_id) || !fresh(w.shared.up.tensor_id) || !fresh(w.shared.down.tensor_id))
            return R::failure(ErrorCode::invalid_mxfp4);
        std::unordered_set<std::uint32_t> selected;
        double sum = 0.0;
        for (std::size_t k = 0; k < experts.size(); ++k) {
            const auto& e = experts[k];
            if (!selected.insert(ids[k]).second || contributions[k] <= 0.0F || !valid_matrix(e.gate, I, D) ||
                !valid_matrix(e.up, I, D) || !valid_matrix(e.down, Dout, I) || !fresh(e.gate.tensor_id) ||
                !fresh(e.up.tensor_id) || !fresh(e.down.tensor_id))
                return R::failure(ErrorCode::invalid_mxfp4);
            sum += contributions[k];
        }
        if (std::abs(sum - 1.0) > 1.0e-5) return R::failure(ErrorCode::invalid_mxfp4);
        if (prepared) prepared_.active = false;   // consumed
        // this library's shapes: expert output width = latent width, bf16
        // linears over multiples of 8, MXFP4 groups of 32, at most 64 slots
        if (Dout != D || H % 8 || D % 32 || I % 32 || experts.size() > 64)
            return unavailable<OfficialMoeFfnResult>("official MoE FFN shape is not on the B200 path");
        ErrorCode st = ErrorCode::ok;
        const auto bf16 = [&](std::uint64_t id, std::span<const std::uint16_t> v, std::size_t rows,
                              std::size_t cols) {
            return static_cast<const std::uint16_t*>(
                resident(id, K3XB_WEIGHT_BF16, rows, cols, v.data(), v.size() * 2, &st));
        };
        k3xb_moe_layer tail{};
        tail.hidden = static_cast<std::uint32_t>(H);
        tail.latent = static_cast<std::uint32_t>(D);
        tail.shared_inter = static_cast<std::uint32_t>(Is);
        tail.routed_down = bf16(w.routed_down.tensor_id, w.routed_down.values, D, H);
        tail.routed_norm = bf16(w.routed_norm.tensor_id, w.routed_norm.values, 1, D);
        tail.routed_up = bf16(w.routed_up.tensor_id, w.routed_up.values, H, D);
        tail.shared_gate = bf16(w.shared.gate.tensor_id, w.shared.gate.values, Is, H);
        tail.shared_up = bf16(w.shared.up.tensor_id, w.shared.up.values, Is, H);
        tail.shared_down = bf16(w.shared.down.tensor_id, w.shared.down.values, H, Is);
        if (st != ErrorCode::ok) return R::failure(st, last_error());
        tail.activation = K3XB_ACT_SITU;
        tail.situ_beta = beta;
        tail.situ_linear_beta = linear ? *linear : 0.0F;
        tail.latent_eps = epsilon;
        std::vector<k3xb_moe_layer> slots(experts.size());
        for (std::size_t k = 0; k < experts.size(); ++k)
            if ((st = expert_of(experts[k], D, I, &slots[k])) != ErrorCode::ok) return R::failure(st, last_error());
        tail.engine = slots.front().engine;
        std::vector<float> out(H);
        const int rc = k3xb_official_moe_ffn_host(ctx_, &tail, slots.data(), static_cast<std::uint32_t>(slots.size()),
                                                  contributions.data(), hidden.data(), prefix.data(), out.data());
        if (rc != K3XB_OK) return R::failure(static_cast<ErrorCode>(rc), last_error());
        ++moe_calls_;
        return R::success({true, std::move(out), {ids.begin(), ids.end()}});
    }

public:

    // ---- expert FFNs on tcgen05 (k3xb_expert_grid_host) --------------------
    Result<std::vector<std::vector<float>>> mxfp4_situ_mlp_group(std::span<const float> input,
                                                                 std::span<const Mxfp4MlpView> experts,
                                                                 float situ_beta, std::optional<float> situ_linear,
                                                                 std::uint32_t, ProfilePhase) override {
        std::size_t H = 0, I = 0;
        if (!valid_experts(experts, &H, &I) || input.size() != H || !valid_activation(situ_beta, situ_linear))
            return Result<std::vector<std::vector<float>>>::failure(ErrorCode::invalid_mxfp4);
        std::vector<std::vector<float>> out;
        out.reserve(experts.size());
        for (const auto& e : experts) {
            auto y = run_expert(e, H, I, input.data(), 1, situ_beta, situ_linear);
            if (!y) return Result<std::vector<std::vector<float>>>::failure(y.error(), y.message());
            out.push_back(std::move(y.value()));
        }
        return Result<std::vector<std::vector<float>>>::success(std::move(out));
    }

    Result<std::vector<std::vector<float>>> mxfp4_situ_mlp_batch(std::span<const float> inputs,
                                                                 std::size_t batch_size, Mxfp4MlpView expert,
                                                                 float situ_beta, std::optional<float> situ_linear,
                                                                 std::uint32_t, ProfilePhase) override {
        std::size_t H = 0, I = 0;
        if (!batch_size || !valid_experts(std::span<const Mxfp4MlpView>(&expert, 1), &H, &I) ||
            inputs.size() != batch_size * H || !valid_activation(situ_beta, situ_linear))
            return Result<std::vector<std::vector<float>>>::failure(ErrorCode::invalid_mxfp4);
        auto y = run_expert(expert, H, I, inputs.data(), batch_size, situ_beta, situ_linear);
        if (!y) return Result<std::vector<std::vector<float>>>::failure(y.error(), y.message());
        std::vector<std::vector<float>> out(batch_size);
        for (std::size_t t = 0; t < batch_size; ++t)
            out[t].assign(y.value().begin() + static_cast<std::ptrdiff_t>(t * H),
                          y.value().begin() + static_cast<std::ptrdiff_t>((t + 1) * H));
        return Result<std::vector<std::vector<float>>>::success(std::move(out));
    }

    // outputs[expert] = [token][H] (backend_cpu.cpp:241-262)
    Result<std::vector<std::vector<float>>> mxfp4_situ_mlp_grid(std::span<const float> inputs,
                                                                std::size_t token_count,
                                                                std::span<const Mxfp4MlpView> experts,
                                                                float situ_beta, std::optional<float> situ_linear,
                                                                std::uint32_t, ProfilePhase) override {
        std::size_t H = 0, I = 0;
        if (!token_count || !valid_experts(experts, &H, &I) || inputs.size() != token_count * H ||
            !valid_activation(situ_beta, situ_linear) || !distinct_ids(experts))
            return Result<std::vector<std::vector<float>>>::failure(ErrorCode::invalid_mxfp4);
        std::vector<std::vector<float>> out;
        out.reserve(experts.size());
        for (const auto& e : experts) {
            auto y = run_expert(e, H, I, inputs.data(), token_count, situ_beta, situ_linear);
            if (!y) return Result<std::vector<std::vector<float>>>::failure(y.error(), y.message());
            out.push_back(std::move(y.value()));
        }
        return Result<std::vector<std::vector<float>>>::success(std::move(out));
    }

    // mixed = sum_slot contribution * y_slot in float, slot order
    // (backend_cpu.cpp:266-303; official_moe.cpp:313-322).
    Result<std::vector<float>> mxfp4_situ_moe(std::span<const float> input, std::span<const Mxfp4MlpView> experts,
                                              std::span<const float> contributions, float situ_beta,
                                              std::optional<float> situ_linear, std::uint32_t layer,
                                              ProfilePhase phase) override {
        if (experts.empty() || experts.size() != contributions.size())
            return Result<std::vector<float>>::failure(ErrorCode::invalid_mxfp4);
        for (const float c : contributions)
            if (!std::isfinite(c)) return Result<std::vector<float>>::failure(ErrorCode::invalid_mxfp4);
        auto ys = mxfp4_situ_mlp_group(input, experts, situ_beta, situ_linear, layer, phase);
        if (!ys) return Result<std::vector<float>>::failure(ys.error(), ys.message());
        ++moe_calls_;
        return Result<std::vector<float>>::success(mix(ys.value(), contributions));
    }

    // Prefetch = upload the experts now (the resident stacks), keep the list
    // for the _prepared call that follows.
    Result<Mxfp4PrefetchToken> prefetch_mxfp4_situ_mlp_group(std::span<const Mxfp4MlpView> experts,
                                                             std::uint64_t use_sequence, std::uint32_t,
                                                             ProfilePhase) override {
        std::size_t H = 0, I = 0;
        if (!valid_experts(experts, &H, &I)) return Result<Mxfp4PrefetchToken>::failure(ErrorCode::invalid_mxfp4);
        for (const auto& e : experts) {
            k3xb_moe_layer L{};
            if (auto st = stack_of(e, H, I, &L); st != ErrorCode::ok) return Result<Mxfp4PrefetchToken>::failure(st);
        }
        const std::uint64_t id = ++next_token_;
        prefetched_[id] = std::vector<Mxfp4MlpView>(experts.begin(), experts.end());
        return Result<Mxfp4PrefetchToken>::success({id, use_sequence});
    }

    Result<std::vector<std::vector<float>>> mxfp4_situ_mlp_group_prepared(std::span<const float> input,
                                                                          Mxfp4PrefetchToken token, float beta,
                                                                          std::optional<float> linear,
                                                                          std::uint32_t layer,
                                                                          ProfilePhase phase) override {
        auto it = prefetched_.find(token.value);
        if (it == prefetched_.end())
            return Result<std::vector<std::vector<float>>>::failure(ErrorCode::invalid_state, "unknown prefetch token");
        const std::vector<Mxfp4MlpView> experts = std::move(it->second);
        prefetched_.erase(it);
        return mxfp4_situ_mlp_group(input, experts, beta, linear, layer, phase);
    }

    Result<std::vector<float>> mxfp4_situ_moe_prepared(std::span<const float> input, Mxfp4PrefetchToken token,
                                                       std::span<const float> contributions, float beta,
                                                       std::optional<float> linear, std::uint32_t layer,
                                                       ProfilePhase phase) override {
        auto it = prefetched_.find(token.value);
        if (it == prefetched_.end())
            return Result<std::vector<float>>::failure(ErrorCode::invalid_state, "unknown prefetch token");
        const std::vector<Mxfp4MlpView> experts = std::move(it->second);
        prefetched_.erase(it);
        return mxfp4_situ_moe(input, experts, contributions, beta, linear, layer, phase);
    }

    // ---- KDA block (k3xb_kda_block_host) -----------------------------------
    Result<OfficialKdaCudaResult> official_kda(std::span<const float> input, OfficialKdaCudaView w,
                                               OfficialKdaCudaStateView state, OfficialKdaCudaConfig config,
                                               std::uint32_t layer, ProfilePhase phase,
                                               OfficialKdaStateControl control) override {
        // the state modes (backend_cuda.cu:2564-2625, :2691-2702): the host
        // round trip brings the state and takes it back; device_seed brings it
        // and the device keeps the new one; device_continue runs from the kept
        // state and keeps the new one; device_publish runs from it and hands
        // the new one back. Layers 1 and 2 have a slot each.
        (void)phase;
        using Mode = OfficialKdaStateMode;
        const Mode mode = control.mode;
        if (mode != Mode::host_roundtrip && mode != Mode::device_seed && mode != Mode::device_continue &&
            mode != Mode::device_publish)
            return Result<OfficialKdaCudaResult>::failure(ErrorCode::invalid_extent);
        const bool host_in = mode == Mode::host_roundtrip || mode == Mode::device_seed;
        const bool from_device = mode == Mode::device_continue || mode == Mode::device_publish;
        const bool publish = mode == Mode::host_roundtrip || mode == Mode::device_publish;
        const bool retain = mode == Mode::device_seed || mode == Mode::device_continue;
        const std::size_t H = config.hidden_size, h = config.heads, d = config.head_dim, cw = config.conv_width;
        const std::size_t P = h * d;
        if (!H || !h || !d || cw < 2 || !std::isfinite(config.rms_norm_epsilon) || config.rms_norm_epsilon <= 0.0F ||
            !std::isfinite(config.gate_lower_bound) || config.gate_lower_bound >= 0.0F || input.empty() ||
            input.size() % H ||
            (host_in && (state.conv_q.size() != (cw - 1) * P || state.conv_k.size() != (cw - 1) * P ||
                         state.conv_v.size() != (cw - 1) * P || state.recurrent_v_first.size() != h * d * d)) ||
            (!host_in && (!state.conv_q.empty() || !state.conv_k.empty() || !state.conv_v.empty() ||
                          !state.recurrent_v_first.empty())) ||
            (host_in && (control.token.owner || control.token.generation)))
            return Result<OfficialKdaCudaResult>::failure(ErrorCode::invalid_extent);
        KdaSlot* slot = layer == 1 ? &kda_slots_[0] : layer == 2 ? &kda_slots_[1] : nullptr;
        if (mode != Mode::host_roundtrip && !slot) return Result<OfficialKdaCudaResult>::failure(ErrorCode::invalid_state);
        if ((mode == Mode::device_seed && slot->active) ||
            (from_device && (!slot->active || control.token.owner != owner_ ||
                             control.token.generation != slot->generation || !same_config(slot->config, config))))
            return Result<OfficialKdaCudaResult>::failure(ErrorCode::invalid_state);
        k3xb_kda_layer K{};
        K.heads = static_cast<std::uint32_t>(h);
        K.head_dim = static_cast<std::uint32_t>(d);
        K.conv_width = static_cast<std::uint32_t>(cw);
        K.eps = config.rms_norm_epsilon;
        K.gate_lower_bound = config.gate_lower_bound;
        ErrorCode st = ErrorCode::ok;
        const auto bf16 = [&](const Bf16WeightView& v, std::size_t rows, std::size_t cols) -> const std::uint16_t* {
            if (st != ErrorCode::ok) return nullptr;
            if (v.rows != rows || v.cols != cols || v.values.size() != rows * cols) {
                st = ErrorCode::invalid_extent;
                return nullptr;
            }
            return static_cast<const std::uint16_t*>(resident(v.tensor_id, K3XB_WEIGHT_BF16, rows, cols,
                                                              v.values.data(), v.values.size() * 2, &st));
        };
        const auto f32 = [&](std::uint64_t id, std::span<const float> v, std::size_t rows,
                             std::size_t cols) -> const float* {
            if (st != ErrorCode::ok) return nullptr;
            if (v.size() != rows * cols) {
                st = ErrorCode::invalid_extent;
                return nullptr;
            }
            return static_cast<const float*>(resident(id, K3XB_WEIGHT_F32, rows, cols, v.data(), v.size() * 4, &st));
        };
        K.q_proj = bf16(w.q_proj, P, H);
        K.k_proj = bf16(w.k_proj, P, H);
        K.v_proj = bf16(w.v_proj, P, H);
        K.q_conv = f32(w.q_conv.tensor_id, w.q_conv.values, P, cw);
        K.k_conv = f32(w.k_conv.tensor_id, w.k_conv.values, P, cw);
        K.v_conv = f32(w.v_conv.tensor_id, w.v_conv.values, P, cw);
        K.f_a_proj = bf16(w.f_a_proj, d, H);
        K.f_b_proj = bf16(w.f_b_proj, P, d);
        K.a_log = f32(w.a_log.tensor_id, w.a_log.values, 1, d);
        K.dt_bias = f32(w.dt_bias.tensor_id, w.dt_bias.values, 1, P);
        K.b_proj = bf16(w.b_proj, h, H);
        K.g_proj = bf16(w.g_proj, P, H);
        K.o_norm = f32(w.o_norm.tensor_id, w.o_norm.values, 1, d);
        K.o_proj = bf16(w.o_proj, H, P);
        if (st != ErrorCode::ok) return Result<OfficialKdaCudaResult>::failure(st, last_error());

        // a host round trip ends the layer's kept state; a continuation ends
        // the token it came with (a new one follows when the state is kept)
        if (slot && (mode == Mode::host_roundtrip || from_device)) slot->active = false;

        const std::size_t hist = (cw - 1) * P;
        std::vector<std::uint16_t> conv(host_in || publish ? 3 * hist : 0);
        if (host_in) {
            std::memcpy(conv.data(), state.conv_q.data(), hist * 2);
            std::memcpy(conv.data() + hist, state.conv_k.data(), hist * 2);
            std::memcpy(conv.data() + 2 * hist, state.conv_v.data(), hist * 2);
        }
        OfficialKdaCudaResult r;
        if (host_in) r.recurrent_v_first.assign(state.recurrent_v_first.begin(), state.recurrent_v_first.end());
        else if (publish) r.recurrent_v_first.resize(h * d * d);
        r.output.resize(input.size());
        const auto T = static_cast<std::uint32_t>(input.size() / H);
        int rc;
        if (mode == Mode::host_roundtrip) {
            rc = k3xb_kda_block_host(ctx_, &K, static_cast<std::uint32_t>(H), input.data(), T, conv.data(),
                                     r.recurrent_v_first.data(), r.output.data());
        } else {
            const std::int32_t held = mode == Mode::device_seed       ? K3XB_KDA_SEED
                                      : mode == Mode::device_continue ? K3XB_KDA_CONTINUE
                                                                      : K3XB_KDA_PUBLISH;
            rc = k3xb_kda_block_held(ctx_, &K, static_cast<std::uint32_t>(H), input.data(), T,
                                     static_cast<std::uint32_t>(slot - kda_slots_), held,
                                     conv.empty() ? nullptr : conv.data(),
                                     r.recurrent_v_first.empty() ? nullptr : r.recurrent_v_first.data(),
                                     r.output.data());
        }
        if (rc != K3XB_OK) {
            if (slot && mode != Mode::host_roundtrip) slot->active = false;
            return Result<OfficialKdaCudaResult>::failure(static_cast<ErrorCode>(rc), last_error());
        }
        if (publish) {
            r.conv_q.assign(conv.begin(), conv.begin() + static_cast<std::ptrdiff_t>(hist));
            r.conv_k.assign(conv.begin() + static_cast<std::ptrdiff_t>(hist),
                            conv.begin() + static_cast<std::ptrdiff_t>(2 * hist));
            r.conv_v.assign(conv.begin() + static_cast<std::ptrdiff_t>(2 * hist), conv.end());
        } else {
            r.recurrent_v_first.clear();
        }
        r.executed = true;
        r.state_published = publish;   // backend_cuda.cu:2578-2580
        if (retain) {
            if (!++kda_generation_) ++kda_generation_;
            slot->generation = kda_generation_;
            slot->config = config;
            slot->active = true;
            r.device_state = {owner_, kda_generation_};
        }
        ++kda_calls_;
        return Result<OfficialKdaCudaResult>::success(std::move(r));
    }

    Result<bool> discard_official_kda_device_state(OfficialKdaDeviceStateToken token) override {
        if (token.owner != owner_) return Result<bool>::failure(ErrorCode::invalid_state);
        for (KdaSlot& s : kda_slots_)
            if (s.active && s.generation == token.generation) {
                s.active = false;
                return Result<bool>::success(true);
            }
        return Result<bool>::failure(ErrorCode::invalid_state);
    }

private:
    std::string last_error() const {
        char buf[512] = {0};
        if (ctx_) k3xb_last_error(ctx_, buf, sizeof buf);
        return buf;
    }

    static bool distinct_ids(std::span<const Mxfp4MlpView> experts) {
        std::unordered_set<std::uint64_t> ids;
        for (const auto& e : experts)
            for (const auto id : {e.gate.tensor_id, e.up.tensor_id, e.down.tensor_id})
                if (!ids.insert(id).second) return false;
        return true;
    }

    static std::vector<float> mix(const std::vector<std::vector<float>>& ys, std::span<const float> contributions) {
        std::vector<float> mixed(ys.front().size(), 0.0F);
        for (std::size_t slot = 0; slot < ys.size(); ++slot)
            for (std::size_t row = 0; row < mixed.size(); ++row) mixed[row] += contributions[slot] * ys[slot][row];
        return mixed;
    }

    // A device copy of one host weight; records a failure in *st.
    const void* resident(std::uint64_t id, std::int32_t kind, std::size_t rows, std::size_t cols, const void* data,
                         std::size_t bytes, ErrorCode* st) {
        k3xb_resident r{};
        const int rc = k3xb_acquire_weight(ctx_, id, kind, rows, cols, 0, data, bytes, nullptr, 0, &r);
        if (rc != K3XB_OK) {
            *st = static_cast<ErrorCode>(rc);
            return nullptr;
        }
        if (r.disposition == K3XB_RESIDENT_BYPASS) {
            *st = ErrorCode::backend_unavailable;   // over cuda_resident_bytes: the kernels read device copies
            return nullptr;
        }
        return r.primary;
    }

    // The expert as a resident stack of one, keyed by its gate tensor id.
    ErrorCode stack_of(const Mxfp4MlpView& e, std::size_t H, std::size_t I, k3xb_moe_layer* L) {
        if (H % 128 || I % 128) return ErrorCode::backend_unavailable;   // the tcgen05 tiles
        const k3xb_mxfp4_expert_host host{bytes_of(e.gate.packed), bytes_of(e.gate.scales), bytes_of(e.up.packed),
                                          bytes_of(e.up.scales),   bytes_of(e.down.packed), bytes_of(e.down.scales)};
        k3xb_resident_stack s{};
        const int rc = k3xb_acquire_expert_stack(ctx_, e.gate.tensor_id, 1, static_cast<std::uint32_t>(H),
                                                 static_cast<std::uint32_t>(I), &host, &s);
        if (rc != K3XB_OK) return static_cast<ErrorCode>(rc);
        if (s.disposition == K3XB_RESIDENT_BYPASS) return ErrorCode::backend_unavailable;
        *L = k3xb_moe_layer{};
        L->hidden = static_cast<std::uint32_t>(H);
        L->inter = static_cast<std::uint32_t>(I);
        L->experts = 1;
        L->top_k = 1;
        L->gate_packed = s.gate_packed;
        L->gate_scales = s.gate_scales;
        L->up_packed = s.up_packed;
        L->up_scales = s.up_scales;
        L->down_packed = s.down_packed;
        L->down_scales = s.down_scales;
        L->gate_scales_tc = s.gate_scales_tc;
        L->up_scales_tc = s.up_scales_tc;
        L->down_scales_tc = s.down_scales_tc;
        L->engine = K3XB_ENGINE_MXF4;
        return ErrorCode::ok;
    }

    // One expert as a one-expert layer: a resident stack on the tcgen05
    // engine where its dims are multiples of 128, else its three matrices
    // resident one by one on the CUDA-core engine (any multiple of 32).
    ErrorCode expert_of(const Mxfp4MlpView& e, std::size_t H, std::size_t I, k3xb_moe_layer* L) {
        if (H % 128 == 0 && I % 128 == 0) return stack_of(e, H, I, L);
        if (H % 32 || I % 32) return ErrorCode::backend_unavailable;
        k3xb_resident g{}, u{}, d{};
        const auto take = [this](const Mxfp4WeightView& w, k3xb_resident* r) {
            const int rc = k3xb_acquire_weight(ctx_, w.tensor_id, K3XB_WEIGHT_MXFP4, w.rows, w.cols, 32,
                                               w.packed.data(), w.packed.size(), w.scales.data(), w.scales.size(), r);
            if (rc != K3XB_OK) return static_cast<ErrorCode>(rc);
            return r->disposition == K3XB_RESIDENT_BYPASS ? ErrorCode::backend_unavailable : ErrorCode::ok;
        };
        ErrorCode st = take(e.gate, &g);
        if (st == ErrorCode::ok) st = take(e.up, &u);
        if (st == ErrorCode::ok) st = take(e.down, &d);
        if (st != ErrorCode::ok) return st;
        *L = k3xb_moe_layer{};
        L->hidden = static_cast<std::uint32_t>(H);
        L->inter = static_cast<std::uint32_t>(I);
        L->experts = 1;
        L->top_k = 1;
        L->gate_packed = static_cast<const std::uint8_t*>(g.primary);
        L->gate_scales = static_cast<const std::uint8_t*>(g.secondary);
        L->up_packed = static_cast<const std::uint8_t*>(u.primary);
        L->up_scales = static_cast<const std::uint8_t*>(u.secondary);
        L->down_packed = static_cast<const std::uint8_t*>(d.primary);
        L->down_scales = static_cast<const std::uint8_t*>(d.secondary);
        L->engine = K3XB_ENGINE_SIMT;
        return ErrorCode::ok;
    }

    // y [tokens][H] of one expert (gate/up, SiTU, down).
    Result<std::vector<float>> run_expert(const Mxfp4MlpView& e, std::size_t H, std::size_t I, const float* x,
                                          std::size_t tokens, float beta, std::optional<float> linear) {
        k3xb_moe_layer L{};
        if (auto st = expert_of(e, H, I, &L); st != ErrorCode::ok)
            return Result<std::vector<float>>::failure(st, last_error());
        L.activation = K3XB_ACT_SITU;
        L.situ_beta = beta;
        L.situ_linear_beta = linear ? *linear : 0.0F;
        std::vector<float> y(tokens * H);
        const std::uint32_t zero = 0;
        const int rc = k3xb_expert_grid_host(ctx_, &L, &zero, 1, x, static_cast<std::uint32_t>(tokens), y.data());
        if (rc != K3XB_OK) return Result<std::vector<float>>::failure(static_cast<ErrorCode>(rc), last_error());
        ++grid_calls_;
        grid_tokens_ += tokens;
        return Result<std::vector<float>>::success(std::move(y));
    }

    BackendOptions options_;
    k3xb_ctx* ctx_;
    std::map<std::uint64_t, std::vector<Mxfp4MlpView>> prefetched_;
    // the one prepared route (prepare_official_moe_route), its owner this backend
    struct PreparedRoute {
        bool active = false;
        std::uint64_t generation = 0;
        std::uint32_t layer = 0;
        std::uint32_t hidden_slot = 2;   // the layer hidden slot it holds (2: none)
        std::vector<float> prefix, hidden;
    } prepared_;
    // a layer's hidden rows between its tail and the next layer's front
    struct HiddenSlot {
        enum State { kFree, kLive, kPrepared } state = kFree;
        std::uint64_t generation = 0;
        std::uint32_t producing_layer = 0;
        std::size_t width = 0;
        std::vector<float> hidden, block;
    } hidden_slots_[2];
    std::uint64_t hidden_generation_ = 0;
    const std::uint64_t owner_ = next_owner();
    std::unordered_set<std::uint64_t> scanned_;   // bf16 route weights checked for non-finite words
    // the KDA states kept on the device for layers 1 and 2 (k3xb_kda_block_held slots 0 and 1)
    struct KdaSlot {
        bool active = false;
        std::uint64_t generation = 0;
        OfficialKdaCudaConfig config{};
    } kda_slots_[2];
    std::uint64_t kda_generation_ = 0;

    static bool same_config(const OfficialKdaCudaConfig& a, const OfficialKdaCudaConfig& b) {
        return a.hidden_size == b.hidden_size && a.heads == b.heads && a.head_dim == b.head_dim &&
               a.conv_width == b.conv_width && a.rms_norm_epsilon == b.rms_norm_epsilon &&
               a.gate_lower_bound == b.gate_lower_bound;
    }

    static std::uint64_t next_owner() {
        static std::atomic<std::uint64_t> n{0};
        return ++n;
    }
    std::uint64_t next_token_ = 0;
    std::uint64_t grid_calls_ = 0, grid_tokens_ = 0, moe_calls_ = 0, kda_calls_ = 0;
};

}  // namespace

std::unique_ptr<ComputeBackend> wrap_b200_context(const BackendOptions& options, k3xb_ctx* ctx) {
    return std::make_unique<B200Backend>(options, ctx);
}

Result<std::unique_ptr<ComputeBackend>> make_b200_backend(const BackendOptions& options, int device) {
    k3xb_ctx* ctx = nullptr;
    const int rc = k3xb_create(device, &ctx);
    if (rc != K3XB_OK)
        return Result<std::unique_ptr<ComputeBackend>>::failure(static_cast<ErrorCode>(rc),
                                                                "B200 backend: k3xb_create failed");
    return Result<std::unique_ptr<ComputeBackend>>::success(wrap_b200_context(options, ctx));
}

}  // namespace k3x
