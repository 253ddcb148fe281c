// k3xb.hpp — C++20 host layer over the C ABI of libk3xb (k3xb.h).
//
// Header-only. It adds ownership (RAII contexts, model descriptors that
// keep their layer arrays alive), status values that cannot be ignored, and
// the host side of batched speculative verification: unpacking the
// device's per-sequence acceptance arrays into per-sequence results, and a
// draft-source interface so a drafter and the device verifier can be driven
// by one loop. Device arrays are passed as std::span views over DEVICE
// memory; the host never dereferences them.
//
// The result shape follows the reference's DraftVerification
// (runtime/include/k3x/speculative.hpp:24-34: accepted count, committed
// tokens, all-accepted flag) and its proposal/update split of DraftProvider
// (speculative.hpp:58-64), so an adapter can copy fields one to one.
#pragma once

#include <algorithm>
#include <array>
#include <cstddef>
#include <cstdint>
#include <limits>
#include <optional>
#include <span>
#include <string>
#include <utility>
#include <vector>

#include "k3xb.h"

namespace k3xb {

// Status values of k3xb.h (the values of k3x::ErrorCode,
// runtime/include/k3x/status.hpp:9-30).
enum class Status : int {
    ok = K3XB_OK,
    invalid_extent = K3XB_INVALID_EXTENT,
    invalid_mxfp4 = K3XB_INVALID_MXFP4,
    invalid_state = K3XB_INVALID_STATE,
    backend_unavailable = K3XB_BACKEND_UNAVAILABLE,
    unsupported_architecture = K3XB_UNSUPPORTED_ARCHITECTURE,
};

// The C ABI counts in uint32_t; a larger host count is an extent error, not a wrap.
constexpr bool fits_u32(std::size_t n) noexcept { return n <= 0xffffffffull; }

inline const char* status_name(Status s) noexcept {
    switch (s) {
        case Status::ok: return "OK";
        case Status::invalid_extent: return "INVALID_EXTENT";
        case Status::invalid_mxfp4: return "INVALID_MXFP4";
        case Status::invalid_state: return "INVALID_STATE";
        case Status::backend_unavailable: return "BACKEND_UNAVAILABLE";
        case Status::unsupported_architecture: return "UNSUPPORTED_ARCHITECTURE";
    }
    return "UNKNOWN";
}

// A status with the context's message; [[nodiscard]] so failures are seen.
class [[nodiscard]] Outcome {
public:
    Outcome() = default;
    Outcome(Status s, std::string message) : status_(s), message_(std::move(message)) {}
    explicit operator bool() const noexcept { return status_ == Status::ok; }
    Status status() const noexcept { return status_; }
    const std::string& message() const noexcept { return message_; }

private:
    Status status_ = Status::ok;
    std::string message_;
};

// Value or failure.
template <class T>
class [[nodiscard]] Result {
public:
    Result(T value) : value_(std::move(value)) {}
    Result(Outcome failure) : failure_(std::move(failure)) {}
    explicit operator bool() const noexcept { return static_cast<bool>(failure_); }
    T& value() & { return value_; }
    T&& value() && { return std::move(value_); }
    const Outcome& outcome() const noexcept { return failure_; }

private:
    T value_{};
    Outcome failure_{};
};

// ---- per-sequence verification results ------------------------------------

struct Verification {
    std::uint32_t accepted = 0;             // accepted draft tokens
    std::vector<std::uint32_t> committed;   // accepted drafts + one target token
    bool all_accepted = false;
};

// Unpacks the device arrays of k3xb_accept_greedy / k3xb_accept_rejection /
// k3xb_verify_step (copied to the host): accepted [S], committed [S][p+1],
// committed_count [S]. Fails on counts that are not accepted + 1 or exceed
// p + 1 (a sequence always commits its accepted drafts plus one token).
inline Result<std::vector<Verification>> unpack_verifications(std::span<const std::uint32_t> accepted,
                                                              std::span<const std::uint32_t> committed,
                                                              std::span<const std::uint32_t> counts,
                                                              std::size_t drafts_per_sequence) {
    const std::size_t S = accepted.size(), stride = drafts_per_sequence + 1;
    if (counts.size() != S || committed.size() != S * stride)
        return Outcome(Status::invalid_extent, "verification arrays of mismatched sizes");
    std::vector<Verification> out(S);
    for (std::size_t s = 0; s < S; ++s) {
        const std::uint32_t a = accepted[s], n = counts[s];
        if (a > drafts_per_sequence || n != a + 1u)
            return Outcome(Status::invalid_state, "committed count must be accepted + 1");
        out[s].accepted = a;
        out[s].committed.assign(committed.begin() + static_cast<std::ptrdiff_t>(s * stride),
                                committed.begin() + static_cast<std::ptrdiff_t>(s * stride + n));
        out[s].all_accepted = a == drafts_per_sequence;
    }
    return out;
}

// ---- context ----------------------------------------------------------------

class Context {
public:
    static Result<Context> create(int device) {
        k3xb_ctx* h = nullptr;
        const int st = k3xb_create(device, &h);
        if (st != K3XB_OK) return Outcome(static_cast<Status>(st), "k3xb_create failed");
        return Context(h);
    }
    Context() = default;
    Context(Context&& o) noexcept : h_(std::exchange(o.h_, nullptr)) {}
    Context& operator=(Context&& o) noexcept {
        if (this != &o) {
            reset();
            h_ = std::exchange(o.h_, nullptr);
        }
        return *this;
    }
    Context(const Context&) = delete;
    Context& operator=(const Context&) = delete;
    ~Context() { reset(); }

    k3xb_ctx* handle() const noexcept { return h_; }
    explicit operator bool() const noexcept { return h_ != nullptr; }

    // Wraps a C status with this context's last error message.
    Outcome check(int st) const {
        if (st == K3XB_OK) return {};
        char buf[512] = {0};
        if (h_) k3xb_last_error(h_, buf, sizeof buf);
        return Outcome(static_cast<Status>(st), buf);
    }

    Outcome set_stream(void* cuda_stream) { return check(k3xb_set_stream(h_, cuda_stream)); }
    Outcome sync() { return check(k3xb_sync(h_)); }
    Result<k3xb_stats> stats() const {
        k3xb_stats s{};
        const Outcome o = check(k3xb_get_stats(h_, &s));
        if (!o) return o;
        return s;
    }

    // (a) routing of T tokens (device views).
    Outcome route(std::span<const float> hidden, std::uint32_t hidden_size, std::span<const std::uint16_t> router,
                  std::span<const float> correction, std::uint32_t top_k, std::span<std::uint32_t> ids,
                  std::span<float> contributions) {
        const auto E = static_cast<std::uint32_t>(correction.size());
        if (!hidden_size || hidden.size() % hidden_size || router.size() != std::size_t(E) * hidden_size ||
            !fits_u32(correction.size()) || !fits_u32(hidden.size() / hidden_size))
            return Outcome(Status::invalid_extent, "route: sizes");
        const auto T = static_cast<std::uint32_t>(hidden.size() / hidden_size);
        if (ids.size() != std::size_t(T) * top_k || contributions.size() != ids.size())
            return Outcome(Status::invalid_extent, "route: output sizes");
        return check(k3xb_route(h_, hidden.data(), T, hidden_size, router.data(), correction.data(), E, top_k,
                                ids.data(), contributions.data(), nullptr));
    }

    // (b)+(c) one MoE layer over resident weights (device views).
    Outcome moe_layer(const k3xb_moe_layer& layer, std::span<const float> hidden, std::span<float> out,
                      std::span<std::uint32_t> ids = {}, std::span<float> contributions = {}) {
        if (!layer.hidden || hidden.size() % layer.hidden || out.size() != hidden.size())
            return Outcome(Status::invalid_extent, "moe_layer: sizes");
        const auto T = static_cast<std::uint32_t>(hidden.size() / layer.hidden);
        return check(k3xb_moe_layer_forward(h_, &layer, hidden.data(), T, out.data(),
                                            ids.empty() ? nullptr : ids.data(),
                                            contributions.empty() ? nullptr : contributions.data()));
    }

    // Whole verify step (device arrays in `io`); results stay on the device.
    Outcome verify_step(const k3xb_verify_model& model, const k3xb_verify_io& io) {
        return check(k3xb_verify_step(h_, &model, &io));
    }

    // AURORA reduced-Top-K drafts on the device, and a whole on-device round
    // (draft, verify, advance the state, next anchors); the length comes
    // from a DraftLengthScheduler on the host.
    Outcome draft(const k3xb_verify_model& model, const k3xb_draft_io& io) {
        return check(k3xb_draft_greedy(h_, &model, &io));
    }
    Outcome speculative_step(const k3xb_verify_model& model, const k3xb_speculative_io& io) {
        return check(k3xb_speculative_step(h_, &model, &io));
    }

    // Expert parallelism over the GPUs of one box. Every wait on the
    // communicator is bounded by `config.timeout_ms`; past it, or on an error
    // NCCL reports, the communicator is aborted (backend_unavailable) and the
    // expert-parallel calls answer invalid_state until ep_finalize + ep_init.
    Outcome ep_init(std::span<const std::uint8_t, 128> unique_id, int rank, int world,
                    const k3xb_ep_config& config = {0, 0}) {
        return check(k3xb_ep_init_config(h_, unique_id.data(), rank, world, &config));
    }
    Outcome ep_status() { return check(k3xb_ep_status(h_)); }
    Outcome ep_abort() { return check(k3xb_ep_abort(h_)); }
    Outcome ep_finalize() { return check(k3xb_ep_finalize(h_)); }

    // The reference's per-call ComputeBackend shapes (host vectors in and
    // out, device weights): each returns after its results are on the host.
    // f32 dense product (dense_matvec), bit-identical to the CPU backend.
    Outcome dense_matvec(const float* W, std::uint32_t rows, std::span<const float> x, std::span<float> y) {
        if (y.size() != rows || x.empty() || !fits_u32(x.size()))
            return Outcome(Status::invalid_extent, "dense_matvec: sizes");
        return check(k3xb_dense_matvec_host(h_, W, rows, static_cast<std::uint32_t>(x.size()), x.data(), y.data()));
    }
    // MXFP4 product (mxfp4_matvec), bit-identical to mxfp4_matmul.
    Outcome mxfp4_matvec(const std::uint8_t* packed, const std::uint8_t* scales, std::uint32_t rows,
                         std::span<const float> x, std::span<float> y) {
        if (y.size() != rows || x.empty() || !fits_u32(x.size()))
            return Outcome(Status::invalid_extent, "mxfp4_matvec: sizes");
        return check(k3xb_mxfp4_matvec_host(h_, packed, scales, rows, static_cast<std::uint32_t>(x.size()), x.data(),
                                            y.data()));
    }
    // The official LatentMoE FFN of one position, its route given
    // (official_mxfp4_moe_ffn): one one-expert layer per slot.
    Outcome official_moe_ffn(const k3xb_moe_layer& tail, std::span<const k3xb_moe_layer> slots,
                             std::span<const float> contributions, std::span<const float> hidden,
                             std::span<const float> prefix, std::span<float> out) {
        if (slots.size() != contributions.size() || !fits_u32(slots.size()) || hidden.size() != tail.hidden ||
            prefix.size() != tail.hidden || out.size() != tail.hidden)
            return Outcome(Status::invalid_extent, "official_moe_ffn: sizes");
        return check(k3xb_official_moe_ffn_host(h_, &tail, slots.data(), static_cast<std::uint32_t>(slots.size()),
                                                contributions.data(), hidden.data(), prefix.data(), out.data()));
    }
    // The KDA block with its state held on the device between calls
    // (official_kda's device state modes); conv/recurrent as k3xb_kda_block_held.
    // conv is [3][conv_width - 1][heads * head_dim] bf16 words and recurrent
    // [heads][head_dim][head_dim]: SEED reads them and PUBLISH writes them,
    // so there both must have exactly those sizes; CONTINUE ignores them.
    Outcome kda_block_held(const k3xb_kda_layer& w, std::uint32_t hidden, std::span<const float> x,
                           std::uint32_t slot, std::int32_t mode, std::span<std::uint16_t> conv,
                           std::span<float> recurrent, std::span<float> out) {
        if (!hidden || x.size() % hidden || out.size() != x.size() || !fits_u32(x.size() / hidden))
            return Outcome(Status::invalid_extent, "kda_block_held: sizes");
        const std::size_t width = std::size_t(w.heads) * w.head_dim;
        const std::size_t conv_n = w.conv_width ? 3 * std::size_t(w.conv_width - 1) * width : 0;
        const std::size_t rec_n = width * w.head_dim;
        if (mode != K3XB_KDA_CONTINUE && (conv.size() != conv_n || recurrent.size() != rec_n))
            return Outcome(Status::invalid_extent, "kda_block_held: state sizes");
        return check(k3xb_kda_block_held(h_, &w, hidden, x.data(), static_cast<std::uint32_t>(x.size() / hidden),
                                         slot, mode, conv.empty() ? nullptr : conv.data(),
                                         recurrent.empty() ? nullptr : recurrent.data(), out.data()));
    }

private:
    explicit Context(k3xb_ctx* h) : h_(h) {}
    void reset() noexcept {
        if (h_) k3xb_destroy(h_);
        h_ = nullptr;
    }
    k3xb_ctx* h_ = nullptr;
};

// A fresh NCCL id for Context::ep_init on every rank.
inline Result<std::vector<std::uint8_t>> ep_unique_id() {
    std::vector<std::uint8_t> id(128);
    const int st = k3xb_ep_unique_id(id.data());
    if (st != K3XB_OK) return Outcome(static_cast<Status>(st), "k3xb_ep_unique_id failed");
    return id;
}

// A verify stack: owns the layer descriptor array the C model points into.
class VerifyModel {
public:
    VerifyModel(std::vector<k3xb_layer> layers, std::uint32_t vocab, const std::uint16_t* lm_head,
                const std::uint16_t* embedding = nullptr, const std::uint16_t* final_norm = nullptr,
                float final_eps = 1e-6f)
        : layers_(std::move(layers)) {
        model_.layers = static_cast<std::uint32_t>(layers_.size());
        model_.vocab = vocab;
        model_.layer = layers_.data();
        model_.embedding = embedding;
        model_.final_norm = final_norm;
        model_.final_eps = final_eps;
        model_.lm_head = lm_head;
    }
    VerifyModel(const VerifyModel&) = delete;
    VerifyModel& operator=(const VerifyModel&) = delete;
    const k3xb_verify_model& c() const noexcept { return model_; }

private:
    std::vector<k3xb_layer> layers_;
    k3xb_verify_model model_{};
};

// ---- drafting ---------------------------------------------------------------

// What a drafter is asked for and what it returns, per sequence.
struct DraftAsk {
    std::uint32_t anchor = 0;
    std::size_t max_drafts = 0;
};
struct Draft {
    std::uint32_t anchor = 0;
    std::vector<std::uint32_t> tokens;
};

// A drafter: proposes drafts for a batch of sequences, then learns what the
// verifier accepted (the proposal/update split of the reference's
// DraftProvider).
class DraftSource {
public:
    virtual ~DraftSource() = default;
    virtual Result<std::vector<Draft>> propose(std::span<const DraftAsk> asks) = 0;
    virtual void update(std::span<const Verification> results) = 0;
};

// A verifier: the device side of one round for a batch of drafts.
class Verifier {
public:
    virtual ~Verifier() = default;
    virtual Result<std::vector<Verification>> verify(std::span<const Draft> drafts) = 0;
};

// ---- draft length -----------------------------------------------------------

// How many tokens to draft next: the AURORA ladder of 1, 2 or 4 drafts
// (AdaptiveDraftScheduler, aurora_scheduler.cpp:37-199). `fixed` always
// takes the longest rung within the caps. `adaptive` climbs one rung at a
// time while the Laplace-smoothed survival of the last drafted position,
// (accepted there + 1) / (tried there + 2), stays at or above
// minimum_prefix_survival and the rung's unique-expert loads per
// assignment stay at or below maximum_unique_load_ratio; a rejection caps
// the next choice one rung lower (none after a rejection at rung 1, then
// one retry of rung 1).
enum class DraftPolicy { fixed, adaptive };

struct DraftSchedulerConfig {
    DraftPolicy policy = DraftPolicy::fixed;
    std::size_t maximum_length = 1;            // 1, 2 or 4
    double minimum_prefix_survival = 0.5;      // [0, 1]
    double maximum_unique_load_ratio = 0.9;    // [0, 1]
};

// What one verification of `proposed` drafts reported (the fields of
// k3x::DraftVerification the schedule reads, speculative.hpp:25-35).
struct DraftObservation {
    std::size_t proposed = 0, accepted = 0;
    std::size_t positions_evaluated = 0, positions_discarded = 0;
    std::size_t expert_loads = 0, expert_assignments = 0;   // unique experts loaded, (token, slot) pairs
};

struct DraftSchedulerStats {
    std::uint64_t selected_1 = 0, selected_2 = 0, selected_4 = 0;
    std::uint64_t growths = 0, backoffs = 0;
};

class DraftLengthScheduler {
public:
    static Result<DraftLengthScheduler> create(const DraftSchedulerConfig& c) {
        const auto unit = [](double v) { return v == v && v >= 0.0 && v <= 1.0; };   // finite, in [0, 1]
        if (!rung_of(c.maximum_length) || !unit(c.minimum_prefix_survival) || !unit(c.maximum_unique_load_ratio))
            return Outcome(Status::invalid_extent, "draft scheduler: maximum_length in {1, 2, 4}, ratios in [0, 1]");
        DraftLengthScheduler s;
        s.cfg_ = c;
        return s;
    }
    DraftLengthScheduler() = default;

    const DraftSchedulerStats& stats() const noexcept { return stats_; }

    // Drafts to propose when the caller allows at most `request_maximum`.
    Result<std::size_t> select(std::size_t request_maximum) {
        if (request_maximum == 0) return std::size_t{0};
        std::size_t cap = std::min(request_maximum, cfg_.maximum_length);
        if (has_cap_) cap = std::min(cap, cap_after_reject_);
        if (cap == 0) {   // only a rejection at rung 1 gets here: retry rung 1 next time
            if (has_cap_ && cap_after_reject_ == 0) {
                has_cap_ = false;
                retry_first_ = true;
            }
            return std::size_t{0};
        }
        if (cfg_.policy == DraftPolicy::fixed) {
            for (std::size_t r = kRungs.size(); r-- > 0;)
                if (kRungs[r] <= cap) return take(r);
            return std::size_t{0};
        }
        if (retry_first_) {
            retry_first_ = false;
            return take(0);
        }
        const std::size_t top = has_qualified_ ? std::min(qualified_ + 1, *rung_of(cfg_.maximum_length)) : 0;
        for (std::size_t r = top + 1; r-- > 0;) {
            if (kRungs[r] > cap) continue;
            if (seen_[r] && !(survival(kRungs[r] - 1) >= cfg_.minimum_prefix_survival && cost_ok(r))) continue;
            return take(r);
        }
        return std::size_t{0};
    }

    // Learns from one verification of the drafts select() chose.
    Outcome observe(const DraftObservation& o) {
        if (o.proposed == 0) {
            if (o.accepted || o.expert_loads || o.expert_assignments || o.positions_discarded > o.positions_evaluated)
                return Outcome(Status::invalid_extent, "draft scheduler: an empty proposal reports nothing");
            return {};
        }
        const auto rung = rung_of(o.proposed);
        if (!rung || o.proposed > cfg_.maximum_length || o.accepted > o.proposed ||
            o.positions_discarded > o.positions_evaluated || (o.expert_loads && !o.expert_assignments) ||
            o.expert_loads > o.expert_assignments)
            return Outcome(Status::invalid_extent, "draft scheduler: inconsistent observation");
        const std::size_t r = *rung;
        constexpr auto kMax = std::numeric_limits<std::uint64_t>::max();
        for (std::size_t i = 0; i < o.proposed; ++i)
            if (tried_[i] == kMax) return Outcome(Status::invalid_state, "draft scheduler: counter overflow");
        if (o.expert_loads > kMax - loads_[r] || o.expert_assignments > kMax - assignments_[r])
            return Outcome(Status::invalid_state, "draft scheduler: counter overflow");
        for (std::size_t i = 0; i < o.proposed; ++i) {
            ++tried_[i];
            if (o.accepted > i) ++survived_[i];
        }
        loads_[r] += o.expert_loads;
        assignments_[r] += o.expert_assignments;
        seen_[r] = true;
        if (cfg_.policy == DraftPolicy::fixed) return {};
        if (o.accepted < o.proposed) {   // back off one rung (to none from rung 1)
            has_cap_ = true;
            cap_after_reject_ = r == 0 ? 0 : kRungs[r - 1];
            ++stats_.backoffs;
            return {};
        }
        has_cap_ = false;
        if (survival(o.proposed - 1) >= cfg_.minimum_prefix_survival && cost_ok(r) &&
            (!has_qualified_ || r > qualified_)) {
            has_qualified_ = true;
            qualified_ = r;
            if (r + 1 < kRungs.size()) ++stats_.growths;
        }
        return {};
    }

private:
    static constexpr std::array<std::size_t, 3> kRungs{1, 2, 4};
    static std::optional<std::size_t> rung_of(std::size_t length) {
        for (std::size_t r = 0; r < kRungs.size(); ++r)
            if (kRungs[r] == length) return r;
        return std::nullopt;
    }
    double survival(std::size_t position) const {
        return static_cast<double>(survived_[position] + 1) / static_cast<double>(tried_[position] + 2);
    }
    bool cost_ok(std::size_t r) const {
        return assignments_[r] == 0 ||
               static_cast<double>(loads_[r]) / static_cast<double>(assignments_[r]) <= cfg_.maximum_unique_load_ratio;
    }
    std::size_t take(std::size_t r) {
        (r == 0 ? stats_.selected_1 : r == 1 ? stats_.selected_2 : stats_.selected_4) += 1;
        return kRungs[r];
    }

    DraftSchedulerConfig cfg_{};
    std::array<std::uint64_t, 4> tried_{}, survived_{};   // per drafted position
    std::array<std::uint64_t, 3> loads_{}, assignments_{};   // per rung
    std::array<bool, 3> seen_{};
    bool has_qualified_ = false, has_cap_ = false, retry_first_ = false;
    std::size_t qualified_ = 0, cap_after_reject_ = 0;
    DraftSchedulerStats stats_{};
};

// One speculative round: ask the drafter, verify, report back; returns the
// per-sequence results. The next anchors are the last committed tokens.
inline Result<std::vector<Verification>> speculative_round(DraftSource& drafter, Verifier& verifier,
                                                           std::span<const DraftAsk> asks) {
    auto drafts = drafter.propose(asks);
    if (!drafts) return drafts.outcome();
    if (drafts.value().size() != asks.size())
        return Outcome(Status::invalid_state, "drafter returned a different batch size");
    for (std::size_t s = 0; s < asks.size(); ++s)
        if (drafts.value()[s].tokens.size() > asks[s].max_drafts)
            return Outcome(Status::invalid_extent, "drafter exceeded max_drafts");
    auto results = verifier.verify(drafts.value());
    if (!results) return results.outcome();
    drafter.update(results.value());
    return results;
}

}  // namespace k3xb
