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

#include <cstddef>
#include <cstdint>
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
        if (!hidden_size || hidden.size() % hidden_size || router.size() != std::size_t(E) * hidden_size)
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

    // Expert parallelism over the GPUs of one box.
    Outcome ep_init(std::span<const std::uint8_t, 128> unique_id, int rank, int world) {
        return check(k3xb_ep_init(h_, unique_id.data(), rank, world));
    }
    Outcome ep_finalize() { return check(k3xb_ep_finalize(h_)); }

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
