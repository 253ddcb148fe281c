// Host-side checks of the C++20 layer (include/k3xb.hpp): result unpacking,
// the drafting round, and context creation failing loudly without a B200.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "k3xb.hpp"

#define CHECK(cond)                                                              \
    do {                                                                         \
        if (!(cond)) {                                                           \
            std::fprintf(stderr, "check failed: %s (line %d)\n", #cond, __LINE__); \
            return 1;                                                            \
        }                                                                        \
    } while (0)

namespace {

// Proposes anchor+1, anchor+2, ... and records what it was told.
class CountingDrafter final : public k3xb::DraftSource {
public:
    std::vector<k3xb::Verification> seen;
    k3xb::Result<std::vector<k3xb::Draft>> propose(std::span<const k3xb::DraftAsk> asks) override {
        std::vector<k3xb::Draft> out;
        for (const auto& a : asks) {
            k3xb::Draft d{a.anchor, {}};
            for (std::size_t i = 0; i < a.max_drafts; ++i) d.tokens.push_back(a.anchor + 1 + static_cast<uint32_t>(i));
            out.push_back(std::move(d));
        }
        return out;
    }
    void update(std::span<const k3xb::Verification> r) override { seen.assign(r.begin(), r.end()); }
};

// Accepts drafts while they are even, then commits 0 as the target token.
class EvenVerifier final : public k3xb::Verifier {
public:
    k3xb::Result<std::vector<k3xb::Verification>> verify(std::span<const k3xb::Draft> drafts) override {
        std::vector<std::uint32_t> acc, com, cnt;
        std::size_t p = 0;
        for (const auto& d : drafts) p = std::max(p, d.tokens.size());
        for (const auto& d : drafts) {
            std::uint32_t a = 0;
            while (a < d.tokens.size() && d.tokens[a] % 2 == 0) ++a;
            acc.push_back(a);
            for (std::size_t i = 0; i <= p; ++i) com.push_back(i < a ? d.tokens[i] : 0u);
            cnt.push_back(a + 1);
        }
        return k3xb::unpack_verifications(acc, com, cnt, p);
    }
};

}  // namespace

int main() {
    // unpack: 3 sequences of 4 drafts
    const std::vector<std::uint32_t> accepted{0, 4, 2}, counts{1, 5, 3};
    const std::vector<std::uint32_t> committed{7, 0, 0, 0, 0, 1, 2, 3, 4, 9, 5, 6, 8, 0, 0};
    auto r = k3xb::unpack_verifications(accepted, committed, counts, 4);
    CHECK(r);
    CHECK(r.value().size() == 3);
    CHECK(r.value()[0].committed == std::vector<std::uint32_t>{7});
    CHECK(r.value()[1].all_accepted && r.value()[1].committed.size() == 5);
    CHECK(r.value()[2].committed == (std::vector<std::uint32_t>{5, 6, 8}));
    const std::vector<std::uint32_t> bad{2, 5, 3};
    auto b = k3xb::unpack_verifications(accepted, committed, bad, 4);
    CHECK(!b && b.outcome().status() == k3xb::Status::invalid_state);
    auto m = k3xb::unpack_verifications(accepted, std::span(committed).first(10), counts, 4);
    CHECK(!m && m.outcome().status() == k3xb::Status::invalid_extent);

    // one drafting round on host fakes
    CountingDrafter drafter;
    EvenVerifier verifier;
    const std::vector<k3xb::DraftAsk> asks{{1, 3}, {3, 3}};
    auto round = k3xb::speculative_round(drafter, verifier, asks);
    CHECK(round);
    CHECK(drafter.seen.size() == 2);
    CHECK(drafter.seen[0].accepted == 1 && drafter.seen[0].committed == (std::vector<std::uint32_t>{2, 0}));
    CHECK(drafter.seen[1].accepted == 1);

    // the host-vector calls check their sizes before the C ABI; an empty
    // context is answered by the C ABI (INVALID_EXTENT), never by a fallback
    k3xb::Context none;
    const std::vector<float> x(8, 1.0F);
    std::vector<float> y(3), y4(4);
    CHECK(none.dense_matvec(nullptr, 4, x, y).status() == k3xb::Status::invalid_extent);
    CHECK(none.dense_matvec(nullptr, 4, x, y4).status() == k3xb::Status::invalid_extent);
    CHECK(none.mxfp4_matvec(nullptr, nullptr, 4, x, y).status() == k3xb::Status::invalid_extent);
    k3xb_kda_layer w{};
    CHECK(none.kda_block_held(w, 3, x, 0, K3XB_KDA_SEED, {}, {}, y).status() == k3xb::Status::invalid_extent);
    // a seed or publish must bring state arrays of the layer's sizes
    w.heads = 2;
    w.head_dim = 4;
    w.conv_width = 4;
    std::vector<std::uint16_t> conv(3 * 3 * 8), conv_short(3 * 3 * 8 - 1);
    std::vector<float> rec(2 * 4 * 4), y9(9);
    const std::vector<float> x9(9, 1.0F);
    CHECK(none.kda_block_held(w, 3, x9, 0, K3XB_KDA_SEED, conv_short, rec, y9).status() ==
          k3xb::Status::invalid_extent);
    CHECK(none.kda_block_held(w, 3, x9, 0, K3XB_KDA_PUBLISH, conv, {}, y9).status() ==
          k3xb::Status::invalid_extent);

    // no B200 here: creation must fail with a status, never fall back
    auto ctx = k3xb::Context::create(0);
    if (ctx) {
        std::printf("adapter ok (device present)\n");
        return 0;
    }
    const auto st = ctx.outcome().status();
    CHECK(st == k3xb::Status::backend_unavailable || st == k3xb::Status::unsupported_architecture ||
          st == k3xb::Status::invalid_extent);
    std::printf("adapter ok (%s)\n", k3xb::status_name(st));
    return 0;
}
