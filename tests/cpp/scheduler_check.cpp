// The draft-length schedule of include/k3xb.hpp (DraftLengthScheduler)
// driven side by side with the reference's AdaptiveDraftScheduler
// (runtime/src/aurora_scheduler.cpp, compiled in place) on seeded random
// sequences of requests and verification outcomes, valid and invalid, for
// many configurations: every chosen length, status and counter must agree.
#include <cstdio>
#include <random>

#include "k3x/aurora_scheduler.hpp"
#include "k3xb.hpp"

#define CHECK(cond)                                                                        \
    do {                                                                                   \
        if (!(cond)) {                                                                     \
            std::fprintf(stderr, "check failed: %s (line %d, trial %d step %d)\n", #cond, \
                         __LINE__, trial, step);                                           \
            return 1;                                                                      \
        }                                                                                  \
    } while (0)

int main() {
    std::mt19937_64 rng(20260);
    const std::size_t lengths[] = {1, 2, 4};
    const double survivals[] = {0.0, 0.3, 0.5, 0.8, 1.0};
    const double ratios[] = {0.0, 0.2, 0.5, 0.9, 1.0};
    int trial = 0, step = 0;
    std::uint64_t compared = 0;
    for (trial = 0; trial < 400; ++trial) {
        k3x::AuroraSchedulerConfig rc;
        rc.policy = rng() % 2 ? k3x::AuroraBlockPolicy::adaptive : k3x::AuroraBlockPolicy::fixed;
        rc.maximum_length = lengths[rng() % 3];
        rc.minimum_prefix_survival = survivals[rng() % 5];
        rc.maximum_unique_load_ratio = ratios[rng() % 5];
        k3xb::DraftSchedulerConfig oc{rc.policy == k3x::AuroraBlockPolicy::adaptive ? k3xb::DraftPolicy::adaptive
                                                                                     : k3xb::DraftPolicy::fixed,
                                      rc.maximum_length, rc.minimum_prefix_survival, rc.maximum_unique_load_ratio};
        auto ref = k3x::AdaptiveDraftScheduler::create(rc);
        auto ours = k3xb::DraftLengthScheduler::create(oc);
        CHECK(static_cast<bool>(ref) && static_cast<bool>(ours));
        auto& R = ref.value();
        auto& O = ours.value();
        const double accept_rate = (rng() % 100) / 100.0;
        for (step = 0; step < 300; ++step) {
            const std::size_t request = rng() % 6;
            auto a = R.select(request);
            auto b = O.select(request);
            CHECK(static_cast<bool>(a) && static_cast<bool>(b));
            CHECK(a.value() == b.value());
            ++compared;
            const std::size_t len = a.value();
            k3x::DraftVerification v;
            v.proposed_draft_tokens = len;
            std::size_t acc = 0;
            while (acc < len && std::uniform_real_distribution<double>(0, 1)(rng) < accept_rate) ++acc;
            v.accepted_draft_tokens = acc;
            v.target_positions_evaluated = len + 1;
            v.target_positions_discarded = len - acc;
            v.expert_major_assignments = len ? rng() % 64 : 0;
            v.expert_major_payload_loads = v.expert_major_assignments ? rng() % (v.expert_major_assignments + 1) : 0;
            switch (rng() % 16) {   // now and then an inconsistent report
                case 0: v.accepted_draft_tokens = len + 1; break;
                case 1: v.proposed_draft_tokens = 3; break;
                case 2: v.expert_major_payload_loads = v.expert_major_assignments + 1; break;
                case 3: v.target_positions_discarded = v.target_positions_evaluated + 1; break;
                default: break;
            }
            const k3xb::DraftObservation o{v.proposed_draft_tokens, v.accepted_draft_tokens,
                                           v.target_positions_evaluated, v.target_positions_discarded,
                                           v.expert_major_payload_loads, v.expert_major_assignments};
            auto ra = R.observe(v);
            auto ob = O.observe(o);
            CHECK(static_cast<bool>(ra) == static_cast<bool>(ob));
            if (!ra) CHECK(static_cast<int>(ra.error()) == static_cast<int>(ob.status()));
            const auto rs = R.stats();
            const auto& os = O.stats();
            CHECK(rs.selected_length_1 == os.selected_1 && rs.selected_length_2 == os.selected_2 &&
                  rs.selected_length_4 == os.selected_4);
            CHECK(rs.scheduler_growths == os.growths && rs.scheduler_backoffs == os.backoffs);
        }
    }
    // configuration checks
    for (std::size_t len : {0, 3, 5}) {
        k3x::AuroraSchedulerConfig rc;
        rc.maximum_length = len;
        k3xb::DraftSchedulerConfig oc;
        oc.maximum_length = len;
        CHECK(!k3x::AdaptiveDraftScheduler::create(rc) && !k3xb::DraftLengthScheduler::create(oc));
    }
    std::printf("scheduler ok %llu decisions\n", static_cast<unsigned long long>(compared));
    return 0;
}
