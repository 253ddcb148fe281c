// The expert-parallel failure detection (project-k3x_b200/csrc/ep_guard.hpp)
// against a scripted communicator and stream on a fake clock: every wait
// ends by its deadline, errors and expiries abort the communicator exactly
// once, and an aborted communicator refuses further work.
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "ep_guard.hpp"

namespace {

int failures = 0;

#define CHECK(cond)                                                          \
    do {                                                                     \
        if (!(cond)) {                                                       \
            std::fprintf(stderr, "%s:%d: CHECK(%s) failed\n", __FILE__, __LINE__, #cond); \
            ++failures;                                                      \
        }                                                                    \
    } while (0)

// What the communicator and the stream do, poll by poll.
struct Script {
    uint64_t clock = 0;              // ms
    uint64_t tick = 10;              // ms per pause
    std::vector<int> states;         // communicator state per async_error call; the last repeats
    size_t next_state = 0;
    int query_status = 0;            // ncclCommGetAsyncError's own return
    int aborts = 0;
    int async_calls = 0;
    long stream_pending = 0;         // polls before the stream drains; -1: until an abort; -2: never
    bool stream_error = false;
    int stream_polls = 0;
};

struct FakeOps {
    Script* s;
    int async_error(int* state) {
        ++s->async_calls;
        if (s->states.empty()) {
            *state = k3xb::kCommSuccess;
        } else {
            *state = s->states[s->next_state < s->states.size() ? s->next_state : s->states.size() - 1];
            ++s->next_state;
        }
        return s->query_status;
    }
    int abort() {
        ++s->aborts;
        return 0;
    }
    int stream_query() {
        ++s->stream_polls;
        if (s->stream_error) return -1;
        if (s->stream_pending == -2) return 1;
        if (s->stream_pending == -1) return s->aborts ? 0 : 1;
        if (s->stream_pending > 0) {
            --s->stream_pending;
            return 1;
        }
        return 0;
    }
    uint64_t now_ms() const { return s->clock; }
    void pause(uint32_t) const { s->clock += s->tick; }
    const char* describe(int r) const { return r == 6 ? "remote process exited or there was a network error" : "error"; }
};

using Guard = k3xb::CommGuard<FakeOps>;
using k3xb::CommWait;
constexpr int kInProgress = k3xb::kCommInProgress;
constexpr int kRemoteError = 6;   // ncclRemoteError

bool contains(const std::string& s, const char* part) { return s.find(part) != std::string::npos; }

void settle_cases() {
    {   // a blocking call that succeeded: nothing to wait for
        Script s;
        Guard g(FakeOps{&s}, 100);
        CHECK(g.settle(0, "launch") == CommWait::ok);
        CHECK(s.async_calls == 0 && s.aborts == 0 && !g.aborted());
    }
    {   // nonblocking: in progress for two polls, then settled
        Script s;
        s.states = {kInProgress, kInProgress, 0};
        Guard g(FakeOps{&s}, 100);
        CHECK(g.settle(kInProgress, "launch") == CommWait::ok);
        CHECK(s.async_calls == 3 && s.aborts == 0 && !g.aborted());
    }
    {   // never settles: aborted at the deadline, once; then everything refuses
        Script s;
        s.states = {kInProgress};
        Guard g(FakeOps{&s}, 100);
        CHECK(g.settle(kInProgress, "ncclCommInitRankConfig") == CommWait::timed_out);
        CHECK(s.aborts == 1 && g.aborted());
        CHECK(s.clock >= 100 && s.clock <= 100 + s.tick);
        CHECK(contains(g.reason(), "ncclCommInitRankConfig: still in progress after 100 ms"));
        CHECK(g.settle(0, "launch") == CommWait::refused);
        CHECK(g.check("layer") == CommWait::refused);
        CHECK(s.aborts == 1);
    }
    {   // an error returned by the call itself
        Script s;
        Guard g(FakeOps{&s}, 100);
        CHECK(g.settle(kRemoteError, "ncclGroupEnd") == CommWait::failed);
        CHECK(s.aborts == 1 && contains(g.reason(), "ncclGroupEnd: remote process exited"));
    }
    {   // in progress, then the communicator reports a peer's failure
        Script s;
        s.states = {kInProgress, kRemoteError};
        Guard g(FakeOps{&s}, 1000);
        CHECK(g.settle(kInProgress, "dispatch exchange") == CommWait::failed);
        CHECK(s.aborts == 1 && s.clock < 1000);
    }
    {   // the query itself failing counts as a failure
        Script s;
        s.query_status = 5;
        Guard g(FakeOps{&s}, 1000);
        CHECK(g.settle(kInProgress, "launch") == CommWait::failed);
        CHECK(s.aborts == 1);
    }
    {   // a zero bound is one millisecond, not "wait for ever"
        Script s;
        s.states = {kInProgress};
        Guard g(FakeOps{&s}, 0);
        CHECK(g.timeout_ms() == 1);
        CHECK(g.settle(kInProgress, "launch") == CommWait::timed_out);
    }
}

void check_cases() {
    {
        Script s;
        s.states = {kInProgress};   // a launch still settling is not an error
        Guard g(FakeOps{&s}, 100);
        CHECK(g.check("layer") == CommWait::ok && s.aborts == 0);
    }
    {
        Script s;
        s.states = {kRemoteError};
        Guard g(FakeOps{&s}, 100);
        CHECK(g.check("layer") == CommWait::failed && s.aborts == 1);
        CHECK(g.check("layer") == CommWait::refused && s.aborts == 1);
    }
}

void drain_cases() {
    {   // healthy: drains after a few polls
        Script s;
        s.stream_pending = 5;
        Guard g(FakeOps{&s}, 100);
        bool cuda_error = true;
        CHECK(g.drain("sync", &cuda_error) == CommWait::ok);
        CHECK(!cuda_error && s.aborts == 0 && s.stream_polls == 6);
    }
    {   // a peer that never answers: NCCL's kernels spin until the abort
        Script s;
        s.stream_pending = -1;
        Guard g(FakeOps{&s}, 50);
        CHECK(g.drain("sync") == CommWait::timed_out);
        CHECK(s.aborts == 1 && g.aborted() && contains(g.reason(), "sync: stream not drained after 50 ms"));
        CHECK(s.clock >= 50 && s.clock < 100);
    }
    {   // NCCL reports the failure before the deadline
        Script s;
        s.stream_pending = -1;
        s.states = {0, 0, kRemoteError};
        Guard g(FakeOps{&s}, 100000);
        CHECK(g.drain("sync") == CommWait::failed);
        CHECK(s.aborts == 1 && s.clock < 100);
    }
    {   // the stream stays busy even after the abort: the wait still ends
        Script s;
        s.stream_pending = -2;
        Guard g(FakeOps{&s}, 40);
        CHECK(g.drain("sync") == CommWait::stuck);
        CHECK(s.aborts == 1);
        CHECK(s.clock >= 80 && s.clock <= 80 + 2 * s.tick);
    }
    {   // a CUDA error is the caller's to report; the communicator is left alone
        Script s;
        s.stream_error = true;
        Guard g(FakeOps{&s}, 100);
        bool cuda_error = false;
        CHECK(g.drain("sync", &cuda_error) == CommWait::failed);
        CHECK(cuda_error && s.aborts == 0 && !g.aborted());
    }
    {   // after an abort a drain still waits (bounded) and reports the refusal
        Script s;
        s.states = {kRemoteError};
        Guard g(FakeOps{&s}, 100);
        CHECK(g.check("layer") == CommWait::failed);
        s.stream_pending = 3;
        CHECK(g.drain("sync") == CommWait::refused);
        CHECK(s.aborts == 1);
        s.stream_pending = -2;
        const uint64_t t0 = s.clock;
        CHECK(g.drain("sync") == CommWait::stuck);
        CHECK(s.clock - t0 >= 100 && s.clock - t0 <= 100 + s.tick);
    }
    {   // abort_now: no wait, once, and the reason is the caller's
        Script s;
        Guard g(FakeOps{&s}, 100);
        g.abort_now("peer 1 left");
        g.abort_now("again");
        CHECK(s.aborts == 1 && g.aborted() && g.reason() == "peer 1 left" && s.clock == 0);
        CHECK(g.drain("sync") == CommWait::refused);
    }
}

}  // namespace

int main() {
    settle_cases();
    check_cases();
    drain_cases();
    if (failures) {
        std::fprintf(stderr, "%d check(s) failed\n", failures);
        return 1;
    }
    std::printf("ep guard ok\n");
    return 0;
}
