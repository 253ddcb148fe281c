// ep_guard.hpp — bounded waits on the expert-parallel communicator.
//
// A rank that dies or stops answering must not leave the others waiting
// for ever: in NCCL's kernels (a peer that never posts its half of a
// send/recv), in ncclGroupEnd (the first exchange with a peer sets up the
// connection with it) or in communicator creation. Every such wait here has
// a deadline. When it passes, or when NCCL reports an asynchronous error,
// the communicator is aborted (ncclCommAbort makes NCCL's kernels in flight
// return), the stream drains, and the context records why; the context's
// single-GPU entry points keep working, the expert-parallel ones refuse
// until the communicator is made again.
//
// The logic is host code over an `Ops` type, so it is tested on the CPU with
// a scripted communicator (tests/cpp/ep_guard_check.cpp) and used in ep.cu
// with NCCL and the CUDA stream:
//   int  async_error(int* state)  ncclCommGetAsyncError: call status, *state
//                                 = the communicator's state
//   int  abort()                  ncclCommAbort
//   int  stream_query()           0 drained, 1 work pending, -1 CUDA error
//   uint64_t now_ms()             a monotonic clock
//   void pause(uint32_t polls)    back off between polls
//   const char* describe(int r)   ncclGetErrorString
// Codes are nccl.h's ncclResult_t values (ep.cu checks them against it).
#pragma once

#include <cstdint>
#include <string>
#include <utility>

namespace k3xb {

constexpr int kCommSuccess = 0;      // ncclSuccess
constexpr int kCommInProgress = 7;   // ncclInProgress (nonblocking communicators)

// ok; failed (an error, now aborted); timed_out (the bound passed, now
// aborted); refused (aborted earlier); stuck (the stream still busy a bound
// after the abort).
enum class CommWait { ok, failed, timed_out, refused, stuck };

template <class Ops>
class CommGuard {
public:
    CommGuard(Ops ops, uint32_t timeout_ms) : ops_(std::move(ops)), timeout_ms_(timeout_ms ? timeout_ms : 1) {}

    bool aborted() const { return aborted_; }
    const std::string& reason() const { return reason_; }
    uint32_t timeout_ms() const { return timeout_ms_; }
    Ops& ops() { return ops_; }

    // After a communicator call that returned `r` (creation, ncclGroupEnd):
    // success as is; ncclInProgress (a nonblocking communicator) is polled
    // until it settles or the deadline passes; an error aborts.
    CommWait settle(int r, const char* what) {
        if (aborted_) return CommWait::refused;
        const uint64_t t0 = ops_.now_ms();
        for (uint32_t polls = 0; r == kCommInProgress; ++polls) {
            if (ops_.now_ms() - t0 >= timeout_ms_)
                return abort_with(CommWait::timed_out, std::string(what) + ": still in progress after " +
                                                           std::to_string(timeout_ms_) + " ms");
            ops_.pause(polls);
            int state = kCommSuccess;
            const int q = ops_.async_error(&state);
            r = q != kCommSuccess ? q : state;
        }
        if (r != kCommSuccess) return abort_with(CommWait::failed, std::string(what) + ": " + ops_.describe(r));
        return CommWait::ok;
    }

    // Non-waiting look at the communicator: an error reported since the last
    // call (a peer's failure seen by NCCL's proxy thread) aborts.
    CommWait check(const char* what) {
        if (aborted_) return CommWait::refused;
        int state = kCommSuccess;
        const int q = ops_.async_error(&state);
        const int r = q != kCommSuccess ? q : state;
        if (r != kCommSuccess && r != kCommInProgress)
            return abort_with(CommWait::failed, std::string(what) + ": " + ops_.describe(r));
        return CommWait::ok;
    }

    // Ends the communicator at once, without its peers (one of them is known
    // to be gone); later calls are refused.
    void abort_now(std::string reason) { abort_with(CommWait::failed, std::move(reason)); }

    // Waits for the stream (the exchanges' NCCL kernels included) to drain
    // before the deadline, watching the communicator meanwhile. On expiry or
    // an asynchronous error the communicator is aborted, which ends NCCL's
    // kernels, and the stream gets one more period to drain (else: stuck).
    // `stream_error` tells a CUDA error (the caller reports it) from the
    // other outcomes.
    CommWait drain(const char* what, bool* stream_error = nullptr) {
        if (stream_error) *stream_error = false;
        CommWait result = aborted_ ? CommWait::refused : CommWait::ok;
        uint64_t t0 = ops_.now_ms();
        for (uint32_t polls = 0;; ++polls) {
            const int q = ops_.stream_query();
            if (q == 0) return result;
            if (q < 0) {
                if (stream_error) *stream_error = true;
                return CommWait::failed;
            }
            if (!aborted_) {
                int state = kCommSuccess;
                const int a = ops_.async_error(&state);
                const int r = a != kCommSuccess ? a : state;
                if (r != kCommSuccess && r != kCommInProgress) {
                    result = abort_with(CommWait::failed, std::string(what) + ": " + ops_.describe(r));
                    t0 = ops_.now_ms();
                    continue;
                }
            }
            if (ops_.now_ms() - t0 >= timeout_ms_) {
                if (aborted_) return CommWait::stuck;
                result = abort_with(CommWait::timed_out, std::string(what) + ": stream not drained after " +
                                                             std::to_string(timeout_ms_) + " ms");
                t0 = ops_.now_ms();
                continue;
            }
            ops_.pause(polls);
        }
    }

private:
    CommWait abort_with(CommWait why, std::string reason) {
        if (!aborted_) {
            aborted_ = true;
            reason_ = std::move(reason);
            ops_.abort();
        }
        return why;
    }

    Ops ops_;
    uint32_t timeout_ms_;
    bool aborted_ = false;
    std::string reason_;
};

}  // namespace k3xb
