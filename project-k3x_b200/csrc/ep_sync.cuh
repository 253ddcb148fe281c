// ep_sync.cuh — device-side ordering of the expert-parallel exchange over
// peer memory (ep.cu): a grid tells the other ranks that its stores into
// their windows have landed, and a kernel waits, with a bound, until every
// rank has told it so.
//
// Flags hold a call counter (the epoch) and only grow, so they are never
// reset: a rank waits until flag[g] >= epoch for every rank g. Stores go to
// the flag with release semantics at system scope after a system-scope
// fence; loads are acquire at system scope.
#pragma once

#include <cstdint>

#include "common.cuh"
#include "tc.cuh"

namespace k3xb {
namespace eps {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// A wait gives up after this long; a healthy exchange waits microseconds.
constexpr uint64_t kWaitLimitNs = 5000000000ull;

}  // namespace eps

// Every thread of the CTA calls this at the end of its work. Each thread
// fences its own stores (to peers included) at system scope; the CTA's
// thread 0 then counts the CTA done, and the last CTA of the grid resets
// the counter and stores `epoch` into flag word `rank` at win[g] + flag_off
// for every rank g < world.
__device__ __forceinline__ void ep_signal_grid_done(uint32_t* done, uint8_t* const* win, uint64_t flag_off,
                                                    uint32_t rank, uint32_t world, uint32_t epoch) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t total = gridDim.x * gridDim.y * gridDim.z;
        if (atomicAdd(done, 1u) == total - 1u) {
            *done = 0u;   // the next call counts from zero (its kernel starts after this one ends)
            __threadfence_system();
            for (uint32_t g = 0; g < world; ++g)
                eps::st_release_sys(reinterpret_cast<uint32_t*>(win[g] + flag_off) + rank, epoch);
        }
    }
}

// One thread: waits until flags[g] >= epoch for every g < world. Returns
// false without waiting when an earlier wait of this rank gave up
// (*gave_up set), and false after the bound, setting *gave_up and the
// context's status word, so the host sees BACKEND_UNAVAILABLE at its next
// k3xb_sync and no later wait spends the bound again.
__device__ __forceinline__ bool ep_wait_flags(const uint32_t* flags, uint32_t world, uint32_t epoch,
                                              volatile int32_t* gave_up, int32_t* status) {
    if (*gave_up) return false;
    const uint64_t t0 = tc::globaltimer_ns();
    for (uint32_t g = 0; g < world; ++g) {
        while (static_cast<int32_t>(eps::ld_acquire_sys(flags + g) - epoch) < 0) {
            if (*gave_up) return false;
            if (tc::globaltimer_ns() - t0 > eps::kWaitLimitNs) {
                *gave_up = 1;
                atomicExch(status, K3XB_BACKEND_UNAVAILABLE);
                return false;
            }
            __nanosleep(128);
        }
    }
    return true;
}

}  // namespace k3xb
