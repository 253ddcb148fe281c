// profile.cuh — where the device time of a call goes.
//
// Every phase of the path is an NVTX range (free when no tool listens; ncu
// can filter on it with --nvtx-include) and, when profiling is switched on
// (k3xb_set_profiling), a pair of CUDA events on the stream the phase runs
// on. k3xb_get_profile resolves the pairs into device milliseconds per
// phase. This is the B200 counterpart of the reference's Profiler event
// list (runtime/include/k3x/profile.hpp:32-63) and of the CUDA events its
// backend records around each operation (backend_cuda.cu:4036-4038).
// Events are not recorded while a stream is being captured into a graph.
#pragma once

#include <nvtx3/nvToolsExt.h>

#include "common.cuh"

namespace k3xb {

const char* phase_name(int phase);

// Records the start of `phase` on ctx->stream (as it is now) and its end
// when the scope closes, on the same stream.
class PhaseScope {
public:
    PhaseScope(k3xb_ctx* ctx, int phase);
    ~PhaseScope() { end(); }
    PhaseScope(const PhaseScope&) = delete;
    PhaseScope& operator=(const PhaseScope&) = delete;
    // Closes the phase before the scope does (once).
    void end();

private:
    k3xb_ctx* ctx_;
    cudaStream_t stream_;
    int slot_ = -1;
    bool open_ = true;
};

// Frees the profiler of a context (k3xb_destroy).
void release_profiler(k3xb_ctx* ctx);

}  // namespace k3xb
