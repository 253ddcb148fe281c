// accept.cu — (e) acceptance over verify logits.
//
// Greedy (speculative.cpp:74-112 + model.cpp:1174-1176): one CTA per
// (sequence, position) streams one logits row once (HBM-bound) and keeps
// the first index of the maximum; a second tiny kernel compares targets
// with drafts per sequence and writes accepted/committed.
//
// Rejection sampling (no reference counterpart): the FP64 reductions use the
// canonical order of oracle/k3x_oracle.c — 1024 chunks of ceil(V/1024)
// consecutive entries summed sequentially (one thread each), 32 groups of 32
// chunk sums summed sequentially (one lane each), then the 32 group sums
// sequentially — so the GPU and the CPU restatement make the same decisions.
#include "common.cuh"
#include "kernels.cuh"

#include <cfloat>

namespace k3xb {

namespace {

constexpr int kArgmaxThreads = 512;
constexpr int kChunks = 1024;

// Combines two (value, index) candidates of a first-max argmax.
__device__ __forceinline__ void argmax_merge(float& bv, uint32_t& bi, float ov, uint32_t oi) {
    if (oi == 0xffffffffu) return;
    if (bi == 0xffffffffu || bv < ov || (!(ov < bv) && oi < bi)) { bv = ov; bi = oi; }
}

__global__ void __launch_bounds__(kArgmaxThreads) argmax_rows_kernel(
    const float* __restrict__ logits, uint32_t V, uint32_t* __restrict__ targets) {
    const size_t row = blockIdx.x;
    const float* l = logits + row * V;
    float bv = -INFINITY;
    uint32_t bi = 0xffffffffu;
    // strided scan keeps the first maximum of this thread's subsequence
    if ((V % 4 == 0) && ((reinterpret_cast<uintptr_t>(l) & 15) == 0)) {
        const float4* l4 = reinterpret_cast<const float4*>(l);
        for (uint32_t j = threadIdx.x; j < V / 4; j += blockDim.x) {
            const float4 x = __ldg(l4 + j);
            argmax_merge(bv, bi, x.x, 4 * j);
            argmax_merge(bv, bi, x.y, 4 * j + 1);
            argmax_merge(bv, bi, x.z, 4 * j + 2);
            argmax_merge(bv, bi, x.w, 4 * j + 3);
        }
    } else {
        for (uint32_t j = threadIdx.x; j < V; j += blockDim.x) argmax_merge(bv, bi, __ldg(l + j), j);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        argmax_merge(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
    __shared__ float sv[kArgmaxThreads / 32];
    __shared__ uint32_t si[kArgmaxThreads / 32];
    if (threadIdx.x % 32 == 0) { sv[threadIdx.x / 32] = bv; si[threadIdx.x / 32] = bi; }
    __syncthreads();
    if (threadIdx.x < 32) {
        bv = threadIdx.x < kArgmaxThreads / 32 ? sv[threadIdx.x] : -INFINITY;
        bi = threadIdx.x < kArgmaxThreads / 32 ? si[threadIdx.x] : 0xffffffffu;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            argmax_merge(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
        if (threadIdx.x == 0) targets[row] = bi;
    }
}

__global__ void greedy_accept_kernel(const uint32_t* __restrict__ targets,
                                     const uint32_t* __restrict__ drafts, uint32_t S, uint32_t p,
                                     uint32_t* accepted, uint32_t* committed, uint32_t* count) {
    const uint32_t s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= S) return;
    const uint32_t* t = targets + static_cast<size_t>(s) * (p + 1);
    const uint32_t* d = drafts + static_cast<size_t>(s) * p;
    uint32_t* c = committed + static_cast<size_t>(s) * (p + 1);
    uint32_t a = 0;
    while (a < p && d[a] == t[a]) { c[a] = d[a]; ++a; }
    c[a] = t[a];   // the target at the first mismatch, or the bonus token
    accepted[s] = a;
    count[s] = a + 1;
}

// ---------------------------------------------------------------------------
// rejection sampling

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ double uniform01(uint64_t seed, uint64_t seq, uint64_t pos, uint64_t purpose) {
    uint64_t key = splitmix64(seed);
    key = splitmix64(key ^ seq);
    key = splitmix64(key ^ pos);
    key = splitmix64(key ^ purpose);
    return static_cast<double>(key >> 11) * 0x1.0p-53;
}

struct RowSums {
    double chunk[kChunks];
    double group[32];
    double total;
};

__device__ float block_max(const float* l, uint32_t V, float* red) {
    float m = -INFINITY;
    for (uint32_t j = threadIdx.x; j < V; j += blockDim.x) m = fmaxf(m, l[j]);
    m = warp_max(m);
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        m = red[threadIdx.x];
        m = warp_max(m);
        if (threadIdx.x == 0) red[32] = m;
    }
    __syncthreads();
    const float r = red[32];
    __syncthreads();
    return r;
}

__device__ __forceinline__ double softmax_weight(float l, double m, double tau) {
    return exp(__ddiv_rn(__dsub_rn(static_cast<double>(l), m), tau));
}

// Canonical sums of w_j = exp((l_j - max)/tau) (blockDim.x == kChunks).
__device__ void reduce_softmax(const float* l, uint32_t V, double m, double tau, RowSums& s) {
    const uint32_t len = (V + kChunks - 1) / kChunks;
    const uint32_t lo = threadIdx.x * len, hi = min(lo + len, V);
    double acc = 0.0;
    for (uint32_t j = lo; j < hi; ++j) acc = __dadd_rn(acc, softmax_weight(l[j], m, tau));
    s.chunk[threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        double g = 0.0;
        for (int c = 0; c < 32; ++c) g = __dadd_rn(g, s.chunk[threadIdx.x * 32 + c]);
        s.group[threadIdx.x] = g;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int g = 0; g < 32; ++g) t = __dadd_rn(t, s.group[g]);
        s.total = t;
    }
    __syncthreads();
}

// Per (sequence, draft position i < p): p_i(d_i) and q_i(d_i).
__global__ void __launch_bounds__(kChunks) rejection_probs_kernel(
    const float* __restrict__ tl, const float* __restrict__ dl, const uint32_t* __restrict__ drafts,
    uint32_t p, uint32_t V, double tau, double* __restrict__ pd, double* __restrict__ qd) {
    __shared__ RowSums sums;
    __shared__ float red[33];
    const uint32_t s = blockIdx.y, i = blockIdx.x;
    const float* lp = tl + (static_cast<size_t>(s) * (p + 1) + i) * V;
    const float* lq = dl + (static_cast<size_t>(s) * p + i) * V;
    const uint32_t d = drafts[static_cast<size_t>(s) * p + i];
    const double mp = block_max(lp, V, red);
    reduce_softmax(lp, V, mp, tau, sums);
    if (threadIdx.x == 0) pd[static_cast<size_t>(s) * p + i] = __ddiv_rn(softmax_weight(lp[d], mp, tau), sums.total);
    __syncthreads();
    const double mq = block_max(lq, V, red);
    reduce_softmax(lq, V, mq, tau, sums);
    if (threadIdx.x == 0) qd[static_cast<size_t>(s) * p + i] = __ddiv_rn(softmax_weight(lq[d], mq, tau), sums.total);
}

// Sampling search of oracle/k3x_oracle.c:rs_sample, run by thread 0; w(j)
// recomputes an entry's weight.
template <typename W>
__device__ uint32_t canonical_sample(const RowSums& s, uint32_t V, double target, W w) {
    const uint32_t len = (V + kChunks - 1) / kChunks;
    double run = 0.0;
    int g_sel = 32, g_last = 0;
    for (int g = 0; g < 32; ++g) {
        if (s.group[g] > 0.0) g_last = g;
        const double next = __dadd_rn(run, s.group[g]);
        if (next > target) { g_sel = g; break; }
        run = next;
    }
    if (g_sel == 32) {
        g_sel = g_last;
        run = 0.0;
        for (int g = 0; g < g_sel; ++g) run = __dadd_rn(run, s.group[g]);
    }
    int c_sel = kChunks, c_last = g_sel * 32;
    for (int c = g_sel * 32; c < g_sel * 32 + 32; ++c) {
        if (s.chunk[c] > 0.0) c_last = c;
        const double next = __dadd_rn(run, s.chunk[c]);
        if (next > target) { c_sel = c; break; }
        run = next;
    }
    if (c_sel == kChunks) {
        c_sel = c_last;
        run = 0.0;
        for (int g = 0; g < g_sel; ++g) run = __dadd_rn(run, s.group[g]);
        for (int c = g_sel * 32; c < c_sel; ++c) run = __dadd_rn(run, s.chunk[c]);
    }
    const uint32_t lo = c_sel * len, hi = min(lo + len, V);
    uint32_t j_last = lo;
    for (uint32_t j = lo; j < hi; ++j) {
        const double x = w(j);
        if (x > 0.0) j_last = j;
        const double next = __dadd_rn(run, x);
        if (next > target) return j;
        run = next;
    }
    return j_last;
}

__global__ void __launch_bounds__(kChunks) rejection_decide_kernel(
    const float* __restrict__ tl, const float* __restrict__ dl, const uint32_t* __restrict__ drafts,
    const double* __restrict__ pd, const double* __restrict__ qd, uint32_t p, uint32_t V, double tau,
    uint64_t seed, uint64_t seq_base, uint32_t* accepted, uint32_t* committed, uint32_t* count) {
    __shared__ RowSums sp, sq, sr;
    __shared__ float red[33];
    __shared__ uint32_t first_reject;
    const uint32_t s = blockIdx.x;
    const uint64_t seq = seq_base + s;
    const uint32_t* d = drafts + static_cast<size_t>(s) * p;
    uint32_t* c = committed + static_cast<size_t>(s) * (p + 1);
    if (threadIdx.x == 0) {
        uint32_t i = 0;
        for (; i < p; ++i) {
            const double u = uniform01(seed, seq, i, 0);
            if (!(__dmul_rn(u, qd[static_cast<size_t>(s) * p + i]) < pd[static_cast<size_t>(s) * p + i])) break;
            c[i] = d[i];
        }
        first_reject = i;
        accepted[s] = i;
        count[s] = i + 1;
    }
    __syncthreads();
    const uint32_t i = first_reject;
    const float* lp = tl + (static_cast<size_t>(s) * (p + 1) + i) * V;
    const double mp = block_max(lp, V, red);
    reduce_softmax(lp, V, mp, tau, sp);
    const double u2 = uniform01(seed, seq, i, 1);
    if (i == p) {   // all accepted: bonus token from p_p
        if (threadIdx.x == 0)
            c[p] = canonical_sample(sp, V, __dmul_rn(u2, sp.total),
                                    [&](uint32_t j) { return softmax_weight(lp[j], mp, tau); });
        return;
    }
    const float* lq = dl + (static_cast<size_t>(s) * p + i) * V;
    const double mq = block_max(lq, V, red);
    reduce_softmax(lq, V, mq, tau, sq);
    const double zp = sp.total, zq = sq.total;
    auto resid = [&](uint32_t j) {
        const double diff = __dsub_rn(__ddiv_rn(softmax_weight(lp[j], mp, tau), zp),
                                      __ddiv_rn(softmax_weight(lq[j], mq, tau), zq));
        return diff > 0.0 ? diff : 0.0;
    };
    {   // canonical sums of the residual
        const uint32_t len = (V + kChunks - 1) / kChunks;
        const uint32_t lo = threadIdx.x * len, hi = min(lo + len, V);
        double acc = 0.0;
        for (uint32_t j = lo; j < hi; ++j) acc = __dadd_rn(acc, resid(j));
        sr.chunk[threadIdx.x] = acc;
        __syncthreads();
        if (threadIdx.x < 32) {
            double g = 0.0;
            for (int cc = 0; cc < 32; ++cc) g = __dadd_rn(g, sr.chunk[threadIdx.x * 32 + cc]);
            sr.group[threadIdx.x] = g;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            double t = 0.0;
            for (int g = 0; g < 32; ++g) t = __dadd_rn(t, sr.group[g]);
            sr.total = t;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        c[i] = sr.total > 0.0
                   ? canonical_sample(sr, V, __dmul_rn(u2, sr.total), resid)
                   : canonical_sample(sp, V, __dmul_rn(u2, sp.total),
                                      [&](uint32_t j) { return softmax_weight(lp[j], mp, tau); });
    }
}

// Next round's anchor of each sequence: its last committed token
// (committed[s][count[s] - 1], the target token after the accepted drafts).
__global__ void next_round_kernel(const uint32_t* __restrict__ committed, const uint32_t* __restrict__ count,
                                  uint32_t S, uint32_t stride, uint32_t* __restrict__ anchors) {
    const uint32_t s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= S) return;
    const uint32_t n = count[s];
    anchors[s] = committed[static_cast<size_t>(s) * stride + (n ? min(n, stride) - 1 : 0)];
}

}  // namespace

int launch_next_anchor(k3xb_ctx* ctx, const uint32_t* committed, const uint32_t* count, uint32_t S, uint32_t stride,
                       uint32_t* anchors) {
    next_round_kernel<<<(S + 127) / 128, 128, 0, ctx->stream>>>(committed, count, S, stride, anchors);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_accept_greedy(k3xb_ctx* ctx, const float* logits, const uint32_t* drafts, uint32_t S,
                         uint32_t p, uint32_t V, uint32_t* targets, uint32_t* accepted,
                         uint32_t* committed, uint32_t* count) {
    argmax_rows_kernel<<<S * (p + 1), kArgmaxThreads, 0, ctx->stream>>>(logits, V, targets);
    K3XB_LAUNCHED(ctx);
    greedy_accept_kernel<<<(S + 127) / 128, 128, 0, ctx->stream>>>(targets, drafts, S, p, accepted,
                                                                   committed, count);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_accept_rejection(k3xb_ctx* ctx, const float* tl, const float* dl, const uint32_t* drafts,
                            uint32_t S, uint32_t p, uint32_t V, float temperature, uint64_t seed,
                            uint64_t seq_base, double* pd, double* qd, uint32_t* accepted,
                            uint32_t* committed, uint32_t* count) {
    const double tau = temperature;
    if (p) {
        rejection_probs_kernel<<<dim3(p, S), kChunks, 0, ctx->stream>>>(tl, dl, drafts, p, V, tau, pd, qd);
        K3XB_LAUNCHED(ctx);
    }
    rejection_decide_kernel<<<S, kChunks, 0, ctx->stream>>>(tl, dl, drafts, pd, qd, p, V, tau, seed,
                                                            seq_base, accepted, committed, count);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

}  // namespace k3xb
