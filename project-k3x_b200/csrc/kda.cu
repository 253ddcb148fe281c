// kda.cu — (d) KDA gated delta-rule recurrence over linear drafts and draft
// trees (official_kda.cpp:319-369 per node).
//
// In the reference's V-first layout S[h][v][k] every value row v evolves on
// its own: decayed = alpha (.) S[v]; pred = sum_k k_k * decayed_k; delta =
// (v_v - pred) * beta; S[v] = decayed + k * delta; o_v = sum_k q_k * S[v][k].
// One thread owns one value row and holds its d keys in registers; a block
// owns R rows of one head of one sequence. Per node the block stages the
// head's k, q and alpha = exp(log_decay) (computed once per key) in shared
// memory, and every thread then runs both dot products as sequential loops
// in key order: the reference's own float operation order (every product
// and sum rounded, no contraction), so on the same inputs the recurrence
// reproduces official_kda_cpu's arithmetic up to the exp of the decay. The
// state crosses HBM once each way per call (read coalesced through shared
// memory, written as 16-byte rows).
//
// Trees: nodes are visited in DFS preorder (computed on the host). When a
// node's parent is the node just visited, the state stays in registers;
// otherwise the schedule restarts from the prefix state (reloaded from the
// input, in L2) and replays the ancestors without output, so a block keeps
// no per-depth copies of the state and runs with full occupancy. Linear
// drafts never restart. Commit mode replays a root..node path and writes
// that node's state, bit-identical to what the tree pass computed for it;
// with a device commit array the pass writes the state after commit[s]
// instead, and stops there (linear drafts committed from device-side
// acceptance).
#include <atomic>

#include "common.cuh"
#include "kernels.cuh"

namespace k3xb {

namespace {

struct KdaArgs {
    const float* state;
    const int32_t* order;
    const int32_t* flags;   // per entry: 1 = restart from the prefix state, 2 = replay (no output)
    uint32_t visit, nodes, heads;
    const float *q, *k, *v, *log_decay, *beta;
    float* out;
    float* state_out;
    const int32_t* commit;
};

// shared memory: k, q, alpha [D], v [R], beta, then [R][D + 1] for staging
// the prefix rows
template <int D, int R>
constexpr size_t kda_smem_floats() {
    return 3 * D + R + 4 + static_cast<size_t>(R) * (D + 1);
}

// Four consecutive floats of shared memory (16-byte aligned), as a
// volatile load: ptxas keeps these loads in program order, so each group is
// fetched one group ahead of its use instead of all at once (the state
// already holds D registers per thread).
__device__ __forceinline__ float4 lds4(const float* p) {
    float4 v;
    asm volatile("ld.volatile.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))));
    return v;
}

template <int D, int R>
__global__ void __launch_bounds__(R) kda_rows_kernel(const KdaArgs a) {
    extern __shared__ float smem[];
    float* kk = smem;
    float* qq = kk + D;
    float* al = qq + D;
    float* vv = al + D;
    float* bsh = vv + R;
    float* stage = bsh + 4;
    constexpr int kChunks = D / R;
    const uint32_t t = threadIdx.x;
    const uint32_t h = blockIdx.x / kChunks, r0 = (blockIdx.x % kChunks) * R;
    const uint32_t s = blockIdx.y;
    if (h >= a.heads) return;
    const size_t hd = static_cast<size_t>(a.heads) * D;
    const size_t head_state = (static_cast<size_t>(s) * a.heads + h) * D * D + static_cast<size_t>(r0) * D;
    // the prefix rows, coalesced through shared memory, then each thread's row to registers
    const float* src = a.state + head_state;
    for (uint32_t i = t; i < static_cast<uint32_t>(R * D); i += R) stage[(i / D) * (D + 1) + i % D] = src[i];
    __syncthreads();
    float S[D];
#pragma unroll
    for (int i = 0; i < D; ++i) S[i] = stage[t * (D + 1) + i];
    float* dst = a.state_out ? a.state_out + head_state + static_cast<size_t>(t) * D : nullptr;
    auto save = [&]() {
#pragma unroll
        for (int i = 0; i < D; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(S[i], S[i + 1], S[i + 2], S[i + 3]);
    };
    // commit (device array, per sequence): state_out receives the state after
    // node commit[s] (the prefix state for -1) instead of after the last node
    const int32_t keep = a.commit ? a.commit[s] : INT32_MIN;
    if (dst && keep == -1) {
        save();
        return;
    }
    // the next entry's node vectors are loaded into registers while this
    // entry computes (one element of k, q, log_decay per key this thread
    // stages, v of its row, beta)
    constexpr int PER = D / R;
    float pk[PER], pq[PER], pl[PER], pv = 0.0f, pb = 0.0f;
    auto prefetch = [&](uint32_t it) {
        const int32_t n = a.order[it];
        const size_t base = (static_cast<size_t>(s) * a.nodes + n) * hd + static_cast<size_t>(h) * D;
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            pk[j] = a.k[base + t + j * R];
            pq[j] = a.q[base + t + j * R];
            pl[j] = a.log_decay[base + t + j * R];
        }
        pv = a.v[base + r0 + t];
        pb = t == 0 ? a.beta[(static_cast<size_t>(s) * a.nodes + n) * a.heads + h] : 0.0f;
    };
    if (a.visit) prefetch(0);
    for (uint32_t it = 0; it < a.visit; ++it) {
        const int32_t n = a.order[it];
        const int32_t fl = a.flags[it];
        if (fl & 1) {   // restart from the prefix state (this thread's row, 16-byte loads)
#pragma unroll
            for (int i = 0; i < D; i += 4) {
                const float4 q4 = *reinterpret_cast<const float4*>(src + static_cast<size_t>(t) * D + i);
                S[i] = q4.x; S[i + 1] = q4.y; S[i + 2] = q4.z; S[i + 3] = q4.w;
            }
        }
        const bool emit = !(fl & 2);
        const size_t base = (static_cast<size_t>(s) * a.nodes + n) * hd + static_cast<size_t>(h) * D;
        __syncthreads();   // the previous node's vectors are no longer read
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            kk[t + j * R] = pk[j];
            qq[t + j * R] = pq[j];
            al[t + j * R] = expf(pl[j]);
        }
        vv[t] = pv;
        if (t == 0) bsh[0] = pb;
        __syncthreads();
        if (it + 1 < a.visit) prefetch(it + 1);
        // the node vectors in groups of four keys, each group loaded one
        // group ahead of its sums
        float pred = 0.0f;
        {
            float4 na = lds4(al), nk = lds4(kk);
#pragma unroll
            for (int c = 0; c < D; c += 4) {
                const float4 ca = na, ck = nk;
                if (c + 4 < D) {
                    na = lds4(al + c + 4);
                    nk = lds4(kk + c + 4);
                }
                const float xa[4] = {ca.x, ca.y, ca.z, ca.w}, xk[4] = {ck.x, ck.y, ck.z, ck.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    S[c + i] = __fmul_rn(xa[i], S[c + i]);
                    pred = __fadd_rn(pred, __fmul_rn(xk[i], S[c + i]));
                }
            }
        }
        const float delta = __fmul_rn(__fsub_rn(vv[t], pred), bsh[0]);
        float o = 0.0f;
        {
            float4 nk = lds4(kk), nq = lds4(qq);
#pragma unroll
            for (int c = 0; c < D; c += 4) {
                const float4 ck = nk, cq = nq;
                if (c + 4 < D) {
                    nk = lds4(kk + c + 4);
                    nq = lds4(qq + c + 4);
                }
                const float xk[4] = {ck.x, ck.y, ck.z, ck.w}, xq[4] = {cq.x, cq.y, cq.z, cq.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    S[c + i] = __fadd_rn(S[c + i], __fmul_rn(xk[i], delta));
                    o = __fadd_rn(o, __fmul_rn(xq[i], S[c + i]));
                }
            }
        }
        if (a.out && emit) a.out[base + r0 + t] = o;
        if (dst && emit && n == keep) {   // the committed node: nothing after it is needed
            save();
            return;
        }
    }
    if (dst && !a.commit) save();
}

template <int D, int R>
int launch_rows(k3xb_ctx* ctx, const KdaArgs& a, uint32_t sequences) {
    const size_t smem = kda_smem_floats<D, R>() * sizeof(float);
    static std::atomic<uint64_t> configured{0};   // per template instance
    const int cst = configure_once(ctx, configured, [&]() -> int {
        K3XB_CUDA(ctx, cudaFuncSetAttribute(kda_rows_kernel<D, R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(smem)));
        // the whole unified L1 as shared memory, so two blocks (each ~68 KB
        // and 128 threads of ~230 registers) share an SM
        K3XB_CUDA(ctx, cudaFuncSetAttribute(kda_rows_kernel<D, R>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                            cudaSharedmemCarveoutMaxShared));
        return K3XB_OK;
    });
    if (cst) return cst;
    dim3 grid(a.heads * (D / R), sequences);
    kda_rows_kernel<D, R><<<grid, R, smem, ctx->stream>>>(a);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

}  // namespace

int launch_kda(k3xb_ctx* ctx, const float* state, const int32_t* order, const int32_t* depth,
               const int32_t* from_stack, uint32_t visit, uint32_t nodes, uint32_t sequences,
               uint32_t heads, uint32_t head_dim, const float* q, const float* k, const float* v,
               const float* log_decay, const float* beta, float* out, float* state_out,
               uint32_t levels, const int32_t* commit) {
    (void)depth;
    (void)levels;
    const KdaArgs a{state, order, from_stack, visit, nodes, heads, q, k, v, log_decay, beta, out, state_out, commit};
    switch (head_dim) {
        case 32: return launch_rows<32, 32>(ctx, a, sequences);
        case 64: return launch_rows<64, 64>(ctx, a, sequences);
        case 128: return launch_rows<128, 128>(ctx, a, sequences);
        default: return fail(ctx, K3XB_INVALID_EXTENT, "KDA head_dim must be 32, 64 or 128");
    }
}

}  // namespace k3xb
