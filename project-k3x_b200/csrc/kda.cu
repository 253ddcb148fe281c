// kda.cu — (d) KDA gated delta-rule recurrence over linear drafts and draft
// trees (official_kda.cpp:319-369 per node).
//
// In the reference's V-first layout S[h][v][k] every value row v evolves on
// its own: decayed = alpha (.) S[v]; pred = <k, decayed>; delta = (v_v -
// pred) * beta; S[v] = decayed + k * delta; o_v = <q, S[v]>. One warp owns
// ROWS consecutive value rows of one head; lane l holds keys
// [l*KPL, l*KPL+KPL) of each row in registers, so the state is streamed from
// HBM once (coalesced 128*KPL-byte rows), both dot products are warp
// shuffles, and q/k/alpha of a node are read once per warp for ROWS rows.
//
// Trees: nodes are visited in DFS preorder (computed on the host). When a
// node's parent is the node just visited, the state stays in registers;
// otherwise the parent's state is reloaded from a per-warp shared-memory
// stack indexed by depth (the prefix state is depth 0). Linear drafts never
// touch the stack. Commit mode replays a root..node path and writes that
// node's state, bit-identical to what the tree pass computed for it; with a
// device commit array the pass writes the state after commit[s] instead
// (linear drafts committed from device-side acceptance).
#include "common.cuh"
#include "kernels.cuh"

namespace k3xb {

namespace {

constexpr int kRows = 2;   // value rows per warp

template <int KPL>
__global__ void __launch_bounds__(128) kda_tree_kernel(
    const float* __restrict__ state, const int32_t* __restrict__ order,
    const int32_t* __restrict__ depth, const int32_t* __restrict__ from_stack, uint32_t visit,
    uint32_t nodes, uint32_t heads, const float* __restrict__ q, const float* __restrict__ k,
    const float* __restrict__ v, const float* __restrict__ log_decay,
    const float* __restrict__ beta, float* __restrict__ out, float* __restrict__ state_out,
    uint32_t levels, const int32_t* __restrict__ commit) {
    constexpr int D = 32 * KPL;
    extern __shared__ float stack[];   // [warps][levels][kRows][D]; level 0 = prefix
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t s = blockIdx.y;
    const uint32_t row_global = (blockIdx.x * (blockDim.x / 32) + warp) * kRows;   // h*D + v
    if (row_global >= heads * D) return;
    const uint32_t h = row_global / D, v0 = row_global % D;
    const size_t hd = static_cast<size_t>(heads) * D;
    float* my_stack = stack + static_cast<size_t>(warp) * levels * kRows * D;

    float st[kRows][KPL];
    const float* src = state + static_cast<size_t>(s) * heads * D * D + static_cast<size_t>(h) * D * D;
    float* dst = state_out ? state_out + static_cast<size_t>(s) * heads * D * D + static_cast<size_t>(h) * D * D
                           : nullptr;
    // commit (device array, per sequence): state_out receives the state after
    // node commit[s] (the prefix state for -1) instead of after the last node
    const int32_t keep = commit ? commit[s] : INT32_MIN;
    auto save = [&]() {
#pragma unroll
        for (int r = 0; r < kRows; ++r)
#pragma unroll
            for (int i = 0; i < KPL; ++i) dst[static_cast<size_t>(v0 + r) * D + lane * KPL + i] = st[r][i];
    };
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
        for (int i = 0; i < KPL; ++i) {
            st[r][i] = src[static_cast<size_t>(v0 + r) * D + lane * KPL + i];
            if (levels) my_stack[r * D + lane * KPL + i] = st[r][i];
        }
    if (dst && keep == -1) save();

    for (uint32_t it = 0; it < visit; ++it) {
        const int32_t n = order[it];
        const int32_t dn = depth[it];
        if (from_stack[it]) {
#pragma unroll
            for (int r = 0; r < kRows; ++r)
#pragma unroll
                for (int i = 0; i < KPL; ++i)
                    st[r][i] = my_stack[(static_cast<size_t>(dn - 1) * kRows + r) * D + lane * KPL + i];
        }
        const size_t base = (static_cast<size_t>(s) * nodes + n) * hd + static_cast<size_t>(h) * D;
        float kk[KPL], qq[KPL], al[KPL];
#pragma unroll
        for (int i = 0; i < KPL; ++i) {
            kk[i] = k[base + lane * KPL + i];
            qq[i] = q[base + lane * KPL + i];
            al[i] = expf(log_decay[base + lane * KPL + i]);
        }
        const float b = beta[(static_cast<size_t>(s) * nodes + n) * heads + h];
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
            float part = 0.0f;
#pragma unroll
            for (int i = 0; i < KPL; ++i) {
                st[r][i] = __fmul_rn(al[i], st[r][i]);
                part = __fadd_rn(part, __fmul_rn(kk[i], st[r][i]));
            }
            const float pred = warp_sum(part);
            const float delta = __fmul_rn(__fsub_rn(v[base + v0 + r], pred), b);
            float o = 0.0f;
#pragma unroll
            for (int i = 0; i < KPL; ++i) {
                st[r][i] = __fadd_rn(st[r][i], __fmul_rn(kk[i], delta));
                o = __fadd_rn(o, __fmul_rn(qq[i], st[r][i]));
            }
            o = warp_sum(o);
            if (out && lane == 0) out[base + v0 + r] = o;
            if (static_cast<uint32_t>(dn) < levels)
#pragma unroll
                for (int i = 0; i < KPL; ++i)
                    my_stack[(static_cast<size_t>(dn) * kRows + r) * D + lane * KPL + i] = st[r][i];
        }
        if (dst && n == keep) save();
    }
    if (dst && !commit) save();
}

}  // namespace

int launch_kda(k3xb_ctx* ctx, const float* state, const int32_t* order, const int32_t* depth,
               const int32_t* from_stack, uint32_t visit, uint32_t nodes, uint32_t sequences,
               uint32_t heads, uint32_t head_dim, const float* q, const float* k, const float* v,
               const float* log_decay, const float* beta, float* out, float* state_out,
               uint32_t levels, const int32_t* commit) {
    const uint32_t warps = 4;
    const size_t smem = static_cast<size_t>(warps) * levels * kRows * head_dim * sizeof(float);
    if (smem > 200 * 1024) return fail(ctx, K3XB_INVALID_EXTENT, "KDA draft tree too deep for the state stack");
    const uint32_t rows = heads * head_dim;
    dim3 grid((rows / kRows + warps - 1) / warps, sequences);
    switch (head_dim) {
#define K3XB_KDA_CASE(KPL)                                                                      \
    case 32 * KPL:                                                                              \
        K3XB_CUDA(ctx, cudaFuncSetAttribute(kda_tree_kernel<KPL>,                               \
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024)); \
        kda_tree_kernel<KPL><<<grid, 32 * warps, smem, ctx->stream>>>(                          \
            state, order, depth, from_stack, visit, nodes, heads, q, k, v, log_decay, beta, out, \
            state_out, levels, commit);                                                    \
        break;
        K3XB_KDA_CASE(1)
        K3XB_KDA_CASE(2)
        K3XB_KDA_CASE(4)
#undef K3XB_KDA_CASE
        default:
            return fail(ctx, K3XB_INVALID_EXTENT, "KDA head_dim must be 32, 64 or 128");
    }
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

}  // namespace k3xb
