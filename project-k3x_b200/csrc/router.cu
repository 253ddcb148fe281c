// router.cu — (a) router scores, Top-k selection and expert-major bucketing.
//
// Logits follow route_official_moe (runtime/src/official_moe.cpp:255-267):
// each (token, expert) logit is one FP64 chain summed in hidden order, so
// the float result is bit-identical to the reference. A bf16 x float
// product is exact in FP64, so fma(w, x, acc) rounds exactly like the
// reference's `sum += double(w) * x`. Chains are independent per (token,
// expert); a thread carries TOK of them for ILP. The kernel is bound by
// the FP64 dependency chain (H sequential adds), not by HBM: W_r is 5.5 MB
// at the released shape and is read once per TOK tokens from L2.
#include "common.cuh"
#include "kernels.cuh"

#include <cfloat>

namespace k3xb {

namespace {

constexpr int kTok = 8;

__global__ void __launch_bounds__(128) router_logits_kernel(
    const float* __restrict__ hidden, const uint16_t* __restrict__ W, uint32_t T,
    uint32_t H, uint32_t E, float* __restrict__ logits) {
    const uint32_t e = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t t0 = blockIdx.y * kTok;
    if (e >= E) return;
    double acc[kTok];
    const float* x[kTok];
#pragma unroll
    for (int j = 0; j < kTok; ++j) {
        acc[j] = 0.0;
        const uint32_t t = (t0 + j < T) ? t0 + j : T - 1;
        x[j] = hidden + static_cast<size_t>(t) * H;
    }
    const uint16_t* w = W + static_cast<size_t>(e) * H;
    const bool vec = (H % 8 == 0) && ((reinterpret_cast<uintptr_t>(W) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(hidden) & 15) == 0);
    uint32_t h = 0;
    if (vec) {
        for (; h < H; h += 8) {
            const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w + h));
            float wf[8];
            wf[0] = __uint_as_float(wv.x << 16); wf[1] = __uint_as_float(wv.x & 0xffff0000u);
            wf[2] = __uint_as_float(wv.y << 16); wf[3] = __uint_as_float(wv.y & 0xffff0000u);
            wf[4] = __uint_as_float(wv.z << 16); wf[5] = __uint_as_float(wv.z & 0xffff0000u);
            wf[6] = __uint_as_float(wv.w << 16); wf[7] = __uint_as_float(wv.w & 0xffff0000u);
#pragma unroll
            for (int j = 0; j < kTok; ++j) {
                const float4 a = __ldg(reinterpret_cast<const float4*>(x[j] + h));
                const float4 b = __ldg(reinterpret_cast<const float4*>(x[j] + h + 4));
                acc[j] = fma(static_cast<double>(wf[0]), static_cast<double>(a.x), acc[j]);
                acc[j] = fma(static_cast<double>(wf[1]), static_cast<double>(a.y), acc[j]);
                acc[j] = fma(static_cast<double>(wf[2]), static_cast<double>(a.z), acc[j]);
                acc[j] = fma(static_cast<double>(wf[3]), static_cast<double>(a.w), acc[j]);
                acc[j] = fma(static_cast<double>(wf[4]), static_cast<double>(b.x), acc[j]);
                acc[j] = fma(static_cast<double>(wf[5]), static_cast<double>(b.y), acc[j]);
                acc[j] = fma(static_cast<double>(wf[6]), static_cast<double>(b.z), acc[j]);
                acc[j] = fma(static_cast<double>(wf[7]), static_cast<double>(b.w), acc[j]);
            }
        }
    } else {
        for (; h < H; ++h) {
            const double wd = decode_bf16(w[h]);
#pragma unroll
            for (int j = 0; j < kTok; ++j) acc[j] = fma(wd, static_cast<double>(x[j][h]), acc[j]);
        }
    }
#pragma unroll
    for (int j = 0; j < kTok; ++j)
        if (t0 + j < T) logits[static_cast<size_t>(t0 + j) * E + e] = static_cast<float>(acc[j]);
}

// route_official_moe_logits (official_moe.cpp:211-245), one warp per token.
// sigmoid = 1 / (1 + expf(-l)) in float; expf is evaluated as the correctly
// rounded float(exp(double)).
constexpr int kMaxPerLane = 32;   // E <= 1024

__global__ void __launch_bounds__(256) topk_kernel(
    const float* __restrict__ logits, const float* __restrict__ correction, uint32_t T,
    uint32_t E, uint32_t K, uint32_t* __restrict__ ids, float* __restrict__ contrib,
    float* __restrict__ scores_out, int32_t* __restrict__ status) {
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
    const uint32_t lane = threadIdx.x % 32;
    if (warp >= T) return;
    const float* l = logits + static_cast<size_t>(warp) * E;
    float score[kMaxPerLane], adj[kMaxPerLane];
    bool bad = false;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
        const uint32_t e = lane + 32u * i;
        score[i] = 0.0f;
        adj[i] = -INFINITY;
        if (e < E) {
            const float x = l[e];
            const float c = correction[e];
            bad |= !isfinite(x) || !isfinite(c);
            const float ex = static_cast<float>(exp(-static_cast<double>(x)));
            score[i] = __fdiv_rn(1.0f, __fadd_rn(1.0f, ex));
            adj[i] = __fadd_rn(score[i], c);
            if (scores_out) scores_out[static_cast<size_t>(warp) * E + e] = score[i];
        }
    }
    if (__any_sync(0xffffffffu, bad)) {
        if (lane == 0) atomicExch(status, K3XB_INVALID_EXTENT);
        return;
    }
    uint32_t taken = 0;   // bit i: this lane's entry i is selected
    double total = 0.0;
    float sel_score[32];
    uint32_t sel_id[32];
    for (uint32_t slot = 0; slot < K; ++slot) {
        // lane-local best under (adjusted desc, index asc)
        float bv = -INFINITY;
        uint32_t bi = 0xffffffffu;
        float bs = 0.0f;
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) {
            const uint32_t e = lane + 32u * i;
            if (e < E && !(taken >> i & 1u)) {
                if (bi == 0xffffffffu || adj[i] > bv) { bv = adj[i]; bi = e; bs = score[i]; }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            const float os = __shfl_xor_sync(0xffffffffu, bs, o);
            const bool better = (oi != 0xffffffffu) &&
                                (bi == 0xffffffffu || ov > bv || (ov == bv && oi < bi));
            if (better) { bv = ov; bi = oi; bs = os; }
        }
        if ((bi % 32) == lane) taken |= 1u << (bi / 32);
        if (slot < 32) { sel_score[slot] = bs; sel_id[slot] = bi; }
        total += static_cast<double>(bs);   // slot order, like the reference
    }
    if (!isfinite(total) || total <= 0.0) {
        if (lane == 0) atomicExch(status, K3XB_INVALID_EXTENT);
        return;
    }
    if (lane == 0) {
        for (uint32_t slot = 0; slot < K && slot < 32; ++slot) {
            ids[static_cast<size_t>(warp) * K + slot] = sel_id[slot];
            contrib[static_cast<size_t>(warp) * K + slot] =
                static_cast<float>(static_cast<double>(sel_score[slot]) / total);
        }
    }
}

// build_expert_major_plan (expert_major.cpp:10-54) in one CTA. A bitmap
// bits[e][t/32] marks which tokens chose expert e; the in-group index of
// (t, e) is the number of set bits below t, which reproduces the
// reference's (token, slot) order inside a group. Groups are ranked by the
// first flat (token*k + slot) index that used them.
__global__ void __launch_bounds__(1024) plan_kernel(
    const uint32_t* __restrict__ ids, const float* __restrict__ contrib, uint32_t T,
    uint32_t K, uint32_t E, k3xb_plan plan) {
    extern __shared__ uint32_t smem[];
    const uint32_t words = (T + 31) / 32;
    uint32_t* bits = smem;                    // [E][words]
    uint32_t* first = bits + E * words;       // [E]
    uint32_t* count = first + E;              // [E]
    uint32_t* rank = count + E;               // [E]
    uint32_t* offs = rank + E;                // [E + 1] (by rank)
    __shared__ int32_t st;
    __shared__ uint32_t ngroups;
    const uint32_t tid = threadIdx.x, nt = blockDim.x;
    if (tid == 0) { st = K3XB_OK; ngroups = 0; }
    for (uint32_t i = tid; i < E * words; i += nt) bits[i] = 0;
    for (uint32_t i = tid; i < E; i += nt) { first[i] = 0xffffffffu; count[i] = 0; }
    __syncthreads();
    const uint32_t n = T * K;
    for (uint32_t f = tid; f < n; f += nt) {
        const uint32_t e = ids[f], t = f / K;
        if (e >= E) { st = K3XB_INVALID_EXTENT; continue; }
        if (!isfinite(contrib[f])) st = K3XB_INVALID_STATE;
        const uint32_t bit = 1u << (t % 32);
        const uint32_t old = atomicOr(&bits[e * words + t / 32], bit);
        if (old & bit) st = K3XB_INVALID_STATE;   // duplicate expert in a token
        atomicMin(&first[e], f);
    }
    __syncthreads();
    if (st != K3XB_OK) {
        if (tid == 0) { *plan.status = st; *plan.group_count = 0; plan.group_offset[0] = 0; }
        return;
    }
    for (uint32_t e = tid; e < E; e += nt) {
        uint32_t c = 0;
        for (uint32_t w = 0; w < words; ++w) c += __popc(bits[e * words + w]);
        count[e] = c;
        uint32_t r = 0;
        if (first[e] != 0xffffffffu) {
            for (uint32_t o = 0; o < E; ++o) r += first[o] < first[e];
            atomicAdd(&ngroups, 1u);
        }
        rank[e] = r;
    }
    __syncthreads();
    for (uint32_t e = tid; e < E; e += nt)
        if (first[e] != 0xffffffffu) {
            offs[rank[e]] = count[e];
            plan.group_expert[rank[e]] = e;
        }
    __syncthreads();
    if (tid == 0) {   // exclusive scan over <= E group sizes
        uint32_t run = 0;
        for (uint32_t g = 0; g < ngroups; ++g) {
            const uint32_t c = offs[g];
            offs[g] = run;
            run += c;
        }
        offs[ngroups] = run;
        *plan.group_count = ngroups;
        *plan.status = K3XB_OK;
    }
    __syncthreads();
    for (uint32_t g = tid; g <= ngroups; g += nt) plan.group_offset[g] = offs[g];
    for (uint32_t f = tid; f < n; f += nt) {
        const uint32_t e = ids[f], t = f / K, s = f % K;
        const uint32_t* row = bits + e * words;
        uint32_t local = __popc(row[t / 32] & ((1u << (t % 32)) - 1u));
        for (uint32_t w = 0; w < t / 32; ++w) local += __popc(row[w]);
        const uint32_t pos = offs[rank[e]] + local;
        plan.assign_token[pos] = t;
        plan.assign_slot[pos] = s;
        plan.assign_contrib[pos] = contrib[f];
    }
}

}  // namespace

size_t plan_smem_bytes(uint32_t T, uint32_t E) {
    const size_t words = (T + 31) / 32;
    return (static_cast<size_t>(E) * words + 4 * static_cast<size_t>(E) + 1) * sizeof(uint32_t);
}

int launch_router_logits(k3xb_ctx* ctx, const float* hidden, uint32_t T, uint32_t H,
                         const uint16_t* W, uint32_t E, float* logits) {
    dim3 grid((E + 127) / 128, (T + kTok - 1) / kTok);
    router_logits_kernel<<<grid, 128, 0, ctx->stream>>>(hidden, W, T, H, E, logits);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_topk(k3xb_ctx* ctx, const float* logits, const float* correction, uint32_t T,
                uint32_t E, uint32_t K, uint32_t* ids, float* contrib, float* scores,
                int32_t* status) {
    if (E > 32u * kMaxPerLane || K == 0 || K > E || K > 32)
        return fail(ctx, K3XB_INVALID_EXTENT, "route: need 0 < top_k <= min(32, experts) and experts <= 1024");
    const uint32_t warps_per_block = 8;
    topk_kernel<<<(T + warps_per_block - 1) / warps_per_block, 32 * warps_per_block, 0,
                  ctx->stream>>>(logits, correction, T, E, K, ids, contrib, scores, status);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_plan(k3xb_ctx* ctx, const uint32_t* ids, const float* contrib, uint32_t T,
                uint32_t K, uint32_t E, const k3xb_plan& plan) {
    const size_t smem = plan_smem_bytes(T, E);
    if (smem > 200 * 1024)
        return fail(ctx, K3XB_INVALID_EXTENT, "expert-major plan: experts * ceil(tokens/32) too large");
    static bool configured = false;
    if (!configured) {
        K3XB_CUDA(ctx, cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            200 * 1024));
        configured = true;
    }
    plan_kernel<<<1, 1024, smem, ctx->stream>>>(ids, contrib, T, K, E, plan);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

}  // namespace k3xb
