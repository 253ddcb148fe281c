// attnres.cu — block attention residual over many sources: the depth
// attention of the K3 model's token graph (runtime/src/model.cpp:645-666;
// the torch form is reference/k3x_ref/attn_res.py:9-23). Per row t the
// values are the block sources in push order, then the prefix:
//
//   key_d   = rms_norm(value_d, norm, eps)       ops.cpp:10-18 (FP64 squares,
//                                                float inverse, (v*inv)*w)
//   score_d = key_d . projection
//   p       = softmax(score) over the depths      (max, exp, sequential sum)
//   out     = sum_d p_d * value_d                 (float, depth order from 0)
//
// One CTA per row, one pass over the values for the scores and one for the
// output. The squares and sum(v * norm * proj) of each depth are FP64 sums;
// the score is float(inv * that sum), where the reference rounds every key
// element and product to float and chains float adds, so scores differ
// from the reference's by about its own float rounding error. The softmax
// and the output sum follow the reference's operation order exactly. The
// output pass reads every depth's row again, mostly from L2 (a CTA's rows
// are read moments before).
#include "common.cuh"
#include "kernels.cuh"

namespace k3xb {

namespace {

constexpr uint32_t kAttnResThreads = 256;
// norm * projection held in shared memory: H <= 48K floats
constexpr size_t kBlockAttnResMaxSmem = 192u << 10;

// Correctly rounded expf through the double exp (glibc's expf, which the
// reference calls through std::exp(float), agrees except on ~0.06% of
// inputs, by one ulp).
__device__ __forceinline__ float expf_cr(float x) { return static_cast<float>(exp(static_cast<double>(x))); }

__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// VEC: H % 4 == 0 and every base pointer 16-byte aligned, so each thread
// moves float4s. Phase 1 streams one depth at a time with up to kI loads of
// it in flight per thread and no barrier between depths: each warp leaves
// its partial sums of a depth in smem and moves on. The threads of depth d
// then add the 8 warp partials in warp order (deterministic). The output
// sweep reads kD depths per round trip, from L2.
constexpr uint32_t kWarps = kAttnResThreads / 32;
constexpr uint32_t kI = 8;   // phase 1: chunks of a depth in flight per thread
constexpr uint32_t kO = 4;   // output sweep: chunks per thread ...
constexpr uint32_t kD = 2;   // ... times depths per round trip

template <bool VEC>
__global__ void __launch_bounds__(kAttnResThreads, 4) block_attnres_kernel(
    const float* __restrict__ prefix, const float* __restrict__ sources, uint32_t S, uint32_t T, uint32_t H,
    const float* __restrict__ norm, const float* __restrict__ proj, float eps, float* __restrict__ out) {
    extern __shared__ __align__(16) unsigned char attnres_smem[];
    float* wp = reinterpret_cast<float*>(attnres_smem);   // [H]: norm * projection
    __shared__ double part[kBlockAttnResMaxDepth][2][kWarps];
    __shared__ float prob[kBlockAttnResMaxDepth];
    constexpr uint32_t W = VEC ? 4u : 1u;
    const uint32_t t = blockIdx.x, lane = threadIdx.x % 32, warp = threadIdx.x / 32;
    const uint32_t n = H / W;
    auto row = [&](uint32_t d) -> const float* {
        return d < S ? sources + (static_cast<size_t>(d) * T + t) * H : prefix + static_cast<size_t>(t) * H;
    };
    auto ld = [](const float* p, uint32_t i, float (&v)[W]) {
        if constexpr (VEC) {
            const float4 q = __ldg(reinterpret_cast<const float4*>(p) + i);
            v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
        } else {
            v[0] = __ldg(p + i);
        }
    };
    // shared-memory row: plain loads
    auto lds = [](const float* p, uint32_t i, float (&v)[W]) {
        if constexpr (VEC) {
            const float4 q = reinterpret_cast<const float4*>(p)[i];
            v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
        } else {
            v[0] = p[i];
        }
    };
    for (uint32_t i = threadIdx.x; i < H; i += kAttnResThreads) wp[i] = __fmul_rn(__ldg(norm + i), __ldg(proj + i));
    __syncthreads();
    // phase 1: squares and the score's dot product, each in FP64. Depths
    // are read last to first, so the first ones the output sum needs are the
    // most recently cached in L2.
    for (uint32_t d = S + 1; d-- > 0;) {
        const float* v = row(d);
        double sq = 0.0, dot = 0.0;
        for (uint32_t i0 = threadIdx.x; i0 < n; i0 += kI * kAttnResThreads) {
            float x[kI][W];
#pragma unroll
            for (uint32_t j = 0; j < kI; ++j)
                if (i0 + j * kAttnResThreads < n) ld(v, i0 + j * kAttnResThreads, x[j]);
#pragma unroll
            for (uint32_t j = 0; j < kI; ++j) {
                if (i0 + j * kAttnResThreads >= n) break;
                float c[W];
                lds(wp, i0 + j * kAttnResThreads, c);
#pragma unroll
                for (uint32_t k = 0; k < W; ++k) {
                    const double xd = static_cast<double>(x[j][k]);
                    sq += xd * xd;
                    dot += xd * static_cast<double>(c[k]);
                }
            }
        }
        sq = warp_sum_f64(sq);
        dot = warp_sum_f64(dot);
        if (lane == 0) {
            part[d][0][warp] = sq;
            part[d][1][warp] = dot;
        }
    }
    __syncthreads();
    // score_d = float(inv_d * sum (v * norm * proj)); inv_d as ops.cpp:14:
    // 1 / sqrt(float(squares / n) + eps)
    if (threadIdx.x <= S) {
        const uint32_t d = threadIdx.x;
        double sq = 0.0, dot = 0.0;
#pragma unroll
        for (uint32_t w = 0; w < kWarps; ++w) {
            sq += part[d][0][w];
            dot += part[d][1][w];
        }
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(sq / H), eps)));
        prob[d] = static_cast<float>(static_cast<double>(inv) * dot);
    }
    __syncthreads();
    // model.cpp:657-659: max, exp(score - max) and their float sum in depth
    // order; probability = exp / sum
    if (threadIdx.x == 0) {
        float m = prob[0];
        for (uint32_t d = 1; d <= S; ++d) m = fmaxf(m, prob[d]);
        float den = 0.0f;
        for (uint32_t d = 0; d <= S; ++d) {
            prob[d] = expf_cr(__fsub_rn(prob[d], m));
            den = __fadd_rn(den, prob[d]);
        }
        for (uint32_t d = 0; d <= S; ++d) prob[d] = __fdiv_rn(prob[d], den);
    }
    __syncthreads();
    // model.cpp:660-664: output[i] += p_d * value_d[i], depth order from 0
    float* o = out + static_cast<size_t>(t) * H;
    for (uint32_t i0 = threadIdx.x; i0 < n; i0 += kO * kAttnResThreads) {
        float acc[kO][W];
#pragma unroll
        for (uint32_t j = 0; j < kO; ++j)
#pragma unroll
            for (uint32_t k = 0; k < W; ++k) acc[j][k] = 0.0f;
        for (uint32_t d0 = 0; d0 <= S; d0 += kD) {
            float x[kD][kO][W];
#pragma unroll
            for (uint32_t e = 0; e < kD; ++e) {
                if (d0 + e > S) break;
                const float* v = row(d0 + e);
#pragma unroll
                for (uint32_t j = 0; j < kO; ++j)
                    if (i0 + j * kAttnResThreads < n) ld(v, i0 + j * kAttnResThreads, x[e][j]);
            }
#pragma unroll
            for (uint32_t e = 0; e < kD; ++e) {
                if (d0 + e > S) break;
                const float pd = prob[d0 + e];
#pragma unroll
                for (uint32_t j = 0; j < kO; ++j) {
                    if (i0 + j * kAttnResThreads >= n) break;
#pragma unroll
                    for (uint32_t k = 0; k < W; ++k) acc[j][k] = __fadd_rn(acc[j][k], __fmul_rn(pd, x[e][j][k]));
                }
            }
        }
#pragma unroll
        for (uint32_t j = 0; j < kO; ++j) {
            const uint32_t i = i0 + j * kAttnResThreads;
            if (i >= n) break;
            if constexpr (VEC) reinterpret_cast<float4*>(o)[i] = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
            else o[i] = acc[j][0];
        }
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int launch_block_attnres(k3xb_ctx* ctx, const float* prefix, const float* sources, uint32_t S, uint32_t T, uint32_t H,
                         const float* norm, const float* proj, float eps, float* out) {
    const bool vec = H % 4 == 0 && aligned16(prefix) && (!S || aligned16(sources)) && aligned16(norm) &&
                     aligned16(proj) && aligned16(out);
    const size_t smem = static_cast<size_t>(H) * sizeof(float);
    if (smem > kBlockAttnResMaxSmem) return fail(ctx, K3XB_INVALID_EXTENT, "block attention residual: hidden too large");
    static std::atomic<uint64_t> configured{0};
    const int cst = configure_once(ctx, configured, [&]() -> int {
        K3XB_CUDA(ctx, cudaFuncSetAttribute(block_attnres_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(kBlockAttnResMaxSmem)));
        K3XB_CUDA(ctx, cudaFuncSetAttribute(block_attnres_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(kBlockAttnResMaxSmem)));
        return K3XB_OK;
    });
    if (cst) return cst;
    if (vec)
        block_attnres_kernel<true><<<T, kAttnResThreads, smem, ctx->stream>>>(prefix, sources, S, T, H, norm, proj,
                                                                              eps, out);
    else
        block_attnres_kernel<false><<<T, kAttnResThreads, smem, ctx->stream>>>(prefix, sources, S, T, H, norm, proj,
                                                                               eps, out);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

}  // namespace k3xb
