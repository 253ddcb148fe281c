// layer.cu — the non-GEMM steps of the official KDA block and of the
// KDA + MoE layer, for S sequences that share one draft topology.
//
// Reference: official_kda.cpp:198-426 (block), official_layer.cpp:42-125
// (attention residual, RMSNorm), official_layer.cpp:134-244 (layer
// composition), official_moe.cpp:156-209 (MoE input preparation). The
// projections run on the tcgen05 bf16 linear kernel (linear_tc.cu) and the
// recurrence on the draft-tree kernel (kda.cu).
//
// Rows are nodes: row t = s * N + n for sequence s, node n. Float
// arithmetic is written with explicit _rn intrinsics in the reference's
// operation order (no contraction). Reductions the reference does
// sequentially (FP64 squares and scores, FP32 norms) are done as
// deterministic trees here, so values can differ in the last bits; the
// parity tests hold them to the hidden-state tolerance.
#include "common.cuh"
#include "kernels.cuh"

namespace k3xb {

namespace {

// Correctly rounded expf (glibc's expf agrees except on ~0.06% of inputs).
__device__ __forceinline__ float exp_cr(float x) { return static_cast<float>(exp(static_cast<double>(x))); }

__device__ __forceinline__ float sigmoid_ref(float x) {   // 1 / (1 + expf(-x))
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_cr(-x)));
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Deterministic block sum (blockDim.x = 256): per-thread partials, warp
// trees, then warp 0 over the 8 warp sums. Every thread gets the result.
__device__ double block_sum_d(double v, double* red) {
    const uint32_t lane = threadIdx.x % 32, warp = threadIdx.x / 32;
    v = warp_sum_d(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double t = lane < blockDim.x / 32 ? red[lane] : 0.0;
    t = warp_sum_d(t);
    return t;
}

// attention_residual (official_layer.cpp:42-102) followed by rms_norm
// (:104-125); one CTA per row. With `delta`, the first source is
// prefix = round_bf16(round_bf16(a) + delta) (official_layer.cpp:190-193),
// also written to prefix_out. With VEC (H % 4 == 0 and every row pointer
// 16-byte aligned, weights 8-byte aligned) each thread moves 4 columns per
// access and the loops are unrolled, so several loads are in flight; the
// sums of squares and scores are FP64 partials per thread combined by a
// deterministic block tree, rounded to float as the reference's sequential
// double sums are.
template <bool VEC>
__global__ void __launch_bounds__(256) attnres_norm_kernel(const float* __restrict__ a, const float* __restrict__ delta,
                                                           const float* __restrict__ block,
                                                           const uint16_t* __restrict__ rnorm,
                                                           const uint16_t* __restrict__ rproj,
                                                           const uint16_t* __restrict__ post, uint32_t H, float eps,
                                                           float* __restrict__ prefix_out, float* __restrict__ out) {
    extern __shared__ __align__(16) unsigned char attn_smem[];
    float* rp = reinterpret_cast<float*>(attn_smem);   // [H]
    float* rb = rp + H;                                // [H]
    __shared__ double red[32];
    const size_t row = blockIdx.x;
    const float* pa = a + row * H;
    const float* pb = block + row * H;
    const float* pd = delta ? delta + row * H : nullptr;
    float* po = prefix_out ? prefix_out + row * H : nullptr;
    constexpr uint32_t W = VEC ? 4u : 1u;
    const uint32_t n = H / W;
    auto ld = [](const float* p, uint32_t i, float (&v)[W]) {
        if constexpr (VEC) {
            const float4 q = __ldg(reinterpret_cast<const float4*>(p) + i);
            v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
        } else {
            v[0] = p[i];
        }
    };
    // shared-memory rows (rp, rb): plain loads (__ldg is for global memory only)
    auto lds = [](const float* p, uint32_t i, float (&v)[W]) {
        if constexpr (VEC) {
            const float4 q = reinterpret_cast<const float4*>(p)[i];
            v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
        } else {
            v[0] = p[i];
        }
    };
    auto st = [](float* p, uint32_t i, const float (&v)[W]) {
        if constexpr (VEC) reinterpret_cast<float4*>(p)[i] = make_float4(v[0], v[1], v[2], v[3]);
        else p[i] = v[0];
    };
    auto ldw = [](const uint16_t* p, uint32_t i, float (&v)[W]) {
        if constexpr (VEC) {
            const uint2 q = __ldg(reinterpret_cast<const uint2*>(p) + i);
            v[0] = __uint_as_float(q.x << 16); v[1] = __uint_as_float(q.x & 0xffff0000u);
            v[2] = __uint_as_float(q.y << 16); v[3] = __uint_as_float(q.y & 0xffff0000u);
        } else {
            v[0] = decode_bf16(p[i]);
        }
    };
    double sq_p = 0.0, sq_b = 0.0;
    // batches of kB iterations: every global load of a batch is issued
    // before any of its values is used
    constexpr uint32_t kB = 4;
    for (uint32_t i0 = threadIdx.x; i0 < n; i0 += kB * blockDim.x) {
        float va[kB][W], vb[kB][W], vd[kB][W];
#pragma unroll
        for (uint32_t j = 0; j < kB; ++j) {
            const uint32_t i = i0 + j * blockDim.x;
            if (i < n) {
                ld(pa, i, va[j]);
                ld(pb, i, vb[j]);
                if (pd) ld(pd, i, vd[j]);
            }
        }
#pragma unroll
        for (uint32_t j = 0; j < kB; ++j) {
            const uint32_t i = i0 + j * blockDim.x;
            if (i >= n) break;
#pragma unroll
            for (uint32_t k = 0; k < W; ++k) {
                if (pd) va[j][k] = round_bf16(__fadd_rn(round_bf16(va[j][k]), vd[j][k]));
                va[j][k] = round_bf16(va[j][k]);
                vb[j][k] = round_bf16(vb[j][k]);
                sq_p = fma(static_cast<double>(va[j][k]), static_cast<double>(va[j][k]), sq_p);
                sq_b = fma(static_cast<double>(vb[j][k]), static_cast<double>(vb[j][k]), sq_b);
            }
            if (po) st(po, i, va[j]);   // the prefix: round_bf16 leaves it unchanged
            st(rp, i, va[j]);
            st(rb, i, vb[j]);
        }
    }
    sq_p = block_sum_d(sq_p, red);
    sq_b = block_sum_d(sq_b, red);
    const float inv_p = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(sq_p / H), eps)));
    const float inv_b = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(sq_b / H), eps)));
    double sc_p = 0.0, sc_b = 0.0;
    for (uint32_t i0 = threadIdx.x; i0 < n; i0 += kB * blockDim.x) {
        float nv[kB][W], pv[kB][W];
#pragma unroll
        for (uint32_t j = 0; j < kB; ++j) {
            const uint32_t i = i0 + j * blockDim.x;
            if (i < n) {
                ldw(rnorm, i, nv[j]);
                ldw(rproj, i, pv[j]);
            }
        }
#pragma unroll
        for (uint32_t j = 0; j < kB; ++j) {
            const uint32_t i = i0 + j * blockDim.x;
            if (i >= n) break;
            float xp[W], xb[W];
            lds(rp, i, xp);
            lds(rb, i, xb);
#pragma unroll
            for (uint32_t k = 0; k < W; ++k) {
                const double nw = static_cast<double>(nv[j][k]) * static_cast<double>(pv[j][k]);
                sc_p += static_cast<double>(__fmul_rn(xp[k], inv_p)) * nw;   // exact product, as (v*inv)*norm*proj
                sc_b += static_cast<double>(__fmul_rn(xb[k], inv_b)) * nw;
            }
        }
    }
    const float score_p = static_cast<float>(block_sum_d(sc_p, red));
    const float score_b = static_cast<float>(block_sum_d(sc_b, red));
    const float m = score_b > score_p ? score_b : score_p;
    const float eb = exp_cr(__fsub_rn(score_b, m)), ep = exp_cr(__fsub_rn(score_p, m));
    const float den = __fadd_rn(eb, ep);
    const float wb = __fdiv_rn(eb, den), wp = __fdiv_rn(ep, den);
    double sq = 0.0;
#pragma unroll 4
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        float xp[W], xb[W];
        lds(rp, i, xp);
        lds(rb, i, xb);
#pragma unroll
        for (uint32_t k = 0; k < W; ++k) {
            xb[k] = round_bf16(__fadd_rn(__fmul_rn(wb, xb[k]), __fmul_rn(wp, xp[k])));
            sq = fma(static_cast<double>(xb[k]), static_cast<double>(xb[k]), sq);
        }
        st(rb, i, xb);
    }
    sq = block_sum_d(sq, red);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(sq / H), eps)));
#pragma unroll 4
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        float xb[W], pw[W];
        lds(rb, i, xb);
        ldw(post, i, pw);
#pragma unroll
        for (uint32_t k = 0; k < W; ++k) xb[k] = round_bf16(__fmul_rn(__fmul_rn(xb[k], inv), pw[k]));
        st(out + row * H, i, xb);
    }
}

// Short causal conv + SiLU (official_kda.cpp:95-143) along each node's
// ancestor path. anc[n][j-1] (j = 1..w-1) is node n's j-th ancestor, or
// -(r+1) for row r of the sequence's conv history (oldest row 0) once the
// path leaves the draft tree. One thread per (projection, row, channel).
struct ConvArgs {
    const float* proj[3];     // projected q, k, v [T][P] (bf16 values)
    const float* weight[3];   // [P][w]
    float* out[3];            // conv outputs [T][P]
};

__global__ void __launch_bounds__(256) short_conv_kernel(ConvArgs args, const uint16_t* __restrict__ conv,
                                                         const int32_t* __restrict__ anc, uint32_t S, uint32_t N,
                                                         uint32_t P, uint32_t w) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint32_t type = blockIdx.y;
    if (i >= static_cast<size_t>(S) * N * P) return;
    const uint32_t c = static_cast<uint32_t>(i % P);
    const size_t t = i / P;
    const uint32_t s = static_cast<uint32_t>(t / N), n = static_cast<uint32_t>(t % N);
    const float* proj = args.proj[type];
    const float* wt = args.weight[type] + static_cast<size_t>(c) * w;
    const uint16_t* hist = conv + (static_cast<size_t>(s) * 3 + type) * (w - 1) * P;
    float sum = 0.0f;
    for (uint32_t j = w - 1; j >= 1; --j) {   // oldest first, as the state rows
        const int32_t a = anc[static_cast<size_t>(n) * (w - 1) + j - 1];
        const float v = a >= 0 ? proj[(static_cast<size_t>(s) * N + a) * P + c]
                               : decode_bf16(hist[static_cast<size_t>(-a - 1) * P + c]);
        sum = __fadd_rn(sum, __fmul_rn(v, wt[w - 1 - j]));
    }
    sum = __fadd_rn(sum, __fmul_rn(proj[t * P + c], wt[w - 1]));
    args.out[type][t * P + c] = round_bf16(__fdiv_rn(sum, __fadd_rn(1.0f, exp_cr(-sum))));
}

// q/k L2 norms (official_kda.cpp:259-290), log-decay (:292-309) and beta
// (:310-317); one warp per (row, head).
__global__ void __launch_bounds__(256) qk_gates_kernel(const float* __restrict__ cq, const float* __restrict__ ck,
                                                       const float* __restrict__ fg, const float* __restrict__ bp,
                                                       const float* __restrict__ a_log,
                                                       const float* __restrict__ dt_bias, float glb, uint32_t T,
                                                       uint32_t h, uint32_t d, float* __restrict__ qn,
                                                       float* __restrict__ kn, float* __restrict__ ld,
                                                       float* __restrict__ be) {
    const uint32_t wid = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
    if (wid >= static_cast<size_t>(T) * h) return;
    const uint32_t t = wid / h, hh = wid % h;
    const size_t base = (static_cast<size_t>(t) * h + hh) * d;
    float qs = 0.0f, ks = 0.0f;
    for (uint32_t c = lane; c < d; c += 32) {
        qs = __fadd_rn(qs, __fmul_rn(cq[base + c], cq[base + c]));
        ks = __fadd_rn(ks, __fmul_rn(ck[base + c], ck[base + c]));
    }
    qs = warp_sum(qs);
    ks = warp_sum(ks);
    const float q_scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(d)));
    const float qi = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn(qs), 1.0e-12f));
    const float ki = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn(ks), 1.0e-12f));
    for (uint32_t c = lane; c < d; c += 32) {
        qn[base + c] = round_bf16(__fmul_rn(__fmul_rn(cq[base + c], qi), q_scale));
        kn[base + c] = round_bf16(__fmul_rn(ck[base + c], ki));
        const float arg = __fmul_rn(exp_cr(a_log[c]), __fadd_rn(fg[base + c], dt_bias[hh * d + c]));
        ld[base + c] = __fdiv_rn(glb, __fadd_rn(1.0f, exp_cr(-arg)));
    }
    if (lane == 0) be[static_cast<size_t>(t) * h + hh] = sigmoid_ref(bp[static_cast<size_t>(t) * h + hh]);
}

// Gated output RMSNorm (official_kda.cpp:371-395); one warp per (row, head).
__global__ void __launch_bounds__(256) gated_norm_kernel(const float* __restrict__ ro, const float* __restrict__ og,
                                                         const float* __restrict__ o_norm, float eps, uint32_t T,
                                                         uint32_t h, uint32_t d, float* __restrict__ gt) {
    const uint32_t wid = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
    if (wid >= static_cast<size_t>(T) * h) return;
    const size_t base = static_cast<size_t>(wid) * d;
    float sq = 0.0f;
    for (uint32_t c = lane; c < d; c += 32) sq = __fadd_rn(sq, __fmul_rn(ro[base + c], ro[base + c]));
    sq = warp_sum(sq);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sq, static_cast<float>(d)), eps)));
    for (uint32_t c = lane; c < d; c += 32) {
        const float gate = sigmoid_ref(og[base + c]);
        gt[base + c] = round_bf16(__fmul_rn(__fmul_rn(__fmul_rn(ro[base + c], inv), o_norm[c]), gate));
    }
}

// out = round_bf16(round_bf16(a) + b) (official_moe.cpp:339-340).
__global__ void residual_kernel(const float* __restrict__ a, const float* __restrict__ b, size_t n,
                                float* __restrict__ out) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) out[i] = round_bf16(__fadd_rn(round_bf16(a[i]), b[i]));
}

__global__ void round_kernel(const float* __restrict__ a, size_t n, float* __restrict__ out) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) out[i] = round_bf16(a[i]);
}

// Conv histories after the commit node (official_kda.cpp:136-141 applied
// along the path): row r (oldest first) is the value w-2-r steps before the
// commit node; rows older than the path come from the input history.
// anc_commit[s][j] (j = 0..w-2) is the commit node (j = 0) and its
// ancestors, or -(r+1) for input row r. One thread per (s, type, channel).
__global__ void conv_commit_kernel(ConvArgs args, const uint16_t* __restrict__ conv_in,
                                   const int32_t* __restrict__ anc_commit, uint32_t S, uint32_t N, uint32_t P,
                                   uint32_t w, uint16_t* __restrict__ conv_out) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<size_t>(S) * 3 * P) return;
    const uint32_t c = static_cast<uint32_t>(i % P);
    const uint32_t type = static_cast<uint32_t>((i / P) % 3), s = static_cast<uint32_t>(i / P / 3);
    const uint16_t* hin = conv_in + (static_cast<size_t>(s) * 3 + type) * (w - 1) * P;
    uint16_t* hout = conv_out + (static_cast<size_t>(s) * 3 + type) * (w - 1) * P;
    // rows in increasing order: an input row read is never below the row
    // being written, so conv_out may alias conv_in
    for (uint32_t r = 0; r + 1 < w; ++r) {
        const int32_t a = anc_commit[static_cast<size_t>(s) * (w - 1) + (w - 2 - r)];
        hout[static_cast<size_t>(r) * P + c] =
            a >= 0 ? encode_bf16(args.proj[type][(static_cast<size_t>(s) * N + a) * P + c])
                   : hin[static_cast<size_t>(-a - 1) * P + c];
    }
}

// rms_norm (official_layer.cpp:104-125): one CTA per row.
__global__ void __launch_bounds__(256) rms_norm_kernel(const float* __restrict__ x, const uint16_t* __restrict__ w,
                                                       uint32_t H, float eps, float* __restrict__ out) {
    __shared__ double red[32];
    const size_t row = blockIdx.x;
    const float* px = x + row * H;
    double sq = 0.0;
    for (uint32_t i = threadIdx.x; i < H; i += blockDim.x)
        sq = fma(static_cast<double>(px[i]), static_cast<double>(px[i]), sq);
    sq = block_sum_d(sq, red);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(sq / H), eps)));
    for (uint32_t i = threadIdx.x; i < H; i += blockDim.x)
        out[row * H + i] = round_bf16(__fmul_rn(__fmul_rn(px[i], inv), decode_bf16(w[i])));
}

// Embedding rows of token ids (bf16 table [V][H]); an id >= V zeroes the
// row and sets the status word.
__global__ void embed_kernel(const uint32_t* __restrict__ tokens, const uint16_t* __restrict__ table, uint32_t V,
                             uint32_t H, size_t n, float* __restrict__ out, int* status) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t tok = tokens[i / H];
    if (tok >= V) {
        out[i] = 0.0f;
        if (status) atomicExch(status, K3XB_INVALID_EXTENT);
        return;
    }
    out[i] = decode_bf16(table[static_cast<size_t>(tok) * H + i % H]);
}

// Conv histories after a device-chosen node of a LINEAR draft (node c =
// commit[s]): row r is node c - (w-2-r) when >= 0, else input history row
// w-1-j+c for j = w-2-r steps back.
__global__ void conv_commit_linear_kernel(ConvArgs args, const uint16_t* __restrict__ conv_in,
                                          const uint32_t* __restrict__ commit, uint32_t S, uint32_t N, uint32_t P,
                                          uint32_t w, uint16_t* __restrict__ conv_out) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<size_t>(S) * 3 * P) return;
    const uint32_t c = static_cast<uint32_t>(i % P);
    const uint32_t type = static_cast<uint32_t>((i / P) % 3), s = static_cast<uint32_t>(i / P / 3);
    const int32_t node = static_cast<int32_t>(min(commit[s], N - 1));
    const uint16_t* hin = conv_in + (static_cast<size_t>(s) * 3 + type) * (w - 1) * P;
    uint16_t* hout = conv_out + (static_cast<size_t>(s) * 3 + type) * (w - 1) * P;
    for (uint32_t r = 0; r + 1 < w; ++r) {   // increasing rows: in-place safe
        const int32_t j = static_cast<int32_t>(w) - 2 - static_cast<int32_t>(r);
        const int32_t a = node - j;
        hout[static_cast<size_t>(r) * P + c] =
            a >= 0 ? encode_bf16(args.proj[type][(static_cast<size_t>(s) * N + a) * P + c])
                   : hin[static_cast<size_t>(static_cast<int32_t>(w) - 1 - j + node) * P + c];
    }
}

}  // namespace

int launch_rms_norm(k3xb_ctx* ctx, const float* x, const uint16_t* w, uint32_t T, uint32_t H, float eps, float* out) {
    rms_norm_kernel<<<T, 256, 0, ctx->stream>>>(x, w, H, eps, out);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_embed(k3xb_ctx* ctx, const uint32_t* tokens, const uint16_t* table, uint32_t V, uint32_t T, uint32_t H,
                 float* out) {
    const size_t n = static_cast<size_t>(T) * H;
    embed_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, ctx->stream>>>(tokens, table, V, H, n, out,
                                                                                  ctx->status_word);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_conv_commit_linear(k3xb_ctx* ctx, const float* const proj[3], const uint16_t* conv_in,
                              const uint32_t* commit, uint32_t S, uint32_t N, uint32_t P, uint32_t w,
                              uint16_t* conv_out) {
    ConvArgs args{{proj[0], proj[1], proj[2]}, {nullptr, nullptr, nullptr}, {nullptr, nullptr, nullptr}};
    const size_t n = static_cast<size_t>(S) * 3 * P;
    conv_commit_linear_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, ctx->stream>>>(args, conv_in, commit,
                                                                                               S, N, P, w, conv_out);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

size_t attnres_smem_bytes(uint32_t H) { return 2ull * H * sizeof(float); }

int launch_attnres_norm(k3xb_ctx* ctx, const float* a, const float* delta, const float* block, const uint16_t* rnorm,
                        const uint16_t* rproj, const uint16_t* post, uint32_t T, uint32_t H, float eps,
                        float* prefix_out, float* out) {
    const size_t smem = attnres_smem_bytes(H);
    if (smem > 200 * 1024) return fail(ctx, K3XB_INVALID_EXTENT, "attention residual: hidden too large");
    static std::atomic<uint64_t> configured{0};
    const int cst = configure_once(ctx, configured, [&]() -> int {
        K3XB_CUDA(ctx, cudaFuncSetAttribute(attnres_norm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            200 * 1024));
        K3XB_CUDA(ctx, cudaFuncSetAttribute(attnres_norm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            200 * 1024));
        return K3XB_OK;
    });
    if (cst) return cst;
    auto al = [](const void* p, uintptr_t m) { return (reinterpret_cast<uintptr_t>(p) & m) == 0; };
    const bool vec = H % 4 == 0 && al(a, 15) && al(delta, 15) && al(block, 15) && al(prefix_out, 15) && al(out, 15) &&
                     al(rnorm, 7) && al(rproj, 7) && al(post, 7);
    if (vec)
        attnres_norm_kernel<true><<<T, 256, smem, ctx->stream>>>(a, delta, block, rnorm, rproj, post, H, eps,
                                                                 prefix_out, out);
    else
        attnres_norm_kernel<false><<<T, 256, smem, ctx->stream>>>(a, delta, block, rnorm, rproj, post, H, eps,
                                                                  prefix_out, out);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_short_conv(k3xb_ctx* ctx, const float* const proj[3], const float* const weight[3], const uint16_t* conv,
                      const int32_t* anc, uint32_t S, uint32_t N, uint32_t P, uint32_t w, float* const out[3]) {
    ConvArgs args{{proj[0], proj[1], proj[2]}, {weight[0], weight[1], weight[2]}, {out[0], out[1], out[2]}};
    const size_t n = static_cast<size_t>(S) * N * P;
    dim3 grid(static_cast<unsigned>((n + 255) / 256), 3);
    short_conv_kernel<<<grid, 256, 0, ctx->stream>>>(args, conv, anc, S, N, P, w);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_qk_gates(k3xb_ctx* ctx, const float* cq, const float* ck, const float* fg, const float* bp,
                    const float* a_log, const float* dt_bias, float glb, uint32_t T, uint32_t h, uint32_t d,
                    float* qn, float* kn, float* ld, float* be) {
    const size_t warps = static_cast<size_t>(T) * h;
    qk_gates_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, ctx->stream>>>(
        cq, ck, fg, bp, a_log, dt_bias, glb, T, h, d, qn, kn, ld, be);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_gated_norm(k3xb_ctx* ctx, const float* ro, const float* og, const float* o_norm, float eps, uint32_t T,
                      uint32_t h, uint32_t d, float* gt) {
    const size_t warps = static_cast<size_t>(T) * h;
    gated_norm_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, ctx->stream>>>(ro, og, o_norm, eps,
                                                                                                 T, h, d, gt);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_residual_round(k3xb_ctx* ctx, const float* a, size_t n, float* out) {
    round_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, ctx->stream>>>(a, n, out);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_residual(k3xb_ctx* ctx, const float* a, const float* b, size_t n, float* out) {
    residual_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, ctx->stream>>>(a, b, n, out);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_conv_commit(k3xb_ctx* ctx, const float* const proj[3], const uint16_t* conv_in, const int32_t* anc_commit,
                       uint32_t S, uint32_t N, uint32_t P, uint32_t w, uint16_t* conv_out) {
    ConvArgs args{{proj[0], proj[1], proj[2]}, {nullptr, nullptr, nullptr}, {nullptr, nullptr, nullptr}};
    const size_t n = static_cast<size_t>(S) * 3 * P;
    conv_commit_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, ctx->stream>>>(args, conv_in, anc_commit, S,
                                                                                        N, P, w, conv_out);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

}  // namespace k3xb
