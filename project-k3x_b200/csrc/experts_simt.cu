// experts_simt.cu — CUDA-core expert FFN (FP4 decode + FP32 FMA), the
// slot-ordered routed combine (c), and the bf16 shared-expert matvecs.
//
// The SIMT engine is the cross-check for the tcgen05 engine and the
// fallback-free reference point for its numerics: every output element
// is a float dot product of decoded MXFP4 weights (exact values) with the
// float activation, followed by the reference's float activation and bf16
// rounding (official_moe.cpp:82-103).
//
// Work split (gate/up): one CTA = 32 output rows of one expert group, both
// gate and up; each warp owns 4 rows; lane l covers elements [8l, 8l+8) of
// every 256-wide K superblock, so a warp reads one coalesced 128-byte
// segment per row and 8 scale bytes. Tokens of the group are processed 4 at
// a time against a shared-memory copy of their activations.
#include "common.cuh"
#include "kernels.cuh"

namespace k3xb {

namespace {

constexpr int kRowsPerWarp = 4;
constexpr int kWarps = 8;
constexpr int kRowsPerCta = kRowsPerWarp * kWarps;   // 32
constexpr int kTokChunk = 4;
constexpr int kKChunk = 1024;                         // activations staged per pass

__device__ __forceinline__ void decode8(uint32_t packed, float scale, float* out) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t code = (packed >> (4 * i)) & 15u;
        const float mag = e2m1_magnitude(code & 7u) * scale;
        out[i] = (code & 8u) ? -mag : mag;
    }
}

__device__ __forceinline__ float activate(float g, float u, int act, float beta, float lbeta) {
    // SwiGLU: (g * sigmoid(g)) * u; SiTU: ops.cpp:20-30.
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
    if (act == K3XB_ACT_SITU) {
        const float bg = __fmul_rn(__fmul_rn(beta, tanhf(__fdiv_rn(g, beta))), sig);
        const float bu = lbeta > 0.0f ? __fmul_rn(lbeta, tanhf(__fdiv_rn(u, lbeta))) : u;
        return __fmul_rn(bg, bu);
    }
    return __fmul_rn(__fmul_rn(g, sig), u);
}

// Accumulates rows [row0, row0+4) of NMAT MXFP4 matrices (all [rows][K])
// against kTokChunk activation rows staged in smem. acc[m][r][j].
template <int NMAT>
__device__ __forceinline__ void mxfp4_rows_dot(
    const uint8_t* const* packed, const uint8_t* const* scales, uint32_t K,
    uint32_t row0, const float* xs, uint32_t k0, uint32_t klen, uint32_t lane,
    float (&acc)[NMAT][kRowsPerWarp][kTokChunk]) {
    for (uint32_t kb = 0; kb < klen; kb += 256) {
        float xv[kTokChunk][8];
#pragma unroll
        for (int j = 0; j < kTokChunk; ++j) {
            const float4 a = *reinterpret_cast<const float4*>(xs + j * kKChunk + kb + 8 * lane);
            const float4 b = *reinterpret_cast<const float4*>(xs + j * kKChunk + kb + 8 * lane + 4);
            xv[j][0] = a.x; xv[j][1] = a.y; xv[j][2] = a.z; xv[j][3] = a.w;
            xv[j][4] = b.x; xv[j][5] = b.y; xv[j][6] = b.z; xv[j][7] = b.w;
        }
        const uint32_t kk = k0 + kb + 8 * lane;   // first element of this lane
        if (kb + 8 * lane >= klen) continue;      // K not a multiple of 256
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
#pragma unroll
            for (int r = 0; r < kRowsPerWarp; ++r) {
                const size_t row = row0 + r;
                const uint32_t p = __ldg(reinterpret_cast<const uint32_t*>(
                    packed[m] + row * (K / 2) + kk / 2));
                const uint32_t sb = __ldg(scales[m] + row * (K / 32) + kk / 32);
                float w[8];
                decode8(p, exp2i(static_cast<int>(sb) - 127), w);
#pragma unroll
                for (int j = 0; j < kTokChunk; ++j)
#pragma unroll
                    for (int i = 0; i < 8; ++i) acc[m][r][j] = fmaf(w[i], xv[j][i], acc[m][r][j]);
            }
        }
    }
}

// gate/up for one group: act[assign][I] (float)
__global__ void __launch_bounds__(256) simt_gateup_kernel(
    const float* __restrict__ hidden, uint32_t H, uint32_t I, const uint8_t* gate_p,
    const uint8_t* gate_s, const uint8_t* up_p, const uint8_t* up_s, const uint32_t* group_expert,
    const uint32_t* group_offset, const uint32_t* group_count, const uint32_t* assign_token,
    int act, float beta, float lbeta, float* __restrict__ act_out) {
    extern __shared__ float xs[];   // [kTokChunk][kKChunk]
    const uint32_t g = blockIdx.y;
    if (g >= *group_count) return;
    const uint32_t e = group_expert[g];
    const uint32_t a0 = group_offset[g], a1 = group_offset[g + 1];
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t row0 = blockIdx.x * kRowsPerCta + warp * kRowsPerWarp;
    const uint8_t* packed[2] = {gate_p + static_cast<size_t>(e) * I * (H / 2),
                                up_p + static_cast<size_t>(e) * I * (H / 2)};
    const uint8_t* scales[2] = {gate_s + static_cast<size_t>(e) * I * (H / 32),
                                up_s + static_cast<size_t>(e) * I * (H / 32)};
    for (uint32_t a = a0; a < a1; a += kTokChunk) {
        float acc[2][kRowsPerWarp][kTokChunk] = {};
        for (uint32_t k0 = 0; k0 < H; k0 += kKChunk) {
            const uint32_t klen = min(kKChunk, H - k0);
            __syncthreads();
            for (uint32_t i = threadIdx.x; i < kTokChunk * kKChunk; i += blockDim.x) {
                const uint32_t j = i / kKChunk, k = i % kKChunk;
                float v = 0.0f;
                if (a + j < a1 && k < klen) v = hidden[static_cast<size_t>(assign_token[a + j]) * H + k0 + k];
                xs[i] = v;
            }
            __syncthreads();
            mxfp4_rows_dot<2>(packed, scales, H, row0, xs, k0, klen, lane, acc);
        }
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
            for (int j = 0; j < kTokChunk; ++j) {
                const float gv = warp_sum(acc[0][r][j]);
                const float uv = warp_sum(acc[1][r][j]);
                if (lane == 0 && a + j < a1)
                    act_out[static_cast<size_t>(a + j) * I + row0 + r] = activate(gv, uv, act, beta, lbeta);
            }
    }
}

// down for one group: slot_out[token*k + slot][H] = round_bf16(W_d . act)
__global__ void __launch_bounds__(256) simt_down_kernel(
    const float* __restrict__ act_in, uint32_t H, uint32_t I, uint32_t top_k, const uint8_t* down_p,
    const uint8_t* down_s, const uint32_t* group_expert, const uint32_t* group_offset,
    const uint32_t* group_count, const uint32_t* assign_token, const uint32_t* assign_slot,
    float* __restrict__ slot_out) {
    extern __shared__ float xs[];
    const uint32_t g = blockIdx.y;
    if (g >= *group_count) return;
    const uint32_t e = group_expert[g];
    const uint32_t a0 = group_offset[g], a1 = group_offset[g + 1];
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t row0 = blockIdx.x * kRowsPerCta + warp * kRowsPerWarp;
    const uint8_t* packed[1] = {down_p + static_cast<size_t>(e) * H * (I / 2)};
    const uint8_t* scales[1] = {down_s + static_cast<size_t>(e) * H * (I / 32)};
    for (uint32_t a = a0; a < a1; a += kTokChunk) {
        float acc[1][kRowsPerWarp][kTokChunk] = {};
        for (uint32_t k0 = 0; k0 < I; k0 += kKChunk) {
            const uint32_t klen = min(kKChunk, I - k0);
            __syncthreads();
            for (uint32_t i = threadIdx.x; i < kTokChunk * kKChunk; i += blockDim.x) {
                const uint32_t j = i / kKChunk, k = i % kKChunk;
                xs[i] = (a + j < a1 && k < klen) ? act_in[static_cast<size_t>(a + j) * I + k0 + k] : 0.0f;
            }
            __syncthreads();
            mxfp4_rows_dot<1>(packed, scales, I, row0, xs, k0, klen, lane, acc);
        }
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
            for (int j = 0; j < kTokChunk; ++j) {
                const float y = warp_sum(acc[0][r][j]);
                if (lane == 0 && a + j < a1) {
                    const size_t dst = static_cast<size_t>(assign_token[a + j]) * top_k + assign_slot[a + j];
                    slot_out[dst * H + row0 + r] = round_bf16(y);
                }
            }
    }
}

// (c) routed combine, official_moe.cpp:313-322 + :336: per token,
// mixed = round_bf16(sum_slot c[slot] * y[slot]) in slot order (float,
// two roundings per term like the reference), then out = round_bf16(mixed
// + shared).
__global__ void combine_kernel(const float* __restrict__ slot_out, const float* __restrict__ contrib,
                               const float* __restrict__ shared, uint32_t T, uint32_t K, uint32_t H,
                               float* __restrict__ out) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<size_t>(T) * H) return;
    const size_t t = i / H, h = i % H;
    float mixed = 0.0f;
    for (uint32_t s = 0; s < K; ++s)
        mixed = __fadd_rn(mixed, __fmul_rn(contrib[t * K + s], slot_out[(t * K + s) * H + h]));
    mixed = round_bf16(mixed);
    const float sh = shared ? shared[i] : 0.0f;
    out[i] = round_bf16(__fadd_rn(mixed, sh));
}

// The same combine over bf16 expert rows: the MXF4 engine's down epilogue
// already rounds each row to bf16 (official_moe.cpp:101), so the words hold
// the rows exactly at half the bytes.
__global__ void combine16_kernel(const uint16_t* __restrict__ y, const float* __restrict__ contrib,
                                 const float* __restrict__ shared, uint32_t T, uint32_t K, uint32_t H,
                                 float* __restrict__ out) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<size_t>(T) * H) return;
    const size_t t = i / H, h = i % H;
    float mixed = 0.0f;
    for (uint32_t s = 0; s < K; ++s) {
        const float v = __uint_as_float(static_cast<uint32_t>(y[(t * K + s) * H + h]) << 16);
        mixed = __fadd_rn(mixed, __fmul_rn(contrib[t * K + s], v));
    }
    mixed = round_bf16(mixed);
    const float sh = shared ? shared[i] : 0.0f;
    out[i] = round_bf16(__fadd_rn(mixed, sh));
}

// bf16 matvec for T tokens (official_moe.cpp:39-59 semantics with FP32
// accumulation): out[t][r] = round_bf16(sum_k W[r][k] * x[t][k]). One warp
// per (row, 4 tokens); x may be any float.
__global__ void __launch_bounds__(256) bf16_rows_kernel(
    const float* __restrict__ x, const uint16_t* __restrict__ W, uint32_t T, uint32_t rows,
    uint32_t cols, float* __restrict__ out) {
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
    const uint32_t row = warp;
    const uint32_t t0 = blockIdx.y * kTokChunk;
    if (row >= rows) return;
    float acc[kTokChunk] = {};
    const uint16_t* w = W + static_cast<size_t>(row) * cols;
    for (uint32_t k = lane * 2; k < cols; k += 64) {
        const uint32_t pair = *reinterpret_cast<const uint32_t*>(w + k);
        const float w0 = __uint_as_float(pair << 16), w1 = __uint_as_float(pair & 0xffff0000u);
#pragma unroll
        for (int j = 0; j < kTokChunk; ++j) {
            if (t0 + j < T) {
                const float2 xv = *reinterpret_cast<const float2*>(x + static_cast<size_t>(t0 + j) * cols + k);
                acc[j] = fmaf(w0, xv.x, fmaf(w1, xv.y, acc[j]));
            }
        }
    }
#pragma unroll
    for (int j = 0; j < kTokChunk; ++j) {
        const float v = warp_sum(acc[j]);
        if (lane == 0 && t0 + j < T) out[static_cast<size_t>(t0 + j) * rows + row] = round_bf16(v);
    }
}

__global__ void act_kernel(const float* g, const float* u, size_t n, int act, float beta, float lbeta,
                           float* out) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) out[i] = activate(g[i], u[i], act, beta, lbeta);
}

}  // namespace

int launch_simt_experts(k3xb_ctx* ctx, const k3xb_moe_layer& L, const float* hidden, uint32_t T,
                        const k3xb_plan& plan, float* act_buf, float* slot_out) {
    const uint32_t H = L.hidden, I = L.inter;
    if (H % kRowsPerCta || I % kRowsPerCta)
        return fail(ctx, K3XB_INVALID_EXTENT, "SIMT experts need hidden and inter multiples of 32");
    const size_t smem = sizeof(float) * kTokChunk * kKChunk;
    const uint32_t max_groups = min(L.experts, T * L.top_k);
    simt_gateup_kernel<<<dim3(I / kRowsPerCta, max_groups), 256, smem, ctx->stream>>>(
        hidden, H, I, L.gate_packed, L.gate_scales, L.up_packed, L.up_scales, plan.group_expert,
        plan.group_offset, plan.group_count, plan.assign_token, L.activation, L.situ_beta,
        L.situ_linear_beta, act_buf);
    K3XB_LAUNCHED(ctx);
    simt_down_kernel<<<dim3(H / kRowsPerCta, max_groups), 256, smem, ctx->stream>>>(
        act_buf, H, I, L.top_k, L.down_packed, L.down_scales, plan.group_expert, plan.group_offset,
        plan.group_count, plan.assign_token, plan.assign_slot, slot_out);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_combine(k3xb_ctx* ctx, const float* slot_out, const float* contrib, const float* shared,
                   uint32_t T, uint32_t K, uint32_t H, float* out) {
    const size_t n = static_cast<size_t>(T) * H;
    combine_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, ctx->stream>>>(
        slot_out, contrib, shared, T, K, H, out);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_combine16(k3xb_ctx* ctx, const uint16_t* slot_out16, const float* contrib, const float* shared,
                     uint32_t T, uint32_t K, uint32_t H, float* out) {
    const size_t n = static_cast<size_t>(T) * H;
    combine16_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, ctx->stream>>>(slot_out16, contrib, shared,
                                                                                      T, K, H, out);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_bf16_rows(k3xb_ctx* ctx, const float* x, const uint16_t* W, uint32_t T, uint32_t rows,
                     uint32_t cols, float* out) {
    if (cols % 64) return fail(ctx, K3XB_INVALID_EXTENT, "bf16 matvec needs cols % 64 == 0");
    dim3 grid((rows * 32 + 255) / 256, (T + kTokChunk - 1) / kTokChunk);
    bf16_rows_kernel<<<grid, 256, 0, ctx->stream>>>(x, W, T, rows, cols, out);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_act(k3xb_ctx* ctx, const float* g, const float* u, size_t n, int act, float beta,
               float lbeta, float* out) {
    act_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, ctx->stream>>>(g, u, n, act, beta,
                                                                                 lbeta, out);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

}  // namespace k3xb
