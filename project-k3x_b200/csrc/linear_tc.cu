// linear_tc.cu — bf16 linear layer on tcgen05 kind::f16:
// out[t][r] = (round_bf16)(sum_k W[r][k] * x[t][k]), W [rows][K] bf16 words,
// x [T][K] float. This is bf16_matvec (runtime/src/official_moe.cpp:39-59)
// for many tokens at once, with FP32 accumulation in TMEM instead of FP64.
// x enters as two bf16 terms per token (hi = bf16(x), lo = bf16(x - hi)),
// which carries any float to ~16 bits and bf16-valued x exactly; the
// epilogue adds the two term columns. Used for the LM head (V x H) and the
// KDA projections.
#include "common.cuh"
#include "kernels.cuh"
#include "tc_pipeline.cuh"

namespace k3xb {

namespace {

using tcp::kBlockM;
using tcp::kThreads;

constexpr uint32_t kTok = 64;        // tokens per tile (N = 2 x 64 = 128)
constexpr uint32_t kStages = 6;

struct LinParams {
    uint32_t T, rows, K, items, round_out;
    float* out;      // [T][rows]
    int* error;
};

__global__ void split2_kernel(const float* __restrict__ x, size_t n, uint32_t K, uint16_t* __restrict__ out) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const size_t t = i / K, k = i % K;
    const float hi = round_bf16(x[i]);
    const float lo = round_bf16(__fsub_rn(x[i], hi));
    out[(2 * t) * K + k] = static_cast<uint16_t>(__float_as_uint(hi) >> 16);
    out[(2 * t + 1) * K + k] = static_cast<uint16_t>(__float_as_uint(lo) >> 16);
}

// Weight-tile-major item order: the token tiles of one 128-row weight tile
// are consecutive items, run by neighbouring CTAs at about the same time, so
// the weight tile comes from HBM once and from L2 for the other token tiles.
__device__ __forceinline__ uint4 lin_desc(uint32_t item, uint32_t T) {
    const uint32_t tiles = (T + kTok - 1) / kTok;
    const uint32_t tile = item % tiles, mt = item / tiles;
    const uint32_t ntok = min(kTok, T - tile * kTok);
    return make_uint4(mt * kBlockM, tile * 2 * kTok, ((2 * ntok + 15) / 16 * 16) | (ntok << 16), tile * kTok);
}

__global__ void __launch_bounds__(kThreads, 1) linear_bf16_kernel(const __grid_constant__ CUtensorMap map_w,
                                                                   const __grid_constant__ CUtensorMap map_x,
                                                                   const LinParams p) {
    extern __shared__ uint8_t smem_raw[];
    auto& sm = tcp::smem_from<kStages, 1>(smem_raw);
    auto get_desc = [&](uint32_t item) { return lin_desc(item, p.T); };
    auto epilogue = [&](const uint4& d, uint32_t tmem, uint32_t q, uint32_t lane) {
        const uint32_t used = 2 * tcp::desc_ntok(d);
        const uint32_t lane_base = (32u * q) << 16;
        const uint32_t r = d.x + 32u * q + lane;
        for (uint32_t c0 = 0; c0 < used; c0 += 16) {
            float v[16];
            tc::tmem_ld16(tmem + lane_base + c0, v);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; i += 2) {
                if (c0 + i >= used) break;
                const size_t tok = d.w + (c0 + i) / 2;
                const float y = __fadd_rn(v[i], v[i + 1]);
                if (r < p.rows) p.out[tok * p.rows + r] = p.round_out ? round_bf16(y) : y;
            }
        }
    };
    const uint8_t* none[1] = {nullptr};
    const tcp::Config cfg{p.K, p.items, 256, 0, 0, 128, 0, 0, 0};
    tcp::run_pipeline<kStages, 1, true, 2>(sm, &map_w, &map_w, &map_x, cfg, none, nullptr, p.error, get_desc,
                                           epilogue);
}

}  // namespace

int make_byte_map(k3xb_ctx* ctx, void* map, const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_rows);

size_t linear_scratch_bytes(uint32_t T, uint32_t K) { return static_cast<size_t>(2) * T * K * 2 + 1024; }

int launch_linear_terms(k3xb_ctx* ctx, const uint16_t* xterms, const uint16_t* W, uint32_t T, uint32_t rows,
                        uint32_t K, int round_out, float* out) {
    if (K % 8) return fail(ctx, K3XB_INVALID_EXTENT, "bf16 linear needs K % 8 == 0");
    int st;
    CUtensorMap map_w, map_x;
    if ((st = make_byte_map(ctx, &map_w, W, static_cast<uint64_t>(K) * 2, rows, 128))) return st;
    if ((st = make_byte_map(ctx, &map_x, xterms, static_cast<uint64_t>(K) * 2, 2ull * T, 16))) return st;
    static bool configured = false;
    const size_t smem = tcp::smem_bytes<kStages, 1>();
    if (!configured) {
        K3XB_CUDA(ctx, cudaFuncSetAttribute(linear_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(smem)));
        configured = true;
    }
    const uint32_t items = ((T + kTok - 1) / kTok) * ((rows + kBlockM - 1) / kBlockM);
    LinParams p{T, rows, K, items, static_cast<uint32_t>(round_out ? 1 : 0), out, ctx->status_word};
    linear_bf16_kernel<<<std::min<uint32_t>(ctx->sm_count, items), kThreads, smem, ctx->stream>>>(map_w, map_x, p);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_split_terms(k3xb_ctx* ctx, const float* x, uint32_t T, uint32_t K, uint16_t* xterms) {
    const size_t n = static_cast<size_t>(T) * K;
    split2_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, ctx->stream>>>(x, n, K, xterms);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_linear_bf16(k3xb_ctx* ctx, const float* x, const uint16_t* W, uint32_t T, uint32_t rows, uint32_t K,
                       int round_out, uint16_t* xterms, float* out) {
    if (K % 8) return fail(ctx, K3XB_INVALID_EXTENT, "bf16 linear needs K % 8 == 0");
    int st = launch_split_terms(ctx, x, T, K, xterms);
    if (st) return st;
    return launch_linear_terms(ctx, xterms, W, T, rows, K, round_out, out);
}

}  // namespace k3xb
