// linear_tc.cu — bf16 linear layer on tcgen05 kind::f16:
// out[t][r] = (round_bf16)(sum_k W[r][k] * x[t][k]), W [rows][K] bf16 words,
// x [T][K] float. This is bf16_matvec (runtime/src/official_moe.cpp:39-59)
// for many tokens at once, with FP32 accumulation in TMEM instead of FP64.
// x enters as bf16 terms: one per token when x is bf16-valued (the KDA
// projections and the LM head: every input there is already rounded), or
// two (hi = bf16(x), lo = bf16(x - hi)), which carry any float to ~16 bits;
// the epilogue adds a token's term columns. A B tile is 128 rows: 128
// tokens x 1 term or 64 tokens x 2 terms, loaded with one TMA box per stage.
// Used for the LM head (V x H) and the KDA projections.
#include "common.cuh"
#include "kernels.cuh"
#include "tc_pipeline.cuh"

namespace k3xb {

namespace {

using tcp::kBlockM;
using tcp::kThreads;

constexpr uint32_t kTileRows = 128;   // B rows per tile (tokens x terms)
constexpr uint32_t kStages = 6;

struct LinParams {
    uint32_t T, rows, K, items, round_out, terms;
    float* out;      // [T][rows]
    int* error;
};

__global__ void split1_kernel(const float* __restrict__ x, size_t n, uint16_t* __restrict__ out) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) out[i] = static_cast<uint16_t>(__float_as_uint(round_bf16(x[i])) >> 16);
}

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
__device__ __forceinline__ uint4 lin_desc(uint32_t item, uint32_t T, uint32_t terms) {
    const uint32_t tpt = kTileRows / terms;
    const uint32_t tiles = (T + tpt - 1) / tpt;
    const uint32_t tile = item % tiles, mt = item / tiles;
    const uint32_t ntok = min(tpt, T - tile * tpt);
    return make_uint4(mt * kBlockM, tile * kTileRows, ((terms * ntok + 15) / 16 * 16) | (ntok << 16), tile * tpt);
}

__global__ void __launch_bounds__(kThreads, 1) linear_bf16_kernel(const __grid_constant__ CUtensorMap map_w,
                                                                   const __grid_constant__ CUtensorMap map_x,
                                                                   const LinParams p) {
    extern __shared__ uint8_t smem_raw[];
    auto& sm = tcp::smem_from<kStages, 1>(smem_raw);
    auto get_desc = [&](uint32_t item) { return lin_desc(item, p.T, p.terms); };
    auto epilogue = [&](const uint4& d, uint32_t tmem, uint32_t q, uint32_t lane) {
        const uint32_t terms = p.terms;
        const uint32_t used = terms * tcp::desc_ntok(d);
        const uint32_t lane_base = (32u * q) << 16;
        const uint32_t r = d.x + 32u * q + lane;
        for (uint32_t c0 = 0; c0 < used; c0 += 16) {
            float v[16];
            tc::tmem_ld16(tmem + lane_base + c0, v);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if (c0 + i >= used) break;
                if ((c0 + i) % terms != terms - 1) continue;   // last term column of a token
                const size_t tok = d.w + (c0 + i) / terms;
                const float y = terms == 2 ? __fadd_rn(v[i - 1], v[i]) : v[i];
                if (r < p.rows) p.out[tok * p.rows + r] = p.round_out ? round_bf16(y) : y;
            }
        }
    };
    const uint8_t* none[1] = {nullptr};
    const tcp::Config cfg{p.K, p.items, 256, 0, 0, 128, 0, 0, 0, 0, kTileRows};
    tcp::run_pipeline<kStages, 1, true, 2>(sm, &map_w, &map_w, &map_x, cfg, none, nullptr, p.error, get_desc,
                                           epilogue);
}

}  // namespace

int make_byte_map(k3xb_ctx* ctx, void* map, const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_rows);

size_t linear_scratch_bytes(uint32_t T, uint32_t K) { return static_cast<size_t>(2) * T * K * 2 + 1024; }

int launch_linear_terms(k3xb_ctx* ctx, const uint16_t* xterms, uint32_t terms, const uint16_t* W, uint32_t T,
                        uint32_t rows, uint32_t K, int round_out, float* out) {
    if (K % 8) return fail(ctx, K3XB_INVALID_EXTENT, "bf16 linear needs K % 8 == 0");
    if (terms != 1 && terms != 2) return fail(ctx, K3XB_INVALID_EXTENT, "bf16 linear: 1 or 2 terms");
    int st;
    CUtensorMap map_w, map_x;
    if ((st = make_byte_map(ctx, &map_w, W, static_cast<uint64_t>(K) * 2, rows, 128))) return st;
    if ((st = make_byte_map(ctx, &map_x, xterms, static_cast<uint64_t>(K) * 2, static_cast<uint64_t>(terms) * T,
                            kTileRows)))
        return st;
    static std::atomic<uint64_t> configured{0};
    const size_t smem = tcp::smem_bytes<kStages, 1>();
    const int cst = configure_once(ctx, configured, [&]() -> int {
        K3XB_CUDA(ctx, cudaFuncSetAttribute(linear_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(smem)));
        return K3XB_OK;
    });
    if (cst) return cst;
    const uint32_t tpt = kTileRows / terms;
    const uint32_t items = ((T + tpt - 1) / tpt) * ((rows + kBlockM - 1) / kBlockM);
    LinParams p{T, rows, K, items, static_cast<uint32_t>(round_out ? 1 : 0), terms, out, ctx->status_word};
    linear_bf16_kernel<<<std::min<uint32_t>(ctx->sm_count, items), kThreads, smem, ctx->stream>>>(map_w, map_x, p);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_split_terms(k3xb_ctx* ctx, const float* x, uint32_t T, uint32_t K, uint32_t terms, uint16_t* xterms) {
    const size_t n = static_cast<size_t>(T) * K;
    if (terms == 1) split1_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, ctx->stream>>>(x, n, xterms);
    else split2_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, ctx->stream>>>(x, n, K, xterms);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_linear_bf16(k3xb_ctx* ctx, const float* x, const uint16_t* W, uint32_t T, uint32_t rows, uint32_t K,
                       int round_out, uint16_t* xterms, float* out) {
    if (K % 8) return fail(ctx, K3XB_INVALID_EXTENT, "bf16 linear needs K % 8 == 0");
    int st = launch_split_terms(ctx, x, T, K, 2, xterms);
    if (st) return st;
    return launch_linear_terms(ctx, xterms, 2, W, T, rows, K, round_out, out);
}

}  // namespace k3xb
