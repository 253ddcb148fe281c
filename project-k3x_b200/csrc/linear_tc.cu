// linear_tc.cu — bf16 linear layer on tcgen05 kind::f16:
// out[t][r] = (round_bf16)(sum_k W[r][k] * x[t][k]), W [rows][K] bf16 words,
// x [T][K] float. This is bf16_matvec (runtime/src/official_moe.cpp:39-59)
// for many tokens at once, with FP32 accumulation in TMEM instead of FP64.
// x enters as bf16 terms: one per token when x is bf16-valued (the KDA
// projections and the LM head: every input there is already rounded), or
// two (hi = bf16(x), lo = bf16(x - hi)), which carry any float to ~16 bits;
// the epilogue adds a token's term columns. A B tile holds up to 128 rows
// (or 256 once the tokens need more), the tokens spread evenly over as few
// tiles as that allows, loaded with one TMA box per stage. Used for the LM
// head (V x H), the KDA projections (grouped: one launch for the six of a
// block) and the LatentMoE projections.
#include "common.cuh"
#include "kernels.cuh"
#include "tc_pipeline.cuh"

namespace k3xb {

namespace {

using tcp::kBlockM;
using tcp::kThreads;

// B tiles of up to 128 rows keep 6 stages of 32 KB in flight (small token
// counts: the weight stream from HBM bounds the kernel); above 128 rows the
// tile grows to 256 rows with 4 stages of 48 KB, which halves the bytes a
// stage moves per FLOP once the contraction, fed from L2, is the bound.
template <uint32_t NB> struct LinCfg;
template <> struct LinCfg<128> { static constexpr uint32_t kStages = 6; };
template <> struct LinCfg<256> { static constexpr uint32_t kStages = 4; };

// One launch runs up to kMaxJobs products with the same input rows and K
// (the KDA block's q/k/v/g/f_a/b projections): job j is rows_j x K weights,
// its items are (128-row weight tile, token tile) pairs, weight-tile-major,
// after the items of jobs < j. The job index rides in the top 4 bits of the
// descriptor's weight row (tc_pipeline.cuh picks its tensor map).
constexpr uint32_t kMaxJobs = 8;

struct LinParams {
    uint32_t T, K, items, round_out, terms;
    uint32_t tpt, tiles;             // tokens per token tile, token tiles
    uint32_t njobs;
    uint32_t item_off[kMaxJobs + 1];
    uint32_t rows[kMaxJobs];
    float* out[kMaxJobs];            // [T][rows_j]
    int* error;
};

struct LinMaps {
    CUtensorMap w[kMaxJobs];
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
__device__ __forceinline__ uint4 lin_desc(uint32_t item, const LinParams& p) {
    uint32_t j = 0;
    while (j + 1 < p.njobs && item >= p.item_off[j + 1]) ++j;
    const uint32_t local = item - p.item_off[j];
    const uint32_t tile = local % p.tiles, mt = local / p.tiles;
    const uint32_t ntok = min(p.tpt, p.T - tile * p.tpt);
    return make_uint4((j << 28) | (mt * kBlockM), tile * p.tpt * p.terms,
                      ((p.terms * ntok + 15) / 16 * 16) | (ntok << 16), tile * p.tpt);
}

template <uint32_t NB>
__global__ void __launch_bounds__(kThreads, 1) linear_bf16_kernel(const __grid_constant__ LinMaps maps,
                                                                   const __grid_constant__ CUtensorMap map_x,
                                                                   const LinParams p) {
    extern __shared__ uint8_t smem_raw[];
    constexpr uint32_t S = LinCfg<NB>::kStages;
    auto& sm = tcp::smem_from<S, 1, NB>(smem_raw);
    auto get_desc = [&](uint32_t item) { return lin_desc(item, p); };
    auto epilogue = [&](const uint4& d, uint32_t tmem, uint32_t q, uint32_t lane) {
        const uint32_t terms = p.terms;
        const uint32_t used = terms * tcp::desc_ntok(d);
        const uint32_t lane_base = (32u * q) << 16;
        const uint32_t j = d.x >> 28;
        const uint32_t rows = p.rows[j];
        float* out = p.out[j];
        const uint32_t r = (d.x & 0x0fffffffu) + 32u * q + lane;
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
                if (r < rows) out[tok * rows + r] = p.round_out ? round_bf16(y) : y;
            }
        }
    };
    const uint8_t* none[1] = {nullptr};
    // one B box per stage: its height round16(tpt * terms) covers every item's MMA N
    tcp::Config cfg{p.K, p.items, 2 * NB, 0, 0, NB, 0, 0, 0, 0, (p.tpt * p.terms + 15) / 16 * 16};
    cfg.a_maps = p.njobs;
    tcp::run_pipeline<S, 1, true, 2>(sm, &maps.w[0], &maps.w[0], &map_x, cfg, none, nullptr, p.error, get_desc,
                                     epilogue);
}

}  // namespace

int make_byte_map(k3xb_ctx* ctx, void* map, const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_rows);

size_t linear_scratch_bytes(uint32_t T, uint32_t K) { return static_cast<size_t>(2) * T * K * 2 + 1024; }

template <uint32_t NB>
int launch_linear_nb(k3xb_ctx* ctx, const LinMaps& maps, const CUtensorMap& map_x, const LinParams& p) {
    static std::atomic<uint64_t> configured{0};   // per template instance
    const size_t smem = tcp::smem_bytes<LinCfg<NB>::kStages, 1, NB>();
    const int cst = configure_once(ctx, configured, [&]() -> int {
        K3XB_CUDA(ctx, cudaFuncSetAttribute(linear_bf16_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(smem)));
        return K3XB_OK;
    });
    if (cst) return cst;
    linear_bf16_kernel<NB><<<std::min<uint32_t>(ctx->sm_count, p.items), kThreads, smem, ctx->stream>>>(maps, map_x,
                                                                                                      p);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_linear_group(k3xb_ctx* ctx, const uint16_t* xterms, uint32_t terms, uint32_t T, uint32_t K,
                        const LinearJob* jobs, uint32_t njobs, int round_out) {
    if (K % 8) return fail(ctx, K3XB_INVALID_EXTENT, "bf16 linear needs K % 8 == 0");
    if (terms != 1 && terms != 2) return fail(ctx, K3XB_INVALID_EXTENT, "bf16 linear: 1 or 2 terms");
    if (!njobs || njobs > kMaxJobs) return fail(ctx, K3XB_INVALID_EXTENT, "bf16 linear: 1 to 8 products per launch");
    // token tiles: as few as the B tile allows, balanced (576 tokens -> 3 x 192)
    const uint32_t nb = terms * T > 128 ? 256u : 128u;
    const uint32_t cap = nb / terms;
    const uint32_t tiles = (T + cap - 1) / cap;
    const uint32_t tpt = (T + tiles - 1) / tiles;
    LinParams p{};
    p.T = T;
    p.K = K;
    p.round_out = round_out ? 1u : 0u;
    p.terms = terms;
    p.tpt = tpt;
    p.tiles = tiles;
    p.njobs = njobs;
    p.error = ctx->status_word;
    LinMaps maps;
    int st;
    uint64_t items = 0;
    for (uint32_t j = 0; j < njobs; ++j) {
        if (jobs[j].rows >= (1u << 28)) return fail(ctx, K3XB_INVALID_EXTENT, "bf16 linear: rows < 2^28");
        if ((st = make_byte_map(ctx, &maps.w[j], jobs[j].W, static_cast<uint64_t>(K) * 2, jobs[j].rows, 128)))
            return st;
        p.item_off[j] = static_cast<uint32_t>(items);
        p.rows[j] = jobs[j].rows;
        p.out[j] = jobs[j].out;
        items += static_cast<uint64_t>(tiles) * ((jobs[j].rows + kBlockM - 1) / kBlockM);
    }
    if (items >= (1ull << 31)) return fail(ctx, K3XB_INVALID_EXTENT, "bf16 linear: too many tiles");
    p.item_off[njobs] = static_cast<uint32_t>(items);
    p.items = static_cast<uint32_t>(items);
    CUtensorMap map_x;
    if ((st = make_byte_map(ctx, &map_x, xterms, static_cast<uint64_t>(K) * 2, static_cast<uint64_t>(terms) * T,
                            (tpt * terms + 15) / 16 * 16)))
        return st;
    return nb == 256 ? launch_linear_nb<256>(ctx, maps, map_x, p) : launch_linear_nb<128>(ctx, maps, map_x, p);
}

int launch_linear_terms(k3xb_ctx* ctx, const uint16_t* xterms, uint32_t terms, const uint16_t* W, uint32_t T,
                        uint32_t rows, uint32_t K, int round_out, float* out) {
    const LinearJob job{W, rows, out};
    return launch_linear_group(ctx, xterms, terms, T, K, &job, 1, round_out);
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
