// experts_tc.cu — (b)+(c) the MoE expert FFNs on tcgen05 tensor cores.
//
// Routed experts: block-scaled kind::mxf4 (E2M1 x E2M1, UE8M0 per-32
// scales, FP32 accumulation in TMEM). Weights are consumed in the
// reference's own MXFP4 layout — packed [rows][K/2] bytes, low nibble = even
// column (runtime/src/ops.cpp:32-55) — and TMA-loaded straight from HBM into
// 128B-swizzled shared memory (0.53 B per weight, no dequantisation). Only
// the E8M0 scales are re-laid once into the 128-row x 4-block atoms that
// tcgen05.cp moves into TMEM.
//
// The activation operand must be E2M1 as well, so each activation row is
// split exactly into `terms` E2M1 rows with their own E8M0 block scales
// (x = sum_t q_t + r, |r| shrinks >= 4x per term; 6 terms reproduce bf16
// inputs exactly and fp32 SwiGLU outputs to ~2^-12 of the block maximum).
// A token's terms are consecutive B rows (the MMA N dimension) and the
// epilogue adds their accumulator columns.
//
// Shared expert: kind::f16 (bf16 weights x bf16 activation terms).
//
// Launches per MoE layer (routed):
//   worklist       tiles of <= floor(NM/terms) tokens per expert group and
//                  one 16-byte descriptor per work item: (tile, 128-row
//                  m-tile) for gate/up, (tile, 256-row m-tile pair) for down
//   split_tokens   E2M1-term split of every hidden row, once per token
//   gather_gu      tile-major gate/up B operand + scale atoms
//   gateup         gate and up share the B tile; the epilogue applies
//                  SwiGLU / SiTU (official_moe.cpp:95-96) and stores the
//                  activation rows (coalesced floats)
//   split_act      the activation rows split into the down projection's
//                  E2M1 operand and scale atoms, all tiles in parallel
//   down           two weight tiles per item; the epilogue sums term
//                  columns, rounds to bf16 (official_moe.cpp:101) and
//                  scatters each row to its (token, slot) for the ordered
//                  combine (c)
#include "common.cuh"
#include "ep_sync.cuh"
#include "kernels.cuh"
#include "profile.cuh"
#include "tc_pipeline.cuh"

namespace k3xb {

namespace {

using tcp::kAtomBytes;
using tcp::kBlockM;
using tcp::kThreads;

// B-tile height NM (activation rows = tokens x terms per tile) is 64 or 112.
// With few tokens per expert (c2: ~3) a 64-row B slot leaves room for more
// weight stages in shared memory — bytes in flight are what bound an
// HBM-streaming GEMM. Both keep the two accumulators (gate and up, or the
// down projection's two weight tiles) double-buffered in TMEM, so the MMAs
// of one item overlap the epilogue of the previous one and the weight
// stream never waits for an epilogue: 112 is the widest N for which two
// buffers of two accumulators and the 24 block-scale columns fit in 512.
// TMEM columns (buffer b adds b * kStrideGU): accumulator 0 at 0,
// accumulator 1 at kColUp; block scales of A0, A1 and B at kColSf*.
template <uint32_t NM> struct RoutedCfg;
template <> struct RoutedCfg<64> {
    static constexpr uint32_t kStagesGU = 5, kAccbGU = 2;
    static constexpr uint32_t kColUp = 64, kStrideGU = 128;
    static constexpr uint32_t kColSfa0 = 256, kColSfa1 = 264, kColSfb = 272;
};
template <> struct RoutedCfg<112> {
    static constexpr uint32_t kStagesGU = 4, kAccbGU = 2;
    static constexpr uint32_t kColUp = 128, kStrideGU = 256;
    static constexpr uint32_t kColSfa0 = 112, kColSfa1 = 240, kColSfb = 368;   // gaps after N <= 112
};
constexpr uint32_t kStagesGU = 4;   // shared expert (kind::f16) pipelines
constexpr uint32_t kStagesD = 6;

constexpr uint32_t round16(uint32_t x) { return (x + 15u) / 16u * 16u; }

// ---------------------------------------------------------------------------
// one-time scale re-layout: [rows][K/32] -> atoms[rows/128][K/128][512]
__global__ void sf_relayout_kernel(const uint8_t* __restrict__ in, size_t rows, uint32_t K,
                                   uint8_t* __restrict__ out) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint32_t kb_count = K / 32;
    if (i >= rows * kb_count) return;
    const size_t r = i / kb_count;
    const uint32_t kb = static_cast<uint32_t>(i % kb_count);
    const size_t atom = (r / 128) * (K / 128) + kb / 4;
    const uint32_t rr = static_cast<uint32_t>(r % 128);
    out[atom * kAtomBytes + (rr % 32) * 16 + (rr / 32) * 4 + kb % 4] = in[i];
}

// ---------------------------------------------------------------------------
struct Tables {
    uint32_t* counts;       // [0] tiles, [1] gate/up items, [2] down items
    uint32_t* tile_ntok;
    uint32_t* tile_tok0;    // index into the plan's assignment arrays
    uint4* desc_gu;         // {a_row, b_row, n | ntok << 16, tok0}
    uint4* desc_d;
};

// One CTA of 1024 threads: one thread per group, Hillis-Steele scan of the
// per-group tile counts, then each group writes its tiles and descriptors
// (group-major, then m-tile, then n-tile, so the n-tiles that share a
// weight tile run back to back and the second read hits L2).
__global__ void __launch_bounds__(1024) worklist_kernel(const uint32_t* group_count, const uint32_t* group_offset,
                                                        const uint32_t* group_expert, uint32_t terms, uint32_t H,
                                                        uint32_t I, uint32_t nmax, Tables t) {
    __shared__ uint32_t scan[2][1024];
    __shared__ uint32_t tile_base[1025];
    const uint32_t ng = *group_count;
    const uint32_t tpt = nmax / terms;
    const uint32_t mt_gu = I / kBlockM, mt_d = (H + 2 * kBlockM - 1) / (2 * kBlockM);   // down: 256-row pairs
    const uint32_t g = threadIdx.x;
    scan[0][g] = g < ng ? (group_offset[g + 1] - group_offset[g] + tpt - 1) / tpt : 0u;
    __syncthreads();
    uint32_t src = 0;
    for (uint32_t off = 1; off < 1024; off <<= 1) {
        scan[src ^ 1u][g] = scan[src][g] + (g >= off ? scan[src][g - off] : 0u);
        src ^= 1u;
        __syncthreads();
    }
    tile_base[g + 1] = scan[src][g];
    if (g == 0) tile_base[0] = 0;
    __syncthreads();
    if (g == 0) {
        t.counts[0] = tile_base[ng];
        t.counts[1] = tile_base[ng] * mt_gu;
        t.counts[2] = tile_base[ng] * mt_d;
    }
    if (g >= ng) return;
    const uint32_t ntok_g = group_offset[g + 1] - group_offset[g];
    const uint32_t tb = tile_base[g], nt = tile_base[g + 1] - tb;
    const uint32_t e = group_expert[g];
    for (uint32_t j = 0; j < nt; ++j) {
        const uint32_t ntok = min(tpt, ntok_g - j * tpt), tok0 = group_offset[g] + j * tpt;
        t.tile_ntok[tb + j] = ntok;
        t.tile_tok0[tb + j] = tok0;
        const uint32_t nz = round16(ntok * terms) | (ntok << 16);
        for (uint32_t mt = 0; mt < mt_gu; ++mt)
            t.desc_gu[tb * mt_gu + mt * nt + j] = make_uint4(e * I + mt * kBlockM, (tb + j) * nmax, nz, tok0);
        for (uint32_t mt = 0; mt < mt_d; ++mt)
            t.desc_d[tb * mt_d + mt * nt + j] = make_uint4(e * H + mt * 2 * kBlockM, (tb + j) * nmax, nz, tok0);
    }
}

// ---------------------------------------------------------------------------
// Eight floats to eight E2M1 codes, nibble i = x[i]: the hardware
// conversion rounds to nearest even on the E2M1 grid and saturates at 6,
// which is e2m1_code's rounding. A negative value that rounds to zero comes
// out as code 8 (-0); the split writes 0 there, so the sign bit is kept only
// on nonzero magnitudes.
__device__ __forceinline__ uint32_t e2m1_pack8(const float* x) {
    uint32_t w;
    asm("{\n.reg .b8 b0, b1, b2, b3;\n"
        "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n"
        "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n"
        "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n"
        "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n"
        "mov.b32 %0, {b0, b1, b2, b3};\n}"
        : "=r"(w)
        : "f"(x[0]), "f"(x[1]), "f"(x[2]), "f"(x[3]), "f"(x[4]), "f"(x[5]), "f"(x[6]), "f"(x[7]));
    const uint32_t mag = w & 0x77777777u;
    const uint32_t nonzero = (mag + 0x77777777u) & 0x88888888u;   // bit 3 of each nibble with a magnitude
    return mag | (w & nonzero);
}

// One E2M1 term of a 32-element MX block held by one thread (bit-identical
// to a term of oracle/k3x_oracle.c:k3xo_e2m1_terms): the block maximum, its
// E8M0 exponent s, each element's code of v * 2^-s, and v replaced by the
// exact residual. Returns s; w gets the 16 packed bytes (low nibble = even
// element).
__device__ __forceinline__ int e2m1_term32(float (&v)[32], uint32_t (&w)[4]) {
    float m16[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) m16[i] = fmaxf(fabsf(v[i]), fabsf(v[i + 16]));
#pragma unroll
    for (int h = 8; h > 0; h >>= 1)
#pragma unroll
        for (int i = 0; i < h; ++i) m16[i] = fmaxf(m16[i], m16[i + h]);
    const float amax = m16[0];
    const int s = amax > 0.0f ? e2m1_block_exponent(amax) : 0;
    const float inv = exp2i(-s), scale = exp2i(s);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        float x[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = v[8 * k + i] * inv;
        w[k] = e2m1_pack8(x);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t c = (w[k] >> (4 * i)) & 15u;
            const float qv = e2m1_magnitude(c & 7u) * scale;
            v[8 * k + i] = (c & 8u) ? __fadd_rn(v[8 * k + i], qv) : __fsub_rn(v[8 * k + i], qv);
        }
    }
    return s;
}

// E2M1-term split (bit-identical to oracle/k3x_oracle.c:k3xo_e2m1_terms) of
// one 32-element MX block held by one thread. Term t's 16 packed bytes go to
// rows[t * row_stride], its scale byte to scales[t * scale_stride].
__device__ __forceinline__ void split_block32(float (&v)[32], uint32_t terms, uint8_t* rows, size_t row_stride,
                                              uint8_t* scales, size_t scale_stride) {
    for (uint32_t t = 0; t < terms; ++t) {
        uint32_t w[4];
        const int s = e2m1_term32(v, w);
        *reinterpret_cast<uint4*>(rows + t * row_stride) = make_uint4(w[0], w[1], w[2], w[3]);
        scales[t * scale_stride] = static_cast<uint8_t>(s + 127);
    }
}

__device__ __forceinline__ void load_block32(const float* src, float (&v)[32]) {
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
        const float4 q = *reinterpret_cast<const float4*>(src + i);
        v[i] = q.x; v[i + 1] = q.y; v[i + 2] = q.z; v[i + 3] = q.w;
    }
}

// Every token's hidden row once: tsplit[t][term][H/2], tsf[t][term][H/32].
// One thread per (row, 32-element block); rows are floats, or bf16 words
// when hidden16 is given (the expert-parallel receive window).
__global__ void __launch_bounds__(256) split_tokens_kernel(const float* __restrict__ hidden,
                                                           const uint16_t* __restrict__ hidden16, uint32_t T,
                                                           uint32_t H, uint32_t terms,
                                                           uint8_t* __restrict__ tsplit,
                                                           uint8_t* __restrict__ tsf) {
    const uint32_t kbc = H / 32;
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<size_t>(T) * kbc) return;
    const uint32_t t = static_cast<uint32_t>(i / kbc), kb = static_cast<uint32_t>(i % kbc);
    const size_t at = static_cast<size_t>(t) * H + kb * 32;
    float v[32];
    if (hidden16) {
#pragma unroll
        for (int k = 0; k < 32; k += 8) {
            const uint4 q = *reinterpret_cast<const uint4*>(hidden16 + at + k);
            const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                v[k + 2 * m] = __uint_as_float(w[m] << 16);
                v[k + 2 * m + 1] = __uint_as_float(w[m] & 0xffff0000u);
            }
        }
    } else {
        load_block32(hidden + at, v);
    }
    const size_t row = static_cast<size_t>(t) * terms;
    split_block32(v, terms, tsplit + row * (H / 2) + kb * 16, H / 2, tsf + row * kbc + kb, kbc);
}

// Tile-major gate/up B operand (+ scale atoms) gathered from the per-token
// split; zero rows pad the MMA N to a 16-multiple.
__global__ void __launch_bounds__(256) gather_gu_kernel(const uint8_t* __restrict__ tsplit,
                                                        const uint8_t* __restrict__ tsf, uint32_t H,
                                                        const uint32_t* __restrict__ assign_token, Tables tb,
                                                        uint32_t terms, uint32_t nmax, uint8_t* __restrict__ b,
                                                        uint8_t* __restrict__ sfb) {
    const uint32_t tile = blockIdx.x;
    if (tile >= tb.counts[0]) return;
    const uint32_t ntok = tb.tile_ntok[tile], tok0 = tb.tile_tok0[tile];
    const uint32_t used = ntok * terms, n = round16(used);
    const uint32_t kbc = H / 32;
    const size_t row_stride = H / 2;
    uint8_t* base = b + static_cast<size_t>(tile) * nmax * row_stride;
    uint8_t* atoms = sfb + static_cast<size_t>(tile) * (kbc / 4) * kAtomBytes;
    for (uint32_t i = threadIdx.x; i < n * kbc; i += blockDim.x) {
        const uint32_t r = i / kbc, v = i % kbc;
        uint4 val = make_uint4(0, 0, 0, 0);
        uint8_t sf = 127;
        if (r < used) {
            const size_t src = static_cast<size_t>(assign_token[tok0 + r / terms]) * terms + r % terms;
            val = *reinterpret_cast<const uint4*>(tsplit + src * row_stride + v * 16);
            sf = tsf[src * kbc + v];
        }
        *reinterpret_cast<uint4*>(base + static_cast<size_t>(r) * row_stride + v * 16) = val;
        atoms[(v / 4) * kAtomBytes + (r % 32) * 16 + (r / 32) * 4 + v % 4] = sf;
    }
}

// The down projection's B operand from the activation rows (gate/up
// epilogue output): per tile, token j's row becomes `terms` E2M1 rows
// j*terms + t with their scale atoms, and rows [ntok*terms, n) are zero,
// n the tile's MMA N. One thread per (token, 32-element block of I).
__global__ void __launch_bounds__(256) split_act_kernel(const float* __restrict__ act, Tables tb, uint32_t I,
                                                        uint32_t terms, uint32_t tpt, uint32_t nmax,
                                                        uint8_t* __restrict__ b, uint8_t* __restrict__ sfb) {
    const uint32_t tile = blockIdx.y;
    if (tile >= tb.counts[0]) return;
    const uint32_t ntok = tb.tile_ntok[tile], used = ntok * terms, n = round16(used);
    const uint32_t kbc = I / 32;
    const size_t row_stride = I / 2;
    uint8_t* base = b + static_cast<size_t>(tile) * nmax * row_stride;
    uint8_t* atoms = sfb + static_cast<size_t>(tile) * (I / 128) * kAtomBytes;
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < ntok * kbc; i += stride) {
        const uint32_t j = i / kbc, kb = i % kbc;
        float v[32];
        load_block32(act + (static_cast<size_t>(tile) * tpt + j) * I + kb * 32, v);
        // term t of token j is MMA row j*terms + t: bytes at row * row_stride + kb * 16, its scale in
        // atom kb / 4 at byte (row % 32) * 16 + (row / 32) * 4 + kb % 4
        for (uint32_t t = 0; t < terms; ++t) {
            uint32_t w[4];
            const int s = e2m1_term32(v, w);
            const uint32_t row = j * terms + t;
            *reinterpret_cast<uint4*>(base + static_cast<size_t>(row) * row_stride + kb * 16) =
                make_uint4(w[0], w[1], w[2], w[3]);
            atoms[(kb / 4) * kAtomBytes + (row % 32) * 16 + (row / 32) * 4 + kb % 4] = static_cast<uint8_t>(s + 127);
        }
    }
    // padding rows of the MMA N: zero codes, unit scales
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < (n - used) * kbc; i += stride) {
        const uint32_t row = used + i / kbc, kb = i % kbc;
        *reinterpret_cast<uint4*>(base + static_cast<size_t>(row) * row_stride + kb * 16) = make_uint4(0, 0, 0, 0);
        atoms[(kb / 4) * kAtomBytes + (row % 32) * 16 + (row / 32) * 4 + kb % 4] = 127;
    }
}

// ---------------------------------------------------------------------------
__device__ __forceinline__ float activate(float g, float u, int act, float beta, float lbeta) {
    // SwiGLU: (g * sigmoid(g)) * u; SiTU: runtime/src/ops.cpp:20-30.
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
    if (act == K3XB_ACT_SITU) {
        const float bg = __fmul_rn(__fmul_rn(beta, tanhf(__fdiv_rn(g, beta))), sig);
        const float bu = lbeta > 0.0f ? __fmul_rn(lbeta, tanhf(__fdiv_rn(u, lbeta))) : u;
        return __fmul_rn(bg, bu);
    }
    return __fmul_rn(__fmul_rn(g, sig), u);
}

struct GuParams {
    const uint4* desc;
    const uint32_t* n_items;
    const uint8_t* sfa_gate;
    const uint8_t* sfa_up;
    const uint8_t* sfb;       // gather_gu scales
    float* act;               // epilogue output: act[tile * tpt + j][I], token j of the tile
    uint32_t tpt;             // tokens per tile (the act rows a tile owns)
    uint32_t H, I, terms;
    int act_kind;
    float beta, lbeta;
    int* error;
};

struct DParams {
    const uint4* desc;
    const uint32_t* n_items;
    const uint32_t* assign_token;
    const uint32_t* assign_slot;
    const uint8_t* sfa;
    const uint8_t* sfb;
    float* slot_out;
    uint32_t H, I, terms, top_k;
    int* error;
    uint32_t rowblocks;       // 128-row blocks of the stacked down weights (E * H / 128)
    uint16_t* slot_out16;     // when set: bf16 words instead of slot_out floats
    EpTarget ep;              // when ep.world: rows go straight to their home ranks' windows
};

// TMEM columns of the accumulators (routed: RoutedCfg; shared expert: gate
// at 0, up at 128).
constexpr uint32_t kColAccGate = 0, kColAccUp = 128;

template <uint32_t NM>
__global__ void __launch_bounds__(kThreads, 1) gateup_kernel(const __grid_constant__ CUtensorMap map_gate,
                                                              const __grid_constant__ CUtensorMap map_up,
                                                              const __grid_constant__ CUtensorMap map_b,
                                                              const GuParams p) {
    using RC = RoutedCfg<NM>;
    extern __shared__ uint8_t smem_raw[];
    auto& sm = tcp::smem_from<RC::kStagesGU, 2, NM>(smem_raw);
    const uint32_t terms = p.terms;
    const uint32_t mtc = p.I / kBlockM;
    auto get_desc = [&](uint32_t item) { return __ldg(p.desc + item); };
    // The epilogue adds each token's term columns, applies SwiGLU / SiTU and
    // stores the activation row (a warp's 32 rows of I are 32 consecutive
    // floats); split_act_kernel then builds the down projection's operand.
    auto epilogue = [&](const uint4& d, uint32_t tmem, uint32_t q, uint32_t lane) {
        const uint32_t tile = d.y / NM, mt = (d.x / kBlockM) % mtc;
        const uint32_t ntok = tcp::desc_ntok(d);
        const uint32_t used = ntok * terms;
        const uint32_t lane_base = (32u * q) << 16;
        float* arow = p.act + static_cast<size_t>(tile) * p.tpt * p.I + mt * kBlockM + 32u * q + lane;
        float gs = 0.0f, us = 0.0f;
        uint32_t tcount = 0, j = 0;
        for (uint32_t c0 = 0; c0 < used; c0 += 16) {
            float vg[16], vu[16];
            tc::tmem_ld16(tmem + lane_base + kColAccGate + c0, vg);
            tc::tmem_ld16(tmem + lane_base + RC::kColUp + c0, vu);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if (c0 + i >= used) break;
                gs = __fadd_rn(gs, vg[i]);
                us = __fadd_rn(us, vu[i]);
                if (++tcount < terms) continue;
                arow[static_cast<size_t>(j) * p.I] = activate(gs, us, p.act_kind, p.beta, p.lbeta);
                gs = us = 0.0f;
                tcount = 0;
                ++j;
            }
        }
    };
    const uint8_t* sfa[2] = {p.sfa_gate, p.sfa_up};
    const tcp::Config cfg{p.H, *p.n_items, 512, kColAccGate, RC::kColUp, RC::kStrideGU, RC::kColSfa0, RC::kColSfa1,
                          RC::kColSfb, 0, NM};
    tcp::run_pipeline<RC::kStagesGU, 2, false, RC::kAccbGU>(sm, &map_gate, &map_up, &map_b, cfg, sfa, p.sfb,
                                                            p.error, get_desc, epilogue);
}

// Down projection: an item is a PAIR of 128-row weight tiles (rows r0 and
// r0 + 128 of one expert) sharing the activation tile, so a pipeline stage
// moves 32 KB of weights per handful of TMA instructions. When H is an odd
// multiple of 128 the second tile of an expert's last pair is discarded.
template <uint32_t NM>
__global__ void __launch_bounds__(kThreads, 1) down_kernel(const __grid_constant__ CUtensorMap map_down,
                                                            const __grid_constant__ CUtensorMap map_b,
                                                            const DParams p) {
    using RC = RoutedCfg<NM>;
    extern __shared__ uint8_t smem_raw[];
    auto& sm = tcp::smem_from<RC::kStagesGU, 2, NM>(smem_raw);
    const uint32_t terms = p.terms;
    auto get_desc = [&](uint32_t item) { return __ldg(p.desc + item); };
    auto epilogue = [&](const uint4& d, uint32_t tmem, uint32_t q, uint32_t lane) {
        const uint32_t r0 = d.x % p.H, tok0 = d.w;
        const bool second = r0 + kBlockM < p.H;
        const uint32_t ntok = tcp::desc_ntok(d);
        const uint32_t used = ntok * terms;
        const uint32_t lane_base = (32u * q) << 16;
        const uint32_t h0 = r0 + 32u * q + lane, h1 = h0 + kBlockM;
        // destination rows of up to 32 tokens per round trip (lane j holds token j's).
        // Expert parallel: received row r is token r % home_rows of home rank
        // r / home_rows, packed as rank << 24 | (token * top_k + slot)
        auto fetch_dst = [&](uint32_t j0) {
            const uint32_t a = tok0 + j0 + lane;
            if (j0 + lane >= ntok) return 0u;
            const uint32_t row = __ldg(p.assign_token + a), slot = __ldg(p.assign_slot + a);
            if (!p.ep.world) return row * p.top_k + slot;
            const uint32_t g = row / p.ep.home_rows;
            return g << 24 | ((row - g * p.ep.home_rows) * p.top_k + slot);
        };
        uint32_t dsts = fetch_dst(0);
        float y0 = 0.0f, y1 = 0.0f;
        uint32_t tcount = 0, j = 0;
        for (uint32_t c0 = 0; c0 < used; c0 += 16) {
            float v0[16], v1[16];
            tc::tmem_ld16(tmem + lane_base + kColAccGate + c0, v0);
            if (second) tc::tmem_ld16(tmem + lane_base + RC::kColUp + c0, v1);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if (c0 + i >= used) break;
                y0 = __fadd_rn(y0, v0[i]);
                if (second) y1 = __fadd_rn(y1, v1[i]);
                if (++tcount < terms) continue;
                if (j % 32 == 0 && j) dsts = fetch_dst(j);
                const uint32_t packed = __shfl_sync(0xffffffffu, dsts, j % 32);
                if (p.ep.world) {   // a store into the home rank's window (NVLink for a peer)
                    uint16_t* y = reinterpret_cast<uint16_t*>(p.ep.win[packed >> 24] + p.ep.y_off) +
                                  static_cast<size_t>(packed & 0xffffffu) * p.H;
                    y[h0] = encode_bf16(y0);
                    if (second) y[h1] = encode_bf16(y1);
                    y0 = y1 = 0.0f;
                    tcount = 0;
                    ++j;
                    continue;
                }
                const size_t dst = packed;
                if (p.slot_out16) {
                    p.slot_out16[dst * p.H + h0] = encode_bf16(y0);
                    if (second) p.slot_out16[dst * p.H + h1] = encode_bf16(y1);
                } else {
                    p.slot_out[dst * p.H + h0] = round_bf16(y0);
                    if (second) p.slot_out[dst * p.H + h1] = round_bf16(y1);
                }
                y0 = y1 = 0.0f;
                tcount = 0;
                ++j;
            }
        }
    };
    const uint8_t* sfa[2] = {p.sfa, p.sfa};
    const tcp::Config cfg{p.I, *p.n_items, 512, kColAccGate, RC::kColUp, RC::kStrideGU, RC::kColSfa0, RC::kColSfa1,
                          RC::kColSfb, kBlockM, NM, p.rowblocks};
    tcp::run_pipeline<RC::kStagesGU, 2, false, RC::kAccbGU>(sm, &map_down, &map_down, &map_b, cfg, sfa, p.sfb,
                                                            p.error, get_desc, epilogue);
    // Expert parallel: the last CTA to finish tells every home rank that this
    // rank's outputs for the call have landed (every thread's stores first)
    if (p.ep.world) ep_signal_grid_done(p.ep.done, p.ep.win, p.ep.flag_off, p.ep.rank, p.ep.world, p.ep.epoch);
}

// ---------------------------------------------------------------------------
// Shared expert on kind::f16 (shared_ffn, official_moe.cpp:105-117): bf16
// weights, FP32 accumulation. Activations enter as two bf16 terms per token
// (hi = bf16(x), lo = bf16(x - hi)), rows token*2 + t, so any float input is
// carried to ~16 bits and bf16-valued inputs exactly. Tiles are 64 tokens
// (N = 128). gate/up epilogue: g, u rounded to bf16 (bf16_matvec,
// official_moe.cpp:56), activation, split into the down operand's two
// terms. down epilogue: sum of the two term columns, rounded to bf16.
constexpr uint32_t kSharedTok = 64;

struct SharedParams {
    uint32_t T, H, Is, items;
    uint16_t* b_down;   // [2T][Is] bf16 words
    float* out;         // [T][H]
    int act;
    float beta, lbeta;
    int* error;
};

__device__ __forceinline__ uint16_t bf16_word(float v) { return static_cast<uint16_t>(__float_as_uint(v) >> 16); }

__global__ void split_bf16_kernel(const float* __restrict__ x, size_t n, uint32_t H, uint16_t* __restrict__ out) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const size_t t = i / H, h = i % H;
    const float hi = round_bf16(x[i]);
    const float lo = round_bf16(__fsub_rn(x[i], hi));
    out[(2 * t) * H + h] = bf16_word(hi);
    out[(2 * t + 1) * H + h] = bf16_word(lo);
}

__device__ __forceinline__ uint4 shared_desc(uint32_t item, uint32_t mtc, uint32_t T) {
    const uint32_t tile = item / mtc, mt = item % mtc;
    const uint32_t ntok = min(kSharedTok, T - tile * kSharedTok);
    return make_uint4(mt * kBlockM, tile * 2 * kSharedTok, round16(2 * ntok) | (ntok << 16), tile * kSharedTok);
}

__global__ void __launch_bounds__(kThreads, 1) shared_gateup_kernel(const __grid_constant__ CUtensorMap map_gate,
                                                                     const __grid_constant__ CUtensorMap map_up,
                                                                     const __grid_constant__ CUtensorMap map_x,
                                                                     const SharedParams p) {
    extern __shared__ uint8_t smem_raw[];
    auto& sm = tcp::smem_from<kStagesGU, 2>(smem_raw);
    const uint32_t mtc = p.Is / kBlockM;
    auto get_desc = [&](uint32_t item) { return shared_desc(item, mtc, p.T); };
    auto epilogue = [&](const uint4& d, uint32_t tmem, uint32_t q, uint32_t lane) {
        const uint32_t used = 2 * tcp::desc_ntok(d);
        const uint32_t lane_base = (32u * q) << 16;
        const uint32_t m = d.x + 32u * q + lane;
        for (uint32_t c0 = 0; c0 < used; c0 += 16) {
            float vg[16], vu[16];
            tc::tmem_ld16(tmem + lane_base + kColAccGate + c0, vg);
            tc::tmem_ld16(tmem + lane_base + kColAccUp + c0, vu);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; i += 2) {
                if (c0 + i >= used) break;
                const float g = round_bf16(__fadd_rn(vg[i], vg[i + 1]));
                const float u = round_bf16(__fadd_rn(vu[i], vu[i + 1]));
                const float a = activate(g, u, p.act, p.beta, p.lbeta);
                const float hi = round_bf16(a);
                const float lo = round_bf16(__fsub_rn(a, hi));
                const size_t tok = d.w + (c0 + i) / 2;
                p.b_down[(2 * tok) * p.Is + m] = bf16_word(hi);
                p.b_down[(2 * tok + 1) * p.Is + m] = bf16_word(lo);
            }
        }
    };
    const uint8_t* none[2] = {nullptr, nullptr};
    const tcp::Config cfg{p.H, p.items, 256, kColAccGate, kColAccUp, 0, 0, 0, 0, 0, 2 * kSharedTok};
    tcp::run_pipeline<kStagesGU, 2, true, 1>(sm, &map_gate, &map_up, &map_x, cfg, none, nullptr, p.error, get_desc,
                                             epilogue);
}

__global__ void __launch_bounds__(kThreads, 1) shared_down_kernel(const __grid_constant__ CUtensorMap map_down,
                                                                   const __grid_constant__ CUtensorMap map_b,
                                                                   const SharedParams p) {
    extern __shared__ uint8_t smem_raw[];
    auto& sm = tcp::smem_from<kStagesD, 1>(smem_raw);
    const uint32_t mtc = p.H / kBlockM;
    auto get_desc = [&](uint32_t item) { return shared_desc(item, mtc, p.T); };
    auto epilogue = [&](const uint4& d, uint32_t tmem, uint32_t q, uint32_t lane) {
        const uint32_t used = 2 * tcp::desc_ntok(d);
        const uint32_t lane_base = (32u * q) << 16;
        const uint32_t h = d.x + 32u * q + lane;
        for (uint32_t c0 = 0; c0 < used; c0 += 16) {
            float v[16];
            tc::tmem_ld16(tmem + lane_base + kColAccGate + c0, v);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; i += 2) {
                if (c0 + i >= used) break;
                const size_t tok = d.w + (c0 + i) / 2;
                p.out[tok * p.H + h] = round_bf16(__fadd_rn(v[i], v[i + 1]));
            }
        }
    };
    const uint8_t* none[1] = {nullptr};
    const tcp::Config cfg{p.Is, p.items, 256, kColAccGate, kColAccGate, 128, 0, 0, 0, 0, 2 * kSharedTok};
    tcp::run_pipeline<kStagesD, 1, true, 2>(sm, &map_down, &map_down, &map_b, cfg, none, nullptr, p.error, get_desc,
                                            epilogue);
}

// ---------------------------------------------------------------------------
// host side

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct TcState {
    EncodeFn encode = nullptr;
    bool configured = false;
    bool configured_shared = false;
};

TcState* state_of(k3xb_ctx* ctx) {
    if (!ctx->mxf4_state) ctx->mxf4_state = new TcState();
    return static_cast<TcState*>(ctx->mxf4_state);
}

int get_encode(k3xb_ctx* ctx, EncodeFn* out) {
    TcState* s = state_of(ctx);
    if (!s->encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        K3XB_CUDA(ctx, cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (!fn || q != cudaDriverEntryPointSuccess)
            return fail(ctx, K3XB_BACKEND_UNAVAILABLE, "cuTensorMapEncodeTiled unavailable");
        s->encode = reinterpret_cast<EncodeFn>(fn);
    }
    *out = s->encode;
    return K3XB_OK;
}

// 2-D byte tensor [rows][row_bytes], box {128 B, box_rows}, 128B swizzle.
// Every TMA x coordinate used with these maps is a multiple of 128 bytes.
int make_map(k3xb_ctx* ctx, CUtensorMap* map, const void* base, uint64_t row_bytes, uint64_t rows,
             uint32_t box_rows) {
    EncodeFn encode;
    int st = get_encode(ctx, &encode);
    if (st) return st;
    if (reinterpret_cast<uintptr_t>(base) % 16 || row_bytes % 16)
        return fail(ctx, K3XB_INVALID_EXTENT, "tensor-core operands need 16-byte aligned rows");
    const cuuint64_t dims[2] = {row_bytes, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {128, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(ctx, K3XB_BACKEND_UNAVAILABLE, "cuTensorMapEncodeTiled failed");
    return K3XB_OK;
}

int relayout(k3xb_ctx* ctx, const uint8_t* scales, size_t rows, uint32_t K, uint8_t* out) {
    const size_t n = rows * (K / 32);
    sf_relayout_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, ctx->stream>>>(scales, rows, K, out);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

struct Layout {
    uint32_t terms, nmax, tpt, max_tiles, mt_gu, mt_d;
    size_t b_gu, sfb_gu, b_d, sfb_d;
    size_t sf_gate, sf_up, sf_down;   // per-call re-laid scales (0 when prepared)
    size_t tsplit, tsf;               // per-token E2M1 split of the hidden rows
    size_t act;                       // activation rows [max_tiles * tpt][I] (floats)
};

Layout layout_of(const k3xb_moe_layer& L, uint32_t T, uint32_t terms) {
    Layout l{};
    l.terms = terms;
    const uint32_t assigns = T * L.top_k;
    // 64-row B tiles when an average expert gets at most 64 rows of terms
    // (c2: ~3 tokens x 6 terms), otherwise 112
    const uint32_t avg_rows = (assigns + L.experts - 1) / L.experts * l.terms;
    l.nmax = (avg_rows <= 64 && l.terms <= 64) ? 64u : 112u;
    l.tpt = l.nmax / l.terms;
    l.max_tiles = std::min(L.experts, assigns) + (assigns + l.tpt - 1) / l.tpt;
    l.mt_gu = L.inter / kBlockM;
    l.mt_d = (L.hidden + 2 * kBlockM - 1) / (2 * kBlockM);
    l.b_gu = static_cast<size_t>(l.max_tiles) * l.nmax * (L.hidden / 2);
    l.sfb_gu = static_cast<size_t>(l.max_tiles) * (L.hidden / 128) * kAtomBytes;
    l.b_d = static_cast<size_t>(l.max_tiles) * l.nmax * (L.inter / 2);
    l.sfb_d = static_cast<size_t>(l.max_tiles) * (L.inter / 128) * kAtomBytes;
    const size_t sf_gu = static_cast<size_t>(L.experts) * L.inter * (L.hidden / 32);
    l.sf_gate = L.gate_scales_tc ? 0 : sf_gu;
    l.sf_up = L.up_scales_tc ? 0 : sf_gu;
    l.sf_down = L.down_scales_tc ? 0 : sf_gu;
    l.tsplit = static_cast<size_t>(T) * l.terms * (L.hidden / 2);
    l.tsf = static_cast<size_t>(T) * l.terms * (L.hidden / 32);
    l.act = static_cast<size_t>(l.max_tiles) * l.tpt * L.inter;
    return l;
}

struct Buffers {
    Tables tb;
    uint8_t *b_gu, *sfb_gu, *b_d, *sfb_d, *sf[3], *tsplit, *tsf;
    float* act;
};

template <typename A>
void carve(A& a, const Layout& l, Buffers* out) {
    Buffers tmp;
    Buffers& r = out ? *out : tmp;
    r.tb.counts = a.template take<uint32_t>(4);
    r.tb.tile_ntok = a.template take<uint32_t>(l.max_tiles);
    r.tb.tile_tok0 = a.template take<uint32_t>(l.max_tiles);
    r.tb.desc_gu = a.template take<uint4>(static_cast<size_t>(l.max_tiles) * l.mt_gu);
    r.tb.desc_d = a.template take<uint4>(static_cast<size_t>(l.max_tiles) * l.mt_d);
    r.b_gu = a.template take<uint8_t>(l.b_gu, 1024);
    r.sfb_gu = a.template take<uint8_t>(l.sfb_gu, 1024);
    r.b_d = a.template take<uint8_t>(l.b_d, 1024);
    r.sfb_d = a.template take<uint8_t>(l.sfb_d, 1024);
    r.sf[0] = a.template take<uint8_t>(l.sf_gate, 1024);
    r.sf[1] = a.template take<uint8_t>(l.sf_up, 1024);
    r.sf[2] = a.template take<uint8_t>(l.sf_down, 1024);
    r.tsplit = a.template take<uint8_t>(l.tsplit, 1024);
    r.tsf = a.template take<uint8_t>(l.tsf, 1024);
    r.act = a.template take<float>(l.act, 1024);
}

struct SplitArgs {
    const float* act;
    Tables tb;
    uint32_t I, terms, tpt, nmax;
    uint8_t *b, *sfb;
    uint32_t max_tiles;
};

template <uint32_t NM>
int launch_routed(k3xb_ctx* ctx, const CUtensorMap& map_gate, const CUtensorMap& map_up, const CUtensorMap& map_bgu,
                  const CUtensorMap& map_down, const CUtensorMap& map_bd, const GuParams& gp, const SplitArgs& sa,
                  const DParams& dp) {
    using RC = RoutedCfg<NM>;
    const size_t smem_gu = tcp::smem_bytes<RC::kStagesGU, 2, NM>();
    const size_t smem_d = tcp::smem_bytes<RC::kStagesGU, 2, NM>();
    static std::atomic<uint64_t> configured{0};   // per template instance
    const int cst = configure_once(ctx, configured, [&]() -> int {
        K3XB_CUDA(ctx, cudaFuncSetAttribute(gateup_kernel<NM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(smem_gu)));
        K3XB_CUDA(ctx, cudaFuncSetAttribute(down_kernel<NM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(smem_d)));
        return K3XB_OK;
    });
    if (cst) return cst;
    {
        PhaseScope ph(ctx, K3XB_PHASE_EXPERT_GATEUP);
        gateup_kernel<NM><<<ctx->sm_count, kThreads, smem_gu, ctx->stream>>>(map_gate, map_up, map_bgu, gp);
        K3XB_LAUNCHED(ctx);
    }
    // the down projection's phase: its operand from the activation rows, then the GEMM
    PhaseScope ph(ctx, K3XB_PHASE_EXPERT_DOWN);
    {
        // one thread per (token, 32-block) of a tile
        const uint32_t per_tile = (sa.tpt * (sa.I / 32) + 255u) / 256u;
        split_act_kernel<<<dim3(per_tile, sa.max_tiles), 256, 0, ctx->stream>>>(sa.act, sa.tb, sa.I, sa.terms, sa.tpt,
                                                                               sa.nmax, sa.b, sa.sfb);
        K3XB_LAUNCHED(ctx);
    }
    down_kernel<NM><<<ctx->sm_count, kThreads, smem_d, ctx->stream>>>(map_down, map_bd, dp);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

}  // namespace

int make_byte_map(k3xb_ctx* ctx, void* map, const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_rows) {
    return make_map(ctx, static_cast<CUtensorMap*>(map), base, row_bytes, rows, box_rows);
}

int prepare_mxfp4_scales(k3xb_ctx* ctx, const uint8_t* scales, size_t rows, size_t cols, uint8_t* out) {
    if (!scales || !out || !rows || rows % 128 || !cols || cols % 128)
        return fail(ctx, K3XB_INVALID_MXFP4, "prepare scales: rows and cols must be multiples of 128");
    return relayout(ctx, scales, rows, static_cast<uint32_t>(cols), out);
}

uint32_t mxf4_default_terms(uint64_t assignments, uint32_t experts) {
    // Few tokens per expert: the expert GEMM streams weights from HBM and the
    // MMA has slack, so the exact 6-term split costs nothing. From 12 tokens
    // per expert on, the operand and MMA work grow with the terms, and 4
    // terms keep the outputs within the north-star tolerance.
    const uint64_t avg = experts ? (assignments + experts - 1) / experts : 0;
    return avg >= 12 ? 4u : 6u;
}

uint32_t resolve_terms(const k3xb_moe_layer& L, uint32_t T) {
    return L.act_terms > 0 ? static_cast<uint32_t>(L.act_terms)
                           : mxf4_default_terms(static_cast<uint64_t>(T) * L.top_k, L.experts);
}

// With the default term count either split may be chosen at launch (an
// expert-parallel rank resolves it from the whole batch): room for both.
size_t mxf4_scratch_bytes(const k3xb_moe_layer& L, uint32_t T) {
    if (L.engine != K3XB_ENGINE_MXF4) return 0;
    auto bytes = [&](uint32_t terms) {
        Sizer s;
        carve(s, layout_of(L, T, terms), nullptr);
        return s.used;
    };
    const size_t need = L.act_terms > 0 ? bytes(static_cast<uint32_t>(L.act_terms)) : std::max(bytes(4), bytes(6));
    return need + 1024;
}

void set_mxf4_scratch(k3xb_ctx* ctx, void* region) { ctx->mxf4_scratch = region; }

int launch_mxf4_experts(k3xb_ctx* ctx, const k3xb_moe_layer& L, const float* hidden, uint32_t T,
                        const k3xb_plan& plan, float* slot_out, uint16_t* slot_out16, const EpTarget* ep,
                        const uint16_t* hidden16) {
    const uint32_t H = L.hidden, I = L.inter;
    if (H % 128 || I % 128)
        return fail(ctx, K3XB_INVALID_EXTENT, "MXF4 engine needs hidden and inter multiples of 128");
    if (L.act_terms < 0 || L.act_terms > 16)
        return fail(ctx, K3XB_INVALID_EXTENT, "act_terms must be in [1, 16] (0 = the library default)");
    if (L.experts > 1024) return fail(ctx, K3XB_INVALID_EXTENT, "MXF4 engine supports <= 1024 experts");
    const Layout l = layout_of(L, T, resolve_terms(L, T));
    if (static_cast<uint64_t>(l.max_tiles) * l.nmax >= (1ull << 31))
        return fail(ctx, K3XB_INVALID_EXTENT, "MXF4 work list too large");
    int st;
    Carver c(reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(ctx->mxf4_scratch) + 1023) & ~uintptr_t(1023)));
    Buffers bf;
    carve(c, l, &bf);
    PhaseScope prep(ctx, K3XB_PHASE_EXPERT_PREP);
    const uint8_t* sfa_gate = L.gate_scales_tc;
    const uint8_t* sfa_up = L.up_scales_tc;
    const uint8_t* sfa_down = L.down_scales_tc;
    const size_t rows_gu = static_cast<size_t>(L.experts) * I, rows_d = static_cast<size_t>(L.experts) * H;
    if (!sfa_gate) { if ((st = relayout(ctx, L.gate_scales, rows_gu, H, bf.sf[0]))) return st; sfa_gate = bf.sf[0]; }
    if (!sfa_up) { if ((st = relayout(ctx, L.up_scales, rows_gu, H, bf.sf[1]))) return st; sfa_up = bf.sf[1]; }
    if (!sfa_down) { if ((st = relayout(ctx, L.down_scales, rows_d, I, bf.sf[2]))) return st; sfa_down = bf.sf[2]; }

    CUtensorMap map_gate, map_up, map_down, map_bgu, map_bd;
    if ((st = make_map(ctx, &map_gate, L.gate_packed, H / 2, static_cast<uint64_t>(L.experts) * I, 128))) return st;
    if ((st = make_map(ctx, &map_up, L.up_packed, H / 2, static_cast<uint64_t>(L.experts) * I, 128))) return st;
    if ((st = make_map(ctx, &map_down, L.down_packed, I / 2, static_cast<uint64_t>(L.experts) * H, 128))) return st;
    if ((st = make_map(ctx, &map_bgu, bf.b_gu, H / 2, static_cast<uint64_t>(l.max_tiles) * l.nmax, l.nmax))) return st;
    if ((st = make_map(ctx, &map_bd, bf.b_d, I / 2, static_cast<uint64_t>(l.max_tiles) * l.nmax, l.nmax))) return st;

    worklist_kernel<<<1, 1024, 0, ctx->stream>>>(plan.group_count, plan.group_offset, plan.group_expert, l.terms, H,
                                                 I, l.nmax, bf.tb);
    K3XB_LAUNCHED(ctx);
    {
        const size_t n = static_cast<size_t>(T) * (H / 32);
        split_tokens_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, ctx->stream>>>(hidden, hidden16, T, H,
                                                                                          l.terms, bf.tsplit, bf.tsf);
        K3XB_LAUNCHED(ctx);
    }
    gather_gu_kernel<<<l.max_tiles, 256, 0, ctx->stream>>>(bf.tsplit, bf.tsf, H, plan.assign_token, bf.tb, l.terms,
                                                           l.nmax, bf.b_gu, bf.sfb_gu);
    K3XB_LAUNCHED(ctx);
    prep.end();

    GuParams gp{bf.tb.desc_gu, bf.tb.counts + 1, sfa_gate, sfa_up, bf.sfb_gu, bf.act, l.tpt, H, I, l.terms,
                L.activation, L.situ_beta, L.situ_linear_beta, ctx->status_word};
    SplitArgs sa{bf.act, bf.tb, I, l.terms, l.tpt, l.nmax, bf.b_d, bf.sfb_d, l.max_tiles};
    DParams dp{bf.tb.desc_d, bf.tb.counts + 2, plan.assign_token, plan.assign_slot, sfa_down, bf.sfb_d, slot_out,
               H, I, l.terms, L.top_k, ctx->status_word, static_cast<uint32_t>(static_cast<size_t>(L.experts) * H / kBlockM),
               slot_out16, ep ? *ep : EpTarget{}};
    return l.nmax == 64 ? launch_routed<64>(ctx, map_gate, map_up, map_bgu, map_down, map_bd, gp, sa, dp)
                        : launch_routed<112>(ctx, map_gate, map_up, map_bgu, map_down, map_bd, gp, sa, dp);
}

int launch_shared_tc(k3xb_ctx* ctx, const k3xb_moe_layer& L, const float* hidden, uint32_t T, uint16_t* xb,
                     uint16_t* bd, float* out) {
    const uint32_t H = L.hidden, Is = L.shared_inter;
    if (H % 128 || Is % 128)
        return fail(ctx, K3XB_INVALID_EXTENT, "tensor-core shared expert needs hidden and shared_inter multiples of 128");
    int st;
    CUtensorMap map_gate, map_up, map_x, map_down, map_b;
    if ((st = make_map(ctx, &map_gate, L.shared_gate, static_cast<uint64_t>(H) * 2, Is, 128))) return st;
    if ((st = make_map(ctx, &map_up, L.shared_up, static_cast<uint64_t>(H) * 2, Is, 128))) return st;
    if ((st = make_map(ctx, &map_x, xb, static_cast<uint64_t>(H) * 2, 2ull * T, 2 * kSharedTok))) return st;
    if ((st = make_map(ctx, &map_down, L.shared_down, static_cast<uint64_t>(Is) * 2, H, 128))) return st;
    if ((st = make_map(ctx, &map_b, bd, static_cast<uint64_t>(Is) * 2, 2ull * T, 2 * kSharedTok))) return st;
    TcState* s = state_of(ctx);
    const size_t smem_gu = tcp::smem_bytes<kStagesGU, 2>();
    const size_t smem_d = tcp::smem_bytes<kStagesD, 1>();
    if (!s->configured_shared) {
        K3XB_CUDA(ctx, cudaFuncSetAttribute(shared_gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(smem_gu)));
        K3XB_CUDA(ctx, cudaFuncSetAttribute(shared_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(smem_d)));
        s->configured_shared = true;
    }
    const size_t n = static_cast<size_t>(T) * H;
    split_bf16_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, ctx->stream>>>(hidden, n, H, xb);
    K3XB_LAUNCHED(ctx);
    const uint32_t tiles = (T + kSharedTok - 1) / kSharedTok;
    SharedParams p{T, H, Is, tiles * (Is / kBlockM), bd, out, L.activation, L.situ_beta, L.situ_linear_beta,
                   ctx->status_word};
    shared_gateup_kernel<<<std::min<uint32_t>(ctx->sm_count, p.items), kThreads, smem_gu, ctx->stream>>>(
        map_gate, map_up, map_x, p);
    K3XB_LAUNCHED(ctx);
    p.items = tiles * (H / kBlockM);
    shared_down_kernel<<<std::min<uint32_t>(ctx->sm_count, p.items), kThreads, smem_d, ctx->stream>>>(map_down,
                                                                                                    map_b, p);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

void release_mxf4_resources(k3xb_ctx* ctx) {
    if (!ctx->mxf4_state) return;
    delete static_cast<TcState*>(ctx->mxf4_state);
    ctx->mxf4_state = nullptr;
}

}  // namespace k3xb
