// experts_mxf4.cu — (b)+(c) expert FFN on tcgen05 block-scaled tensor cores
// (kind::mxf4: E2M1 x E2M1 with UE8M0 per-32 scales, FP32 accumulation in
// TMEM).
//
// Weights are consumed in the reference's own MXFP4 layout: packed
// [rows][K/2] bytes, low nibble = even column, are TMA-loaded straight from
// HBM into 128B-swizzled shared memory (no dequantisation, 0.53 B/weight);
// only the E8M0 scales are re-laid once into the 128-row x 4-block atoms
// that tcgen05.cp moves into TMEM.
//
// The activation operand must be E2M1 too, so each activation row is split
// exactly into `terms` E2M1 rows with their own E8M0 block scales
// (x = sum_t q_t + r, |r| shrinks >= 4x per term; 6 terms reproduce bf16
// inputs exactly and fp32 SwiGLU outputs to ~2^-12 of the block maximum).
// The terms of one token occupy consecutive B rows (the MMA N dimension)
// and the epilogue sums their accumulator columns.
//
// Kernels per MoE layer:
//   worklist   — tiles of <= floor(128/terms) tokens per expert group and the
//                (tile, 128-row m-tile) work items for both GEMMs
//   split_gu   — E2M1-term split of the gathered hidden rows (B of gate/up)
//   gateup     — persistent, warp-specialised: TMA producer / single-thread
//                MMA issuer / 4 epilogue warps. gate and up share the B tile;
//                the epilogue applies SwiGLU (or SiTU) and splits the result
//                into the E2M1 B operand (+ scales) of the down projection
//   down       — same pipeline; the epilogue sums term columns, rounds to
//                bf16 (official_moe.cpp:101) and scatters rows to their
//                (token, slot) slot for the ordered combine (c)
#include "common.cuh"
#include "kernels.cuh"
#include "tc.cuh"

namespace k3xb {

namespace {

constexpr uint32_t kBlockM = 128;       // weight rows per tile (MMA M)
constexpr uint32_t kKStep = 256;        // K elements per pipeline stage (128 B of FP4)
constexpr uint32_t kNMax = 128;         // activation rows (tokens x terms) per tile
constexpr uint32_t kTileBytes = kBlockM * (kKStep / 2);   // 16 KB
constexpr uint32_t kAtomBytes = 512;    // 128 rows x 4 scale blocks
constexpr uint32_t kThreads = 192;      // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr uint32_t kStagesGU = 4;
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
    uint32_t* tile_group;
    uint32_t* tile_tok0;    // index into the plan's assignment arrays
    uint32_t* tile_ntok;
    uint32_t* items_gu;     // (tile << 12) | m-tile
    uint32_t* items_d;
};

__global__ void worklist_kernel(const uint32_t* group_count, const uint32_t* group_offset, uint32_t terms,
                                uint32_t mt_gu, uint32_t mt_d, Tables t) {
    __shared__ uint32_t tile_base[1025];
    const uint32_t ng = *group_count;
    const uint32_t tpt = kNMax / terms;
    if (threadIdx.x == 0) {
        uint32_t run = 0;
        for (uint32_t g = 0; g < ng; ++g) {
            tile_base[g] = run;
            const uint32_t ntok = group_offset[g + 1] - group_offset[g];
            run += (ntok + tpt - 1) / tpt;
        }
        tile_base[ng] = run;
        t.counts[0] = run;
        t.counts[1] = run * mt_gu;
        t.counts[2] = run * mt_d;
    }
    __syncthreads();
    for (uint32_t g = threadIdx.x; g < ng; g += blockDim.x) {
        const uint32_t ntok = group_offset[g + 1] - group_offset[g];
        const uint32_t tb = tile_base[g], nt = tile_base[g + 1] - tb;
        for (uint32_t j = 0; j < nt; ++j) {
            t.tile_group[tb + j] = g;
            t.tile_tok0[tb + j] = group_offset[g] + j * tpt;
            t.tile_ntok[tb + j] = min(tpt, ntok - j * tpt);
        }
        // items: group-major, then m-tile, then n-tile (n-tiles of one weight
        // tile are adjacent so the second read hits L2)
        for (uint32_t mt = 0; mt < mt_gu; ++mt)
            for (uint32_t j = 0; j < nt; ++j) t.items_gu[tb * mt_gu + mt * nt + j] = ((tb + j) << 12) | mt;
        for (uint32_t mt = 0; mt < mt_d; ++mt)
            for (uint32_t j = 0; j < nt; ++j) t.items_d[tb * mt_d + mt * nt + j] = ((tb + j) << 12) | mt;
    }
}

// ---------------------------------------------------------------------------
// E2M1-term split of one 32-block held by one thread (gate/up B operand).
// Bit-identical to oracle/k3x_oracle.c:k3xo_e2m1_terms.
__device__ __forceinline__ void split_block(float (&r)[32], uint32_t terms, uint8_t* row0, size_t row_stride,
                                            uint8_t* sf, uint32_t sf_row_stride_unused, uint32_t tile,
                                            uint32_t j, uint32_t kb, uint32_t kb_count, uint8_t* sfb) {
    (void)sf; (void)sf_row_stride_unused;
    for (uint32_t t = 0; t < terms; ++t) {
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(r[i]));
        const int s = amax > 0.0f ? e2m1_block_exponent(amax) : 0;
        const float inv = exp2i(-s), scl = exp2i(s);
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint32_t acc = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float v = r[8 * q + i];
                const uint32_t code = e2m1_code(fabsf(v) * inv);
                const bool neg = signbit(v) && code;
                acc |= (code | (neg ? 8u : 0u)) << (4 * i);
                const float qv = e2m1_magnitude(code) * scl;
                r[8 * q + i] = neg ? __fadd_rn(v, qv) : __fsub_rn(v, qv);
            }
            w[q] = acc;
        }
        const uint32_t n = j * terms + t;   // row inside the tile
        *reinterpret_cast<uint4*>(row0 + static_cast<size_t>(n) * row_stride + kb * 16) =
            make_uint4(w[0], w[1], w[2], w[3]);
        sfb[(static_cast<size_t>(tile) * (kb_count / 4) + kb / 4) * kAtomBytes + (n % 32) * 16 + (n / 32) * 4 +
            kb % 4] = static_cast<uint8_t>(s + 127);
    }
}

__global__ void __launch_bounds__(256) split_gu_kernel(const float* __restrict__ hidden, uint32_t H,
                                                       const uint32_t* __restrict__ assign_token,
                                                       Tables tb, uint32_t terms, uint8_t* __restrict__ b,
                                                       uint8_t* __restrict__ sfb) {
    const uint32_t tile = blockIdx.x;
    if (tile >= tb.counts[0]) return;
    const uint32_t ntok = tb.tile_ntok[tile], tok0 = tb.tile_tok0[tile];
    const uint32_t n = round16(ntok * terms);
    const uint32_t kbc = H / 32;
    const size_t row_stride = H / 2;
    uint8_t* base = b + static_cast<size_t>(tile) * kNMax * row_stride;
    for (uint32_t i = threadIdx.x; i < ntok * kbc; i += blockDim.x) {
        const uint32_t j = i / kbc, kb = i % kbc;
        const float* x = hidden + static_cast<size_t>(assign_token[tok0 + j]) * H + kb * 32;
        float r[32];
#pragma unroll
        for (int q = 0; q < 32; q += 4) {
            const float4 v = *reinterpret_cast<const float4*>(x + q);
            r[q] = v.x; r[q + 1] = v.y; r[q + 2] = v.z; r[q + 3] = v.w;
        }
        split_block(r, terms, base, row_stride, nullptr, 0, tile, j, kb, kbc, sfb);
    }
    // zero padding rows up to the MMA N (16-multiple)
    const uint32_t pad0 = ntok * terms;
    for (uint32_t i = threadIdx.x; i < (n - pad0) * kbc; i += blockDim.x) {
        const uint32_t rr = pad0 + i / kbc, kb = i % kbc;
        *reinterpret_cast<uint4*>(base + static_cast<size_t>(rr) * row_stride + kb * 16) = make_uint4(0, 0, 0, 0);
        sfb[(static_cast<size_t>(tile) * (kbc / 4) + kb / 4) * kAtomBytes + (rr % 32) * 16 + (rr / 32) * 4 +
            kb % 4] = 127;
    }
}

// ---------------------------------------------------------------------------
__device__ __forceinline__ float activate(float g, float u, int act, float beta, float lbeta) {
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
    if (act == K3XB_ACT_SITU) {
        const float bg = __fmul_rn(__fmul_rn(beta, tanhf(__fdiv_rn(g, beta))), sig);
        const float bu = lbeta > 0.0f ? __fmul_rn(lbeta, tanhf(__fdiv_rn(u, lbeta))) : u;
        return __fmul_rn(bg, bu);
    }
    return __fmul_rn(__fmul_rn(g, sig), u);
}

struct GuParams {
    Tables tb;
    const uint32_t* group_expert;
    const uint8_t* sfa_gate;
    const uint8_t* sfa_up;
    const uint8_t* sfb;       // split_gu scales
    uint8_t* b_down;          // epilogue outputs: down-projection B operand
    uint8_t* sfb_down;
    uint32_t H, I, terms;
    int act;
    float beta, lbeta;
    int* error;
};

struct DParams {
    Tables tb;
    const uint32_t* group_expert;
    const uint32_t* assign_token;
    const uint32_t* assign_slot;
    const uint8_t* sfa;
    const uint8_t* sfb;
    float* slot_out;
    uint32_t H, I, terms, top_k;
    int* error;
};

template <uint32_t S, uint32_t NA>
struct __align__(1024) Smem {
    uint8_t a[NA][S][kTileBytes];
    uint8_t b[S][kTileBytes];
    uint8_t sfa[NA][S][2 * kAtomBytes];
    uint8_t sfb[S][2 * kAtomBytes];
    uint64_t full[S], empty[S], tmem_full, tmem_empty, teardown;
    uint32_t tmem_base;
    int abort;
};

// TMEM column map
constexpr uint32_t kColAccGate = 0, kColAccUp = 128, kColSfaGate = 256, kColSfaUp = 264, kColSfbGU = 272;
constexpr uint32_t kColsGU = 512;
constexpr uint32_t kColAccD = 0, kColSfaD = 128, kColSfbD = 136;
constexpr uint32_t kColsD = 256;

// Shared pipeline body. NA = number of A matrices sharing the B tile
// (2 for gate/up, 1 for down). Epilogue is a functor called by warps 2-5.
template <uint32_t S, uint32_t NA, typename Decode, typename Epilogue>
__device__ __forceinline__ void run_pipeline(Smem<S, NA>& sm, const CUtensorMap* map_a0, const CUtensorMap* map_a1,
                                             const CUtensorMap* map_b, uint32_t K, uint32_t n_items,
                                             const uint8_t* const* sfa_src, const uint8_t* sfb_src,
                                             uint32_t col_acc0, uint32_t col_acc1, uint32_t col_sfa0,
                                             uint32_t col_sfa1, uint32_t col_sfb, uint32_t ncols, int* error,
                                             Decode decode, Epilogue epilogue) {
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    volatile int* abort = &sm.abort;
    const uint32_t ksteps = (K + kKStep - 1) / kKStep;
    const uint32_t atoms_per_row = K / 128;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            tc::mbar_init(&sm.full[s], 1);
            tc::mbar_init(&sm.empty[s], 1);
        }
        tc::mbar_init(&sm.tmem_full, 1);
        tc::mbar_init(&sm.tmem_empty, 128);
        tc::mbar_init(&sm.teardown, 1);
        sm.abort = 0;
        tc::fence_barrier_init();
    }
    if (warp == 1) tc::tmem_alloc(&sm.tmem_base, ncols);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = sm.tmem_base;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer ----------------
        tc::prefetch_tensormap(map_a0);
        if (NA == 2) tc::prefetch_tensormap(map_a1);
        tc::prefetch_tensormap(map_b);
        uint32_t it = 0;
        for (uint32_t item = blockIdx.x; item < n_items && !*abort; item += gridDim.x) {
            uint32_t a_row, b_row, n, sfb_tile;
            decode(item, a_row, b_row, n, sfb_tile);
            for (uint32_t s = 0; s < ksteps; ++s, ++it) {
                const uint32_t st = it % S, ph = (it / S) & 1u;
                if (!tc::mbar_wait(&sm.empty[st], ph ^ 1u, abort)) break;
                const uint32_t atoms = min(2u, (K - s * kKStep) / 128u);
                const uint32_t bytes = NA * kTileBytes + n * (kKStep / 2) + (NA + 1) * atoms * kAtomBytes;
                tc::mbar_arrive_expect_tx(&sm.full[st], bytes);
                const int x = static_cast<int>(s * (kKStep / 2));
                tc::tma_load_2d(sm.a[0][st], map_a0, &sm.full[st], x, static_cast<int>(a_row));
                if (NA == 2) tc::tma_load_2d(sm.a[NA - 1][st], map_a1, &sm.full[st], x, static_cast<int>(a_row));
                for (uint32_t r = 0; r < n; r += 16)
                    tc::tma_load_2d(sm.b[st] + r * (kKStep / 2), map_b, &sm.full[st], x,
                                    static_cast<int>(b_row + r));
                const size_t a_atom = static_cast<size_t>(a_row / 128) * atoms_per_row + 2 * s;
                for (uint32_t m = 0; m < NA; ++m)
                    tc::bulk_load(sm.sfa[m][st], sfa_src[m] + a_atom * kAtomBytes, atoms * kAtomBytes, &sm.full[st]);
                const size_t b_atom = static_cast<size_t>(sfb_tile) * atoms_per_row + 2 * s;
                tc::bulk_load(sm.sfb[st], sfb_src + b_atom * kAtomBytes, atoms * kAtomBytes, &sm.full[st]);
            }
        }
        // teardown: wait for copies still in flight (bounded)
        for (uint32_t k = 0; k < S && k < it; ++k) {
            const uint32_t j = it - 1 - k;
            tc::mbar_wait(&sm.full[j % S], (j / S) & 1u, abort, 200000000ull);
        }
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        uint32_t it = 0, acc_ph = 0;
        bool issued = false;
        for (uint32_t item = blockIdx.x; item < n_items && !*abort; item += gridDim.x) {
            uint32_t a_row, b_row, n, sfb_tile;
            decode(item, a_row, b_row, n, sfb_tile);
            if (!tc::mbar_wait(&sm.tmem_empty, acc_ph ^ 1u, abort)) break;
            tc::fence_after_sync();
            bool ok = true;
            for (uint32_t s = 0; s < ksteps; ++s, ++it) {
                const uint32_t st = it % S, ph = (it / S) & 1u;
                if (!tc::mbar_wait(&sm.full[st], ph, abort)) { ok = false; break; }
                const uint32_t atoms = min(2u, (K - s * kKStep) / 128u);
                for (uint32_t a = 0; a < atoms; ++a) {
                    tc::cp_32x128b_warpx4(tmem + col_sfa0 + 4 * a, tc::desc_sf_atom(sm.sfa[0][st] + a * kAtomBytes));
                    if (NA == 2)
                        tc::cp_32x128b_warpx4(tmem + col_sfa1 + 4 * a,
                                              tc::desc_sf_atom(sm.sfa[NA - 1][st] + a * kAtomBytes));
                    tc::cp_32x128b_warpx4(tmem + col_sfb + 4 * a, tc::desc_sf_atom(sm.sfb[st] + a * kAtomBytes));
                }
                const uint64_t bdesc = tc::desc_sw128(sm.b[st]);
                const uint64_t a0desc = tc::desc_sw128(sm.a[0][st]);
                const uint64_t a1desc = tc::desc_sw128(sm.a[NA - 1][st]);
                for (uint32_t j = 0; j < 2 * atoms; ++j) {
                    const uint32_t sfid = (j & 1u) * 2u, aoff = 4u * (j >> 1);
                    const uint32_t idesc = tc::idesc_mxf4(n, sfid, sfid);
                    const uint32_t acc = (s > 0 || j > 0) ? 1u : 0u;
                    tc::mma_mxf4(tmem + col_acc0, a0desc + 2 * j, bdesc + 2 * j, idesc, acc, tmem + col_sfa0 + aoff,
                                 tmem + col_sfb + aoff);
                    if (NA == 2)
                        tc::mma_mxf4(tmem + col_acc1, a1desc + 2 * j, bdesc + 2 * j, idesc, acc,
                                     tmem + col_sfa1 + aoff, tmem + col_sfb + aoff);
                }
                tc::commit(&sm.empty[st]);
                issued = true;
            }
            if (!ok) break;
            tc::commit(&sm.tmem_full);
            acc_ph ^= 1u;
        }
        // teardown: all issued MMAs must finish before TMEM is freed
        if (issued) {
            tc::commit(&sm.teardown);
            tc::mbar_wait(&sm.teardown, 0, abort, 200000000ull);
        }
    } else if (warp >= 2) {
        // ---------------- epilogue (4 warps = 128 TMEM lanes) ----------------
        uint32_t acc_ph = 0;
        for (uint32_t item = blockIdx.x; item < n_items && !*abort; item += gridDim.x) {
            if (!tc::mbar_wait(&sm.tmem_full, acc_ph, abort)) break;
            tc::fence_after_sync();
            epilogue(item, tmem, warp % 4, lane);
            tc::fence_before_sync();
            tc::mbar_arrive(&sm.tmem_empty);
            acc_ph ^= 1u;
        }
    }
    __syncthreads();
    if (*abort && threadIdx.x == 0) atomicExch(error, K3XB_BACKEND_UNAVAILABLE);
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, ncols);
    }
}

__global__ void __launch_bounds__(kThreads, 1) gateup_kernel(const __grid_constant__ CUtensorMap map_gate,
                                                              const __grid_constant__ CUtensorMap map_up,
                                                              const __grid_constant__ CUtensorMap map_b,
                                                              const GuParams p) {
    extern __shared__ uint8_t smem_raw[];
    auto& sm = *reinterpret_cast<Smem<kStagesGU, 2>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const Tables& tb = p.tb;
    const uint32_t n_items = tb.counts[1];
    const uint32_t terms = p.terms;
    auto decode = [&](uint32_t item, uint32_t& a_row, uint32_t& b_row, uint32_t& n, uint32_t& sfb_tile) {
        const uint32_t code = tb.items_gu[item], tile = code >> 12, mt = code & 0xfffu;
        a_row = p.group_expert[tb.tile_group[tile]] * p.I + mt * kBlockM;
        b_row = tile * kNMax;
        n = round16(tb.tile_ntok[tile] * terms);
        sfb_tile = tile;
    };
    auto epilogue = [&](uint32_t item, uint32_t tmem, uint32_t q, uint32_t lane) {
        const uint32_t code = tb.items_gu[item], tile = code >> 12, mt = code & 0xfffu;
        const uint32_t ntok = tb.tile_ntok[tile];
        const uint32_t used = ntok * terms, n = round16(used);
        const uint32_t lane_base = (32u * q) << 16;
        const size_t row_stride = p.I / 2;
        uint8_t* brow = p.b_down + static_cast<size_t>(tile) * kNMax * row_stride + mt * 64 + q * 16;
        uint8_t* sfbase = p.sfb_down + (static_cast<size_t>(tile) * (p.I / 128) + mt) * kAtomBytes + q;
        float gs = 0.0f, us = 0.0f;
        uint32_t tcount = 0, j = 0;
        for (uint32_t c0 = 0; c0 < used; c0 += 16) {
            float vg[16], vu[16];
            tc::tmem_ld16(tmem + lane_base + kColAccGate + c0, vg);
            tc::tmem_ld16(tmem + lane_base + kColAccUp + c0, vu);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if (c0 + i >= used) break;
                gs = __fadd_rn(gs, vg[i]);
                us = __fadd_rn(us, vu[i]);
                if (++tcount < terms) continue;
                // token j finished: a = act(g, u), split over this warp's
                // 32 rows (one MX block of the down projection's K)
                float r = activate(gs, us, p.act, p.beta, p.lbeta);
                for (uint32_t t = 0; t < terms; ++t) {
                    const float amax = warp_max(fabsf(r));
                    const int s = amax > 0.0f ? e2m1_block_exponent(amax) : 0;
                    const uint32_t cd = e2m1_code(fabsf(r) * exp2i(-s));
                    const bool neg = signbit(r) && cd;
                    const float qv = e2m1_magnitude(cd) * exp2i(s);
                    r = neg ? __fadd_rn(r, qv) : __fsub_rn(r, qv);
                    uint32_t word = (cd | (neg ? 8u : 0u)) << (4 * (lane % 8));
                    word |= __shfl_xor_sync(0xffffffffu, word, 1);
                    word |= __shfl_xor_sync(0xffffffffu, word, 2);
                    word |= __shfl_xor_sync(0xffffffffu, word, 4);
                    const uint32_t row = j * terms + t;
                    if (lane % 8 == 0)
                        *reinterpret_cast<uint32_t*>(brow + static_cast<size_t>(row) * row_stride + (lane / 8) * 4) = word;
                    if (lane == 0) sfbase[(row % 32) * 16 + (row / 32) * 4] = static_cast<uint8_t>(s + 127);
                }
                gs = us = 0.0f;
                tcount = 0;
                ++j;
            }
        }
        for (uint32_t row = used; row < n; ++row) {   // zero padding rows
            if (lane % 8 == 0) *reinterpret_cast<uint32_t*>(brow + static_cast<size_t>(row) * row_stride + (lane / 8) * 4) = 0u;
            if (lane == 0) sfbase[(row % 32) * 16 + (row / 32) * 4] = 127;
        }
    };
    const uint8_t* sfa[2] = {p.sfa_gate, p.sfa_up};
    run_pipeline<kStagesGU, 2>(sm, &map_gate, &map_up, &map_b, p.H, n_items, sfa, p.sfb, kColAccGate, kColAccUp,
                               kColSfaGate, kColSfaUp, kColSfbGU, kColsGU, p.error, decode, epilogue);
}

__global__ void __launch_bounds__(kThreads, 1) down_kernel(const __grid_constant__ CUtensorMap map_down,
                                                            const __grid_constant__ CUtensorMap map_b,
                                                            const DParams p) {
    extern __shared__ uint8_t smem_raw[];
    auto& sm = *reinterpret_cast<Smem<kStagesD, 1>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const Tables& tb = p.tb;
    const uint32_t n_items = tb.counts[2];
    const uint32_t terms = p.terms;
    auto decode = [&](uint32_t item, uint32_t& a_row, uint32_t& b_row, uint32_t& n, uint32_t& sfb_tile) {
        const uint32_t code = tb.items_d[item], tile = code >> 12, mt = code & 0xfffu;
        a_row = p.group_expert[tb.tile_group[tile]] * p.H + mt * kBlockM;
        b_row = tile * kNMax;
        n = round16(tb.tile_ntok[tile] * terms);
        sfb_tile = tile;
    };
    auto epilogue = [&](uint32_t item, uint32_t tmem, uint32_t q, uint32_t lane) {
        const uint32_t code = tb.items_d[item], tile = code >> 12, mt = code & 0xfffu;
        const uint32_t ntok = tb.tile_ntok[tile], tok0 = tb.tile_tok0[tile];
        const uint32_t used = ntok * terms;
        const uint32_t lane_base = (32u * q) << 16;
        const uint32_t h = mt * kBlockM + 32u * q + lane;
        float ys = 0.0f;
        uint32_t tcount = 0, j = 0;
        for (uint32_t c0 = 0; c0 < used; c0 += 16) {
            float v[16];
            tc::tmem_ld16(tmem + lane_base + kColAccD + c0, v);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if (c0 + i >= used) break;
                ys = __fadd_rn(ys, v[i]);
                if (++tcount < terms) continue;
                const uint32_t a = tok0 + j;
                const size_t dst = static_cast<size_t>(p.assign_token[a]) * p.top_k + p.assign_slot[a];
                p.slot_out[dst * p.H + h] = round_bf16(ys);
                ys = 0.0f;
                tcount = 0;
                ++j;
            }
        }
    };
    const uint8_t* sfa[1] = {p.sfa};
    run_pipeline<kStagesD, 1>(sm, &map_down, &map_down, &map_b, p.I, n_items, sfa, p.sfb, kColAccD, kColAccD,
                              kColSfaD, kColSfaD, kColSfbD, kColsD, p.error, decode, epilogue);
}

// ---------------------------------------------------------------------------
// host side

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct Mxf4State {
    EncodeFn encode = nullptr;
    bool configured = false;
};

Mxf4State* state_of(k3xb_ctx* ctx) {
    if (!ctx->mxf4_state) ctx->mxf4_state = new Mxf4State();
    return static_cast<Mxf4State*>(ctx->mxf4_state);
}

int get_encode(k3xb_ctx* ctx, EncodeFn* out) {
    Mxf4State* s = state_of(ctx);
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
int make_map(k3xb_ctx* ctx, CUtensorMap* map, const void* base, uint64_t row_bytes, uint64_t rows,
             uint32_t box_rows) {
    EncodeFn encode;
    int st = get_encode(ctx, &encode);
    if (st) return st;
    if (reinterpret_cast<uintptr_t>(base) % 16 || row_bytes % 16)
        return fail(ctx, K3XB_INVALID_EXTENT, "MXF4 operands need 16-byte aligned rows");
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

struct Layout {
    uint32_t terms, tpt, max_tiles, mt_gu, mt_d;
    size_t b_gu, sfb_gu, b_d, sfb_d;
    size_t sf_gate, sf_up, sf_down;   // per-call re-laid scales (0 when prepared)
};

Layout layout_of(const k3xb_moe_layer& L, uint32_t T) {
    Layout l{};
    l.terms = L.act_terms > 0 ? static_cast<uint32_t>(L.act_terms) : 6u;
    l.tpt = kNMax / l.terms;
    const uint32_t assigns = T * L.top_k;
    l.max_tiles = std::min(L.experts, assigns) + (assigns + l.tpt - 1) / l.tpt;
    l.mt_gu = L.inter / kBlockM;
    l.mt_d = L.hidden / kBlockM;
    l.b_gu = static_cast<size_t>(l.max_tiles) * kNMax * (L.hidden / 2);
    l.sfb_gu = static_cast<size_t>(l.max_tiles) * (L.hidden / 128) * kAtomBytes;
    l.b_d = static_cast<size_t>(l.max_tiles) * kNMax * (L.inter / 2);
    l.sfb_d = static_cast<size_t>(l.max_tiles) * (L.inter / 128) * kAtomBytes;
    const size_t sf_gu = static_cast<size_t>(L.experts) * L.inter * (L.hidden / 32);
    l.sf_gate = L.gate_scales_tc ? 0 : sf_gu;
    l.sf_up = L.up_scales_tc ? 0 : sf_gu;
    l.sf_down = L.down_scales_tc ? 0 : sf_gu;
    return l;
}

template <typename A>
void carve(A& a, const Layout& l, Tables* t, uint8_t** b_gu, uint8_t** sfb_gu, uint8_t** b_d, uint8_t** sfb_d,
           uint8_t** sf = nullptr) {
    Tables tmp;
    Tables& r = t ? *t : tmp;
    r.counts = a.template take<uint32_t>(4);
    r.tile_group = a.template take<uint32_t>(l.max_tiles);
    r.tile_tok0 = a.template take<uint32_t>(l.max_tiles);
    r.tile_ntok = a.template take<uint32_t>(l.max_tiles);
    r.items_gu = a.template take<uint32_t>(static_cast<size_t>(l.max_tiles) * l.mt_gu);
    r.items_d = a.template take<uint32_t>(static_cast<size_t>(l.max_tiles) * l.mt_d);
    uint8_t* p0 = a.template take<uint8_t>(l.b_gu, 1024);
    uint8_t* p1 = a.template take<uint8_t>(l.sfb_gu, 1024);
    uint8_t* p2 = a.template take<uint8_t>(l.b_d, 1024);
    uint8_t* p3 = a.template take<uint8_t>(l.sfb_d, 1024);
    uint8_t* q0 = a.template take<uint8_t>(l.sf_gate, 1024);
    uint8_t* q1 = a.template take<uint8_t>(l.sf_up, 1024);
    uint8_t* q2 = a.template take<uint8_t>(l.sf_down, 1024);
    if (b_gu) { *b_gu = p0; *sfb_gu = p1; *b_d = p2; *sfb_d = p3; }
    if (sf) { sf[0] = q0; sf[1] = q1; sf[2] = q2; }
}

int relayout(k3xb_ctx* ctx, const uint8_t* scales, size_t rows, uint32_t K, uint8_t* out) {
    const size_t n = rows * (K / 32);
    sf_relayout_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, ctx->stream>>>(scales, rows, K, out);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

}  // namespace

int prepare_mxfp4_scales(k3xb_ctx* ctx, const uint8_t* scales, size_t rows, size_t cols, uint8_t* out) {
    if (!scales || !out || !rows || rows % 128 || !cols || cols % 128)
        return fail(ctx, K3XB_INVALID_MXFP4, "prepare scales: rows and cols must be multiples of 128");
    return relayout(ctx, scales, rows, static_cast<uint32_t>(cols), out);
}

size_t mxf4_scratch_bytes(const k3xb_moe_layer& L, uint32_t T) {
    if (L.engine != K3XB_ENGINE_MXF4) return 0;
    Sizer s;
    carve(s, layout_of(L, T), nullptr, nullptr, nullptr, nullptr, nullptr);
    return s.used + 1024;
}

void set_mxf4_scratch(k3xb_ctx* ctx, void* region) { ctx->mxf4_scratch = region; }

int launch_mxf4_experts(k3xb_ctx* ctx, const k3xb_moe_layer& L, const float* hidden, uint32_t T,
                        const k3xb_plan& plan, float* slot_out) {
    const uint32_t H = L.hidden, I = L.inter;
    if (H % 128 || I % 128)
        return fail(ctx, K3XB_INVALID_EXTENT, "MXF4 engine needs hidden and inter multiples of 128");
    if (L.act_terms < 0 || L.act_terms > 16)
        return fail(ctx, K3XB_INVALID_EXTENT, "act_terms must be in [1, 16] (0 = default 6)");
    if (L.experts > 1024) return fail(ctx, K3XB_INVALID_EXTENT, "MXF4 engine supports <= 1024 experts");
    const Layout l = layout_of(L, T);
    if (l.max_tiles >= (1u << 20) || l.mt_d >= 4096)
        return fail(ctx, K3XB_INVALID_EXTENT, "MXF4 work list too large");
    int st;
    Carver c(reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(ctx->mxf4_scratch) + 1023) & ~uintptr_t(1023)));
    Tables tb;
    uint8_t *b_gu, *sfb_gu, *b_d, *sfb_d, *sf[3];
    carve(c, l, &tb, &b_gu, &sfb_gu, &b_d, &sfb_d, sf);
    const uint8_t* sfa_gate = L.gate_scales_tc;
    const uint8_t* sfa_up = L.up_scales_tc;
    const uint8_t* sfa_down = L.down_scales_tc;
    const size_t rows_gu = static_cast<size_t>(L.experts) * I, rows_d = static_cast<size_t>(L.experts) * H;
    if (!sfa_gate) { if ((st = relayout(ctx, L.gate_scales, rows_gu, H, sf[0]))) return st; sfa_gate = sf[0]; }
    if (!sfa_up) { if ((st = relayout(ctx, L.up_scales, rows_gu, H, sf[1]))) return st; sfa_up = sf[1]; }
    if (!sfa_down) { if ((st = relayout(ctx, L.down_scales, rows_d, I, sf[2]))) return st; sfa_down = sf[2]; }

    CUtensorMap map_gate, map_up, map_down, map_bgu, map_bd;
    if ((st = make_map(ctx, &map_gate, L.gate_packed, H / 2, static_cast<uint64_t>(L.experts) * I, 128))) return st;
    if ((st = make_map(ctx, &map_up, L.up_packed, H / 2, static_cast<uint64_t>(L.experts) * I, 128))) return st;
    if ((st = make_map(ctx, &map_down, L.down_packed, I / 2, static_cast<uint64_t>(L.experts) * H, 128))) return st;
    if ((st = make_map(ctx, &map_bgu, b_gu, H / 2, static_cast<uint64_t>(l.max_tiles) * kNMax, 16))) return st;
    if ((st = make_map(ctx, &map_bd, b_d, I / 2, static_cast<uint64_t>(l.max_tiles) * kNMax, 16))) return st;

    Mxf4State* s = state_of(ctx);
    const size_t smem_gu = sizeof(Smem<kStagesGU, 2>) + 1024;
    const size_t smem_d = sizeof(Smem<kStagesD, 1>) + 1024;
    if (!s->configured) {
        K3XB_CUDA(ctx, cudaFuncSetAttribute(gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(smem_gu)));
        K3XB_CUDA(ctx, cudaFuncSetAttribute(down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(smem_d)));
        s->configured = true;
    }

    worklist_kernel<<<1, 256, 0, ctx->stream>>>(plan.group_count, plan.group_offset, l.terms, l.mt_gu, l.mt_d, tb);
    K3XB_LAUNCHED(ctx);
    split_gu_kernel<<<l.max_tiles, 256, 0, ctx->stream>>>(hidden, H, plan.assign_token, tb, l.terms, b_gu, sfb_gu);
    K3XB_LAUNCHED(ctx);

    GuParams gp{tb, plan.group_expert, sfa_gate, sfa_up, sfb_gu, b_d, sfb_d, H, I, l.terms, L.activation,
                L.situ_beta, L.situ_linear_beta, ctx->status_word};
    gateup_kernel<<<ctx->sm_count, kThreads, smem_gu, ctx->stream>>>(map_gate, map_up, map_bgu, gp);
    K3XB_LAUNCHED(ctx);
    DParams dp{tb, plan.group_expert, plan.assign_token, plan.assign_slot, sfa_down, sfb_d, slot_out,
               H, I, l.terms, L.top_k, ctx->status_word};
    down_kernel<<<ctx->sm_count, kThreads, smem_d, ctx->stream>>>(map_down, map_bd, dp);
    K3XB_LAUNCHED(ctx);
    ctx->stats.moe_layer_experts += 0;
    return K3XB_OK;
}

void release_mxf4_resources(k3xb_ctx* ctx) {
    if (!ctx->mxf4_state) return;
    delete static_cast<Mxf4State*>(ctx->mxf4_state);
    ctx->mxf4_state = nullptr;
}

}  // namespace k3xb
