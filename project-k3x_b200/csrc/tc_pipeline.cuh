// tc_pipeline.cuh — persistent, warp-specialised tcgen05 GEMM pipeline for
// weight-stationary skinny GEMMs: D[128 weight rows][N] = A[rows][K] . B[N][K]^T,
// A streamed from HBM by TMA, B small (activation rows), D in TMEM.
//
// CTA = 192 threads: warp 0 lane 0 issues TMA (A tiles, B rows, block scales),
// warp 1 lane 0 issues tcgen05.mma (and tcgen05.cp for block scales), warps
// 2-5 drain TMEM in the epilogue (warp w owns TMEM lanes 32*(w%4)..+31). A
// stage moves 128-byte rows: 256 FP4 values (kind::mxf4) or 64 bf16 values
// (kind::f16); each MMA consumes 32 bytes of every row.
//
// Work items are 16-byte descriptors {a_row, b_row, n | ntok << 16, aux}
// produced by `get_desc(item)` (with Config::a_maps > 1 the top 4 bits of
// a_row pick one of several A0 tensor maps); every role prefetches the next item's
// descriptor while it works on the current one. With ACCB = 2 the TMEM
// accumulator is double-buffered so the MMA of item i+1 overlaps the
// epilogue of item i.
//
// Safety: every mbarrier wait is bounded (2 s of %globaltimer). A timeout
// sets an abort flag that all roles poll; the producer then waits (bounded)
// for its TMA copies in flight, the MMA thread for its MMAs, TMEM is freed and
// the kernel returns with *error = K3XB_BACKEND_UNAVAILABLE.
#pragma once

#include "common.cuh"
#include "tc.cuh"

namespace k3xb {
namespace tcp {

constexpr uint32_t kBlockM = 128;       // weight rows per tile (MMA M)
constexpr uint32_t kTileBytes = kBlockM * 128;   // 16 KB A tile per stage
constexpr uint32_t kAtomBytes = 512;    // 128 rows x 4 E8M0 scale blocks
constexpr uint32_t kThreads = 192;

// BROWS = rows of the B (activation) tile per stage; a stage holds NA A
// tiles (16 KB each), BROWS x 128 B of B and the stage's block scales.
template <uint32_t S, uint32_t NA, uint32_t BROWS = 128>
struct __align__(1024) Smem {
    uint8_t a[NA][S][kTileBytes];
    uint8_t b[S][BROWS * 128];
    uint8_t sfa[NA][S][2 * kAtomBytes];
    uint8_t sfb[S][2 * kAtomBytes];
    uint64_t full[S], empty[S], tmem_full[2], tmem_empty[2], teardown;
    uint32_t tmem_base;
    int abort;
};

template <uint32_t S, uint32_t NA, uint32_t BROWS = 128>
__device__ __forceinline__ Smem<S, NA, BROWS>& smem_from(uint8_t* raw) {
    return *reinterpret_cast<Smem<S, NA, BROWS>*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
}

template <uint32_t S, uint32_t NA, uint32_t BROWS = 128>
constexpr size_t smem_bytes() { return sizeof(Smem<S, NA, BROWS>) + 1024; }

struct Config {
    uint32_t K;             // reduction length in elements
    uint32_t n_items;
    uint32_t ncols;         // TMEM columns to allocate (power of 2 >= 32)
    uint32_t col_acc0, col_acc1;   // accumulator column of A0 / A1 (buffer 0)
    uint32_t acc_stride;    // column distance between accumulator buffers
    uint32_t col_sfa0, col_sfa1, col_sfb;
    uint32_t a1_row_off = 0;          // A1 tile rows = A0 rows + a1_row_off (same tensor map allowed)
    uint32_t b_box = 16;              // B rows per TMA box (the B tensor map's box height)
    uint32_t a_rowblocks = 0xffffffffu;   // 128-row scale blocks of A (clamps the A1 scale row)
    uint32_t a_maps = 1;              // A0 tensor maps at map_a0[0 .. a_maps): item map = a_row >> 28
};

// A descriptor's A0 row, and which of the cfg.a_maps A0 tensor maps it is in.
__device__ __forceinline__ uint32_t desc_a_row(const uint4& d, const Config& c) {
    return c.a_maps > 1 ? (d.x & 0x0fffffffu) : d.x;
}
__device__ __forceinline__ uint32_t desc_a_map(const uint4& d, const Config& c) {
    return c.a_maps > 1 ? (d.x >> 28) : 0u;
}

__device__ __forceinline__ uint32_t desc_n(const uint4& d) { return d.z & 0xffffu; }
__device__ __forceinline__ uint32_t desc_ntok(const uint4& d) { return d.z >> 16; }

template <uint32_t S, uint32_t NA, bool F16, uint32_t ACCB, uint32_t BROWS, typename GetDesc, typename Epilogue>
__device__ __forceinline__ void run_pipeline(Smem<S, NA, BROWS>& sm, const CUtensorMap* map_a0, const CUtensorMap* map_a1,
                                             const CUtensorMap* map_b, const Config cfg,
                                             const uint8_t* const* sfa_src, const uint8_t* sfb_src, int* error,
                                             GetDesc get_desc, Epilogue epilogue) {
    static_assert(ACCB == 1 || ACCB == 2, "one or two accumulator buffers");
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    volatile int* abort = &sm.abort;
    constexpr uint32_t kStepElems = F16 ? 64u : 256u;
    const uint32_t K = cfg.K;
    const uint32_t ksteps = (K + kStepElems - 1) / kStepElems;
    const uint32_t atoms_per_row = K / 128;
    const uint32_t n_items = cfg.n_items;
    const uint32_t stride = gridDim.x;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            tc::mbar_init(&sm.full[s], 1);
            tc::mbar_init(&sm.empty[s], 1);
        }
        for (uint32_t b = 0; b < 2; ++b) {
            tc::mbar_init(&sm.tmem_full[b], 1);
            tc::mbar_init(&sm.tmem_empty[b], 128);
        }
        tc::mbar_init(&sm.teardown, 1);
        sm.abort = 0;
        tc::fence_barrier_init();
    }
    if (warp == 1) tc::tmem_alloc(&sm.tmem_base, cfg.ncols);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = sm.tmem_base;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer ----------------
        for (uint32_t m = 0; m < cfg.a_maps; ++m) tc::prefetch_tensormap(map_a0 + m);
        if (NA == 2) tc::prefetch_tensormap(map_a1);
        tc::prefetch_tensormap(map_b);
        uint32_t it = 0;
        uint4 d = blockIdx.x < n_items ? get_desc(blockIdx.x) : make_uint4(0, 0, 0, 0);
        for (uint32_t item = blockIdx.x; item < n_items && !*abort; item += stride) {
            const uint4 nd = item + stride < n_items ? get_desc(item + stride) : d;
            const uint32_t a_row = desc_a_row(d, cfg), b_row = d.y, n = desc_n(d);
            const CUtensorMap* ma0 = map_a0 + desc_a_map(d, cfg);
            for (uint32_t s = 0; s < ksteps; ++s, ++it) {
                const uint32_t st = it % S, ph = (it / S) & 1u;
                if (!tc::mbar_wait(&sm.empty[st], ph ^ 1u, abort)) break;
                const uint32_t atoms = F16 ? 0u : min(2u, (K - s * kStepElems) / 128u);
                const uint32_t b_loads = (n + cfg.b_box - 1) / cfg.b_box;
                const uint32_t bytes = NA * kTileBytes + b_loads * cfg.b_box * 128u + (NA + 1) * atoms * kAtomBytes;
                tc::mbar_arrive_expect_tx(&sm.full[st], bytes);
                const int x = static_cast<int>(s * 128u);
                tc::tma_load_2d(sm.a[0][st], ma0, &sm.full[st], x, static_cast<int>(a_row));
                if (NA == 2)
                    tc::tma_load_2d(sm.a[NA - 1][st], map_a1, &sm.full[st], x, static_cast<int>(a_row + cfg.a1_row_off));
                for (uint32_t r = 0; r < b_loads; ++r)
                    tc::tma_load_2d(sm.b[st] + r * cfg.b_box * 128u, map_b, &sm.full[st], x,
                                    static_cast<int>(b_row + r * cfg.b_box));
                if (!F16) {
                    for (uint32_t m = 0; m < NA; ++m) {
                        const uint32_t rb = min((a_row + (m ? cfg.a1_row_off : 0u)) / 128u, cfg.a_rowblocks - 1u);
                        const size_t a_atom = static_cast<size_t>(rb) * atoms_per_row + 2 * s;
                        tc::bulk_load(sm.sfa[m][st], sfa_src[m] + a_atom * kAtomBytes, atoms * kAtomBytes,
                                      &sm.full[st]);
                    }
                    // one scale-atom column per B tile (BROWS rows padded to the atom's 128)
                    const size_t b_atom = static_cast<size_t>(b_row / BROWS) * atoms_per_row + 2 * s;
                    tc::bulk_load(sm.sfb[st], sfb_src + b_atom * kAtomBytes, atoms * kAtomBytes, &sm.full[st]);
                }
            }
            d = nd;
        }
        volatile int never = 0;   // these waits must not be cut short by the abort flag
        for (uint32_t k = 0; k < S && k < it; ++k) {   // copies still in flight
            const uint32_t j = it - 1 - k;
            tc::mbar_wait(&sm.full[j % S], (j / S) & 1u, &never, 200000000ull);
        }
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        uint32_t it = 0, local = 0;
        bool issued = false;
        uint4 d = blockIdx.x < n_items ? get_desc(blockIdx.x) : make_uint4(0, 0, 0, 0);
        for (uint32_t item = blockIdx.x; item < n_items && !*abort; item += stride, ++local) {
            const uint4 nd = item + stride < n_items ? get_desc(item + stride) : d;
            const uint32_t n = desc_n(d);
            const uint32_t buf = ACCB == 2 ? (local & 1u) : 0u;
            const uint32_t use = ACCB == 2 ? (local >> 1) : local;   // uses of this buffer so far
            if (!tc::mbar_wait(&sm.tmem_empty[buf], (use & 1u) ^ 1u, abort)) break;
            tc::fence_after_sync();
            const uint32_t acc0 = tmem + cfg.col_acc0 + buf * cfg.acc_stride;
            const uint32_t acc1 = tmem + cfg.col_acc1 + buf * cfg.acc_stride;
            bool ok = true;
            for (uint32_t s = 0; s < ksteps; ++s, ++it) {
                const uint32_t st = it % S, ph = (it / S) & 1u;
                if (!tc::mbar_wait(&sm.full[st], ph, abort)) { ok = false; break; }
                const uint64_t bdesc = tc::desc_sw128(sm.b[st]);
                const uint64_t a0desc = tc::desc_sw128(sm.a[0][st]);
                const uint64_t a1desc = tc::desc_sw128(sm.a[NA - 1][st]);
                if (F16) {
                    const uint32_t idesc = tc::idesc_bf16(n);
                    for (uint32_t j = 0; j < 4; ++j) {
                        const uint32_t acc = (s > 0 || j > 0) ? 1u : 0u;
                        tc::mma_bf16(acc0, a0desc + 2 * j, bdesc + 2 * j, idesc, acc);
                        if (NA == 2) tc::mma_bf16(acc1, a1desc + 2 * j, bdesc + 2 * j, idesc, acc);
                    }
                } else {
                    const uint32_t atoms = min(2u, (K - s * kStepElems) / 128u);
                    for (uint32_t a = 0; a < atoms; ++a) {
                        tc::cp_32x128b_warpx4(tmem + cfg.col_sfa0 + 4 * a,
                                              tc::desc_sf_atom(sm.sfa[0][st] + a * kAtomBytes));
                        if (NA == 2)
                            tc::cp_32x128b_warpx4(tmem + cfg.col_sfa1 + 4 * a,
                                                  tc::desc_sf_atom(sm.sfa[NA - 1][st] + a * kAtomBytes));
                        tc::cp_32x128b_warpx4(tmem + cfg.col_sfb + 4 * a,
                                              tc::desc_sf_atom(sm.sfb[st] + a * kAtomBytes));
                    }
                    for (uint32_t j = 0; j < 2 * atoms; ++j) {
                        const uint32_t sfid = (j & 1u) * 2u, aoff = 4u * (j >> 1);
                        const uint32_t idesc = tc::idesc_mxf4(n, sfid, sfid);
                        const uint32_t acc = (s > 0 || j > 0) ? 1u : 0u;
                        tc::mma_mxf4(acc0, a0desc + 2 * j, bdesc + 2 * j, idesc, acc, tmem + cfg.col_sfa0 + aoff,
                                     tmem + cfg.col_sfb + aoff);
                        if (NA == 2)
                            tc::mma_mxf4(acc1, a1desc + 2 * j, bdesc + 2 * j, idesc, acc,
                                         tmem + cfg.col_sfa1 + aoff, tmem + cfg.col_sfb + aoff);
                    }
                }
                tc::commit(&sm.empty[st]);
                issued = true;
            }
            if (!ok) break;
            tc::commit(&sm.tmem_full[buf]);
            d = nd;
        }
        if (issued) {   // all issued MMAs finish before TMEM is freed
            volatile int never = 0;
            tc::commit(&sm.teardown);
            tc::mbar_wait(&sm.teardown, 0, &never, 200000000ull);
        }
    } else if (warp >= 2) {
        // ---------------- epilogue (4 warps = 128 TMEM lanes) ----------------
        uint32_t local = 0;
        uint4 d = blockIdx.x < n_items ? get_desc(blockIdx.x) : make_uint4(0, 0, 0, 0);
        for (uint32_t item = blockIdx.x; item < n_items && !*abort; item += stride, ++local) {
            const uint4 nd = item + stride < n_items ? get_desc(item + stride) : d;
            const uint32_t buf = ACCB == 2 ? (local & 1u) : 0u;
            const uint32_t use = ACCB == 2 ? (local >> 1) : local;
            if (!tc::mbar_wait(&sm.tmem_full[buf], use & 1u, abort)) break;
            tc::fence_after_sync();
            epilogue(d, tmem + buf * cfg.acc_stride, warp % 4, lane);
            tc::fence_before_sync();
            tc::mbar_arrive(&sm.tmem_empty[buf]);
            d = nd;
        }
    }
    __syncthreads();
    if (*abort && threadIdx.x == 0) atomicExch(error, K3XB_BACKEND_UNAVAILABLE);
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, cfg.ncols);
    }
}

}  // namespace tcp
}  // namespace k3xb
