// router.cu — (a) router scores, Top-k selection and expert-major bucketing.
//
// Logits follow route_official_moe (runtime/src/official_moe.cpp:255-267):
// each (token, expert) logit is one FP64 chain summed in hidden order, so
// the float result is bit-identical to the reference. A bf16 x float
// product is exact in FP64, so fma(w, x, acc) rounds exactly like the
// reference's `sum += double(w) * x`. Chains are independent per (token,
// expert); a thread carries several of them for ILP. The kernels are bound
// by the FP64 dependency chain (H sequential FMAs), not by HBM: W_r is
// 5.5 MB at the released shape and is re-read from L2 per token group.
#include "common.cuh"
#include "kernels.cuh"
#include "tc.cuh"

#include <cfloat>

namespace k3xb {

namespace {

// CTA tile: 32 experts (one per lane) x 16 tokens (4 per warp, 4 warps).
// W and x stream through a double-buffered shared-memory chunk of kChunk
// hidden columns: W transposed to [h][expert] (float, exact from bf16) so
// lanes read consecutive words, x as double [h][token] so a warp's 4 tokens
// are one broadcast 32-byte read. Padding (h >= H) is zero, and adding
// fma(0, 0, acc) = acc leaves each chain bit-identical.
constexpr int kExp = 32;
constexpr int kTokCta = 16;
constexpr int kChunk = 256;
constexpr size_t kLogitsSmem = 2 * kChunk * kExp * sizeof(float) + 2 * kChunk * kTokCta * sizeof(double);

__global__ void __launch_bounds__(128) router_logits_kernel(
    const float* __restrict__ hidden, const uint16_t* __restrict__ W, uint32_t T,
    uint32_t H, uint32_t E, float* __restrict__ logits) {
    extern __shared__ __align__(16) unsigned char router_smem[];
    float* ws = reinterpret_cast<float*>(router_smem);                        // [2][kChunk][kExp]
    double* xs = reinterpret_cast<double*>(ws + 2 * kChunk * kExp);           // [2][kChunk][kTokCta]
    const uint32_t tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
    const uint32_t e0 = blockIdx.x * kExp, t0 = blockIdx.y * kTokCta;

    // Stage registers: 8 x (8 bf16 of one expert row) and 8 x (4 floats of
    // one token row) per thread, loaded for chunk c+1 while chunk c computes.
    // Vector path when rows are 16-byte aligned; element path otherwise.
    const bool vec = (H % 8 == 0) && ((reinterpret_cast<uintptr_t>(W) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(hidden) & 15) == 0);
    const uint32_t we = e0 + tid % kExp, wseg = tid / kExp;         // W: segments wseg + 4k
    const uint32_t xt = t0 + tid % kTokCta, xseg = tid / kTokCta;   // x: segments xseg + 8k
    uint4 wr[8];
    float4 xr[8];
    auto fetch = [&](uint32_t h0) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint32_t hw = h0 + (wseg + 4 * k) * 8;
            wr[k] = make_uint4(0, 0, 0, 0);
            if (we < E && hw < H) {
                const uint16_t* src = W + static_cast<size_t>(we) * H + hw;
                if (vec) {
                    wr[k] = __ldg(reinterpret_cast<const uint4*>(src));
                } else {
                    uint16_t v[8];
                    for (int i = 0; i < 8; ++i) v[i] = hw + i < H ? src[i] : 0;
                    wr[k] = make_uint4(v[0] | (v[1] << 16), v[2] | (v[3] << 16), v[4] | (v[5] << 16),
                                       v[6] | (v[7] << 16));
                }
            }
            const uint32_t hx = h0 + (xseg + 8 * k) * 4;
            xr[k] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (xt < T && hx < H) {
                const float* src = hidden + static_cast<size_t>(xt) * H + hx;
                if (vec) {
                    xr[k] = __ldg(reinterpret_cast<const float4*>(src));
                } else {
                    xr[k].x = src[0];
                    xr[k].y = hx + 1 < H ? src[1] : 0.f;
                    xr[k].z = hx + 2 < H ? src[2] : 0.f;
                    xr[k].w = hx + 3 < H ? src[3] : 0.f;
                }
            }
        }
    };
    auto stash = [&](uint32_t buf) {
        float* wdst = ws + buf * kChunk * kExp;
        double* xdst = xs + buf * kChunk * kTokCta;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint32_t hw = (wseg + 4 * k) * 8;
            const uint32_t q[4] = {wr[k].x, wr[k].y, wr[k].z, wr[k].w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                wdst[(hw + 2 * i) * kExp + tid % kExp] = __uint_as_float(q[i] << 16);
                wdst[(hw + 2 * i + 1) * kExp + tid % kExp] = __uint_as_float(q[i] & 0xffff0000u);
            }
            const uint32_t hx = (xseg + 8 * k) * 4;
            xdst[(hx + 0) * kTokCta + tid % kTokCta] = xr[k].x;
            xdst[(hx + 1) * kTokCta + tid % kTokCta] = xr[k].y;
            xdst[(hx + 2) * kTokCta + tid % kTokCta] = xr[k].z;
            xdst[(hx + 3) * kTokCta + tid % kTokCta] = xr[k].w;
        }
    };

    double acc[4] = {0.0, 0.0, 0.0, 0.0};
    const uint32_t chunks = (H + kChunk - 1) / kChunk;
    fetch(0);
    stash(0);
    __syncthreads();
    for (uint32_t c = 0; c < chunks; ++c) {
        const uint32_t buf = c & 1u;
        if (c + 1 < chunks) fetch((c + 1) * kChunk);
        const float* wb = ws + buf * kChunk * kExp;
        const double* xb = xs + buf * kChunk * kTokCta + 4 * warp;
#pragma unroll 8
        for (uint32_t h = 0; h < kChunk; ++h) {
            const double w = static_cast<double>(wb[h * kExp + lane]);
            const double2 xa = *reinterpret_cast<const double2*>(xb + h * kTokCta);
            const double2 xc = *reinterpret_cast<const double2*>(xb + h * kTokCta + 2);
            acc[0] = fma(w, xa.x, acc[0]);
            acc[1] = fma(w, xa.y, acc[1]);
            acc[2] = fma(w, xc.x, acc[2]);
            acc[3] = fma(w, xc.y, acc[3]);
        }
        if (c + 1 < chunks) stash(buf ^ 1u);
        __syncthreads();
    }
    const uint32_t e = e0 + lane;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t t = t0 + 4 * warp + j;
        if (e < E && t < T) logits[static_cast<size_t>(t) * E + e] = static_cast<float>(acc[j]);
    }
}

// TMA variant (rows 16-byte aligned, H % 64 == 0, the CTA's TW token rows
// fit in shared memory): lane = expert, a CTA's 4 warps cover 128 experts.
// The TW tokens' hidden rows are staged once as double [h][TW]; the 128
// expert rows stream through kRtStages shared-memory stages of 64 weights,
// each one 2D TMA box (128 rows x 128 B, 128B-swizzled so a warp's 16-byte
// reads hit distinct banks). A chain step is a conversion (float -> double,
// exact), one broadcast shared load and TW independent FMAs; thread 0 also
// refills each stage once all 128 threads have released it.
constexpr int kRtStages = 6;
constexpr uint32_t kRtStageBytes = 128 * 128;
constexpr size_t kRtSmemMax = 220 * 1024;
constexpr uint32_t kRtThreads = 160;   // 4 consumer warps (one expert row per thread) + 1 producer warp

struct RtBars {
    uint64_t full[kRtStages], empty[kRtStages];
    int abort;
};

constexpr size_t rt_smem_bytes(uint32_t H, int tw) {
    return 1024 + kRtStages * kRtStageBytes + static_cast<size_t>(H) * tw * sizeof(double) + sizeof(RtBars);
}

template <int TW>
__global__ void __launch_bounds__(kRtThreads) router_tma_kernel(const __grid_constant__ CUtensorMap map_w,
                                                                const float* __restrict__ hidden, uint32_t T,
                                                                uint32_t H, uint32_t E, float* __restrict__ logits,
                                                                int* error) {
    extern __shared__ __align__(16) unsigned char router_smem[];
    uint8_t* wst = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(router_smem) + 1023) & ~uintptr_t(1023));
    double* xs = reinterpret_cast<double*>(wst + kRtStages * kRtStageBytes);   // [H][TW]
    RtBars* bars = reinterpret_cast<RtBars*>(xs + static_cast<size_t>(H) * TW);
    volatile int* abort = &bars->abort;
    const uint32_t tid = threadIdx.x;
    const uint32_t e0 = blockIdx.x * 128;
    const uint32_t nst = H / 64;
    if (tid == 0) {
        for (int s = 0; s < kRtStages; ++s) {
            tc::mbar_init(&bars->full[s], 1);
            tc::mbar_init(&bars->empty[s], 128);
        }
        bars->abort = 0;
        tc::fence_barrier_init();
    }
    __syncthreads();
    if (tid == 128) {
        // ---- producer: one TMA box per stage, refilled once all 128 consumers released it
        tc::prefetch_tensormap(&map_w);
        uint32_t issued = 0;
        for (uint32_t st = 0; st < nst; ++st) {
            const uint32_t slot = st % kRtStages;
            if (st >= kRtStages && !tc::mbar_wait(&bars->empty[slot], ((st / kRtStages) & 1u) ^ 1u, abort)) break;
            tc::mbar_arrive_expect_tx(&bars->full[slot], kRtStageBytes);
            tc::tma_load_2d(wst + slot * kRtStageBytes, &map_w, &bars->full[slot], static_cast<int>(st * 128),
                            static_cast<int>(e0));
            ++issued;
        }
        volatile int never = 0;   // copies in flight land before the CTA exits, abort or not
        for (uint32_t k = 0; k < kRtStages && k < issued; ++k) {
            const uint32_t j = issued - 1 - k;
            tc::mbar_wait(&bars->full[j % kRtStages], (j / kRtStages) & 1u, &never, 200000000ull);
        }
        if (*abort && error) atomicExch(error, K3XB_BACKEND_UNAVAILABLE);
        return;
    }
    if (tid >= 128) return;
    // ---- consumers. Stage x: 4 hidden columns of every token per thread and
    // iteration, several 16-byte loads in flight (rows 16-byte aligned).
    const uint32_t t0 = blockIdx.y * TW;
#pragma unroll 4
    for (uint32_t h4 = tid; h4 < H / 4; h4 += 128) {
        float4 v[TW];
#pragma unroll
        for (int j = 0; j < TW; ++j)
            v[j] = t0 + j < T ? __ldg(reinterpret_cast<const float4*>(hidden + static_cast<size_t>(t0 + j) * H) + h4)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < TW; ++j) {
            xs[(4 * h4 + 0) * TW + j] = v[j].x;
            xs[(4 * h4 + 1) * TW + j] = v[j].y;
            xs[(4 * h4 + 2) * TW + j] = v[j].z;
            xs[(4 * h4 + 3) * TW + j] = v[j].w;
        }
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");   // consumers only

    double acc[TW];
#pragma unroll
    for (int j = 0; j < TW; ++j) acc[j] = 0.0;
    for (uint32_t st = 0; st < nst; ++st) {
        const uint32_t slot = st % kRtStages;
        if (!tc::mbar_wait(&bars->full[slot], (st / kRtStages) & 1u, abort)) break;
        const uint8_t* row = wst + slot * kRtStageBytes + tid * 128;
        const double* xp = xs + static_cast<size_t>(st) * 64 * TW;
#pragma unroll
        for (uint32_t c = 0; c < 8; ++c) {
            const uint4 cur = *reinterpret_cast<const uint4*>(row + ((c ^ (tid & 7u)) << 4));
            const uint32_t q[4] = {cur.x, cur.y, cur.z, cur.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t f = (i & 1) ? (q[i / 2] & 0xffff0000u) : (q[i / 2] << 16);
                const double w = static_cast<double>(__uint_as_float(f));
                const double* x = xp + (c * 8 + i) * TW;
                if (TW % 2 == 0) {
#pragma unroll
                    for (int j = 0; j < TW; j += 2) {
                        const double2 xv = *reinterpret_cast<const double2*>(x + j);
                        acc[j] = fma(w, xv.x, acc[j]);
                        acc[j + 1] = fma(w, xv.y, acc[j + 1]);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < TW; ++j) acc[j] = fma(w, x[j], acc[j]);
                }
            }
        }
        tc::mbar_arrive(&bars->empty[slot]);
    }
    if (*abort) return;
    const uint32_t e = e0 + tid;
    if (e < E) {
#pragma unroll
        for (int j = 0; j < TW; ++j)
            if (t0 + j < T) logits[static_cast<size_t>(t0 + j) * E + e] = static_cast<float>(acc[j]);
    }
}

// Register-blocked chains for many tokens (rows 16-byte aligned): a CTA of
// 2 warps owns a tile of 8*RE experts x 8*RT tokens and each thread RE x RT
// chains, so one pair of shared loads feeds RE*RT independent FMAs. Lane
// layout: te = lane % 8 picks experts {16p + 2te, 16p + 2te + 1} (p < RE/2),
// so a quarter-warp's 16-byte weight reads cover 128 contiguous bytes;
// tt = lane / 8 + 4*warp picks tokens {RT*tt + j}, shared by the 8 lanes of a
// quarter-warp (broadcast). The hidden dimension streams through two
// shared-memory chunks of kBcChunk columns, both operands converted to
// double once per CTA (exact), while the next chunk's raw words travel in
// registers. Columns past H are zero: fma(0, 0, acc) = acc, as acc starts
// at +0 and a round-to-nearest sum is never -0. Measured on B200 (H 7168,
// E 384): 387 us at 576 tokens against 637 us for the TMA kernel below,
// which stays the better choice up to ~150 tokens (and leaves most SMs to
// the side-stream shared expert there).
constexpr uint32_t kBcChunk = 64;
constexpr uint32_t kBcThreads = 64;

template <int RE, int RT>
__global__ void __launch_bounds__(kBcThreads) router_blocked_kernel(const float* __restrict__ hidden,
                                                                   const uint16_t* __restrict__ W, uint32_t T,
                                                                   uint32_t H, uint32_t E,
                                                                   float* __restrict__ logits) {
    static_assert(RE % 2 == 0 && RT == 2, "expert and token pairs");
    constexpr uint32_t EC = 8 * RE, TC = 8 * RT;
    constexpr uint32_t kWItems = EC * (kBcChunk / 8) / kBcThreads;   // 16-byte weight segments per thread
    constexpr uint32_t kXItems = TC * (kBcChunk / 4) / kBcThreads;   // 16-byte hidden segments per thread
    __shared__ __align__(16) double ws[2][kBcChunk][EC];
    __shared__ __align__(16) double xs[2][kBcChunk][TC];
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint32_t te = lane & 7u, tt = (lane >> 3) + 4u * warp;
    const uint32_t e0 = blockIdx.x * EC, t0 = blockIdx.y * TC;

    uint4 wr[kWItems];
    float4 xr[kXItems];
    auto fetch = [&](uint32_t h0) {
#pragma unroll
        for (uint32_t k = 0; k < kWItems; ++k) {
            const uint32_t idx = tid + kBcThreads * k, r = idx % EC, s = idx / EC;
            const uint32_t h = h0 + 8 * s;
            wr[k] = (e0 + r < E && h < H)
                        ? __ldg(reinterpret_cast<const uint4*>(W + static_cast<size_t>(e0 + r) * H + h))
                        : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (uint32_t k = 0; k < kXItems; ++k) {
            const uint32_t idx = tid + kBcThreads * k, t = idx % TC, s = idx / TC;
            const uint32_t h = h0 + 4 * s;
            xr[k] = (t0 + t < T && h < H)
                        ? __ldg(reinterpret_cast<const float4*>(hidden + static_cast<size_t>(t0 + t) * H + h))
                        : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    auto stash = [&](uint32_t b) {
#pragma unroll
        for (uint32_t k = 0; k < kWItems; ++k) {
            const uint32_t idx = tid + kBcThreads * k, r = idx % EC, s = idx / EC;
            const uint32_t q[4] = {wr[k].x, wr[k].y, wr[k].z, wr[k].w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                ws[b][8 * s + 2 * i][r] = static_cast<double>(__uint_as_float(q[i] << 16));
                ws[b][8 * s + 2 * i + 1][r] = static_cast<double>(__uint_as_float(q[i] & 0xffff0000u));
            }
        }
#pragma unroll
        for (uint32_t k = 0; k < kXItems; ++k) {
            const uint32_t idx = tid + kBcThreads * k, t = idx % TC, s = idx / TC;
            xs[b][4 * s + 0][t] = xr[k].x;
            xs[b][4 * s + 1][t] = xr[k].y;
            xs[b][4 * s + 2][t] = xr[k].z;
            xs[b][4 * s + 3][t] = xr[k].w;
        }
    };

    double acc[RE][RT];
#pragma unroll
    for (int i = 0; i < RE; ++i)
#pragma unroll
        for (int j = 0; j < RT; ++j) acc[i][j] = 0.0;
    const uint32_t chunks = (H + kBcChunk - 1) / kBcChunk;
    fetch(0);
    stash(0);
    __syncthreads();
    for (uint32_t c = 0; c < chunks; ++c) {
        const uint32_t b = c & 1u;
        if (c + 1 < chunks) fetch((c + 1) * kBcChunk);
#pragma unroll 8
        for (uint32_t h = 0; h < kBcChunk; ++h) {
            double w[RE], x[RT];
#pragma unroll
            for (int p = 0; p < RE / 2; ++p) {
                const double2 v = *reinterpret_cast<const double2*>(&ws[b][h][16 * p + 2 * te]);
                w[2 * p] = v.x;
                w[2 * p + 1] = v.y;
            }
            const double2 v = *reinterpret_cast<const double2*>(&xs[b][h][2 * tt]);
            x[0] = v.x;
            x[1] = v.y;
#pragma unroll
            for (int i = 0; i < RE; ++i)
#pragma unroll
                for (int j = 0; j < RT; ++j) acc[i][j] = fma(w[i], x[j], acc[i][j]);
        }
        if (c + 1 < chunks) stash(b ^ 1u);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < RE; ++i) {
        const uint32_t e = e0 + 16u * (i / 2) + 2u * te + (i & 1);
#pragma unroll
        for (int j = 0; j < RT; ++j) {
            const uint32_t t = t0 + RT * tt + j;
            if (e < E && t < T) logits[static_cast<size_t>(t) * E + e] = static_cast<float>(acc[i][j]);
        }
    }
}

// route_official_moe_logits (official_moe.cpp:211-245), one CTA per token:
// all threads compute sigmoid scores (1 / (1 + expf(-l)) in float, with expf
// evaluated as the correctly rounded float(exp(double))), then warp 0 picks
// the Top-k under (adjusted desc, index asc) and forms the contributions.
constexpr int kMaxPerLane = 32;   // E <= 1024
constexpr int kTopkThreads = 128;

__global__ void __launch_bounds__(kTopkThreads) topk_kernel(
    const float* __restrict__ logits, const float* __restrict__ correction, uint32_t T,
    uint32_t E, uint32_t K, uint32_t* __restrict__ ids, float* __restrict__ contrib,
    float* __restrict__ scores_out, int32_t* __restrict__ status) {
    __shared__ float s_score[32 * kMaxPerLane], s_adj[32 * kMaxPerLane];
    __shared__ float sel_score[32];
    __shared__ uint32_t sel_id[32];
    const uint32_t token = blockIdx.x, tid = threadIdx.x, lane = tid % 32;
    if (token >= T) return;
    const float* l = logits + static_cast<size_t>(token) * E;
    int bad = 0;
    for (uint32_t e = tid; e < E; e += blockDim.x) {
        const float x = l[e];
        const float c = correction[e];
        bad |= !isfinite(x) || !isfinite(c);
        const float ex = static_cast<float>(exp(-static_cast<double>(x)));
        const float sc = __fdiv_rn(1.0f, __fadd_rn(1.0f, ex));
        s_score[e] = sc;
        s_adj[e] = __fadd_rn(sc, c);
        if (scores_out) scores_out[static_cast<size_t>(token) * E + e] = sc;
    }
    if (__syncthreads_or(bad)) {
        if (tid == 0) atomicExch(status, K3XB_INVALID_EXTENT);
        return;
    }
    if (tid >= 32) return;
    float adj[kMaxPerLane];
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
        const uint32_t e = lane + 32u * i;
        adj[i] = e < E ? s_adj[e] : -INFINITY;
    }
    uint32_t taken = 0;   // bit i: this lane's entry i is selected
    double total = 0.0;
    for (uint32_t slot = 0; slot < K; ++slot) {
        float bv = -INFINITY;
        uint32_t bi = 0xffffffffu;
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) {
            const uint32_t e = lane + 32u * i;
            if (e < E && !(taken >> i & 1u)) {
                if (bi == 0xffffffffu || adj[i] > bv) { bv = adj[i]; bi = e; }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            const bool better = (oi != 0xffffffffu) &&
                                (bi == 0xffffffffu || ov > bv || (ov == bv && oi < bi));
            if (better) { bv = ov; bi = oi; }
        }
        if ((bi % 32) == lane) taken |= 1u << (bi / 32);
        const float bs = s_score[bi];
        if (lane == 0) { sel_score[slot] = bs; sel_id[slot] = bi; }
        total += static_cast<double>(bs);   // slot order, like the reference
    }
    __syncwarp();
    if (!isfinite(total) || total <= 0.0) {
        if (lane == 0) atomicExch(status, K3XB_INVALID_EXTENT);
        return;
    }
    if (lane < K) {
        ids[static_cast<size_t>(token) * K + lane] = sel_id[lane];
        contrib[static_cast<size_t>(token) * K + lane] =
            static_cast<float>(static_cast<double>(sel_score[lane]) / total);
    }
}

// select_routing (routing_policy.cpp:31-159), one CTA per token: the first
// natural_k entries of the stable order (adjusted score desc, index asc) by
// warp selection as in topk_kernel, then lane 0 runs the policy over at most
// 32 slots in the reference's float order. logf/expf of the entropy are the
// correctly rounded values (float of the double function).
struct RoutingArgs {
    int32_t mode;
    uint32_t fixed_k, floor_k;
    float mass_target, minimum_gap;
};

__device__ __forceinline__ bool routing_allowed(uint32_t k) {
    return k == 4 || k == 6 || k == 8 || k == 12 || k == 16;
}

__device__ float routing_boundary(const float* probs, uint32_t n, uint32_t k) {
    if (k >= n) return 1.0f;
    const float gap = fmaxf(0.0f, __fsub_rn(probs[k - 1], probs[k]));
    return __fdiv_rn(gap, fmaxf(probs[0], FLT_MIN));
}

__device__ uint32_t routing_adaptive(const float* probs, uint32_t n, float support, const RoutingArgs& a,
                                     uint32_t floor_k) {
    const float eps = 1.0e-5f;
    float cumulative = 0.0f;
    for (uint32_t slot = 0; slot < n; ++slot) {
        cumulative = __fadd_rn(cumulative, probs[slot]);
        const uint32_t k = slot + 1;
        if (!routing_allowed(k) || k < floor_k) continue;
        const float confidence = routing_boundary(probs, n, k);
        if (__fadd_rn(cumulative, eps) >= a.mass_target && __fadd_rn(static_cast<float>(k), eps) >= support &&
            __fadd_rn(confidence, eps) >= a.minimum_gap)
            return k;
    }
    return n;
}

__global__ void __launch_bounds__(kTopkThreads) select_routing_kernel(
    const float* __restrict__ scores, const float* __restrict__ bias, uint32_t T, uint32_t E, uint32_t K,
    RoutingArgs args, uint32_t* __restrict__ ids, float* __restrict__ weights, uint32_t* __restrict__ selected,
    uint32_t* __restrict__ escalated, float* __restrict__ stats, int32_t* __restrict__ status) {
    __shared__ float s_score[32 * kMaxPerLane], s_adj[32 * kMaxPerLane];
    __shared__ float sel_score[32];
    __shared__ uint32_t sel_id[32];
    const uint32_t token = blockIdx.x, tid = threadIdx.x, lane = tid % 32;
    if (token >= T) return;
    const float* sc = scores + static_cast<size_t>(token) * E;
    int bad = 0;
    for (uint32_t e = tid; e < E; e += blockDim.x) {
        const float x = sc[e], b = bias[e];
        const float adj = __fadd_rn(x, b);
        bad |= !isfinite(x) || x < 0.0f || x > 1.0f || !isfinite(b) || !isfinite(adj);
        s_score[e] = x;
        s_adj[e] = adj;
    }
    if (__syncthreads_or(bad)) {
        if (tid == 0) atomicExch(status, K3XB_INVALID_STATE);
        return;
    }
    if (tid >= 32) return;
    float adj[kMaxPerLane];
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
        const uint32_t e = lane + 32u * i;
        adj[i] = e < E ? s_adj[e] : -INFINITY;
    }
    uint32_t taken = 0;
    for (uint32_t slot = 0; slot < K; ++slot) {
        float bv = -INFINITY;
        uint32_t bi = 0xffffffffu;
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) {
            const uint32_t e = lane + 32u * i;
            if (e < E && !(taken >> i & 1u)) {
                if (bi == 0xffffffffu || adj[i] > bv) { bv = adj[i]; bi = e; }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            const bool better = (oi != 0xffffffffu) && (bi == 0xffffffffu || ov > bv || (ov == bv && oi < bi));
            if (better) { bv = ov; bi = oi; }
        }
        if ((bi % 32) == lane) taken |= 1u << (bi / 32);
        if (lane == 0) { sel_score[slot] = s_score[bi]; sel_id[slot] = bi; }
    }
    __syncwarp();
    if (lane != 0) return;
    float denom = 0.0f;
    for (uint32_t slot = 0; slot < K; ++slot) denom = __fadd_rn(denom, sel_score[slot]);
    if (!isfinite(denom) || denom <= 0.0f) {
        atomicExch(status, K3XB_INVALID_STATE);
        return;
    }
    float probs[32];
    float entropy = 0.0f;
    for (uint32_t slot = 0; slot < K; ++slot) {
        probs[slot] = __fdiv_rn(sel_score[slot], denom);
        if (probs[slot] > 0.0f)
            entropy = __fsub_rn(entropy, __fmul_rn(probs[slot], static_cast<float>(log(static_cast<double>(probs[slot])))));
    }
    const float support = static_cast<float>(exp(static_cast<double>(entropy)));
    uint32_t chosen = K, unfloored = K;
    if (args.mode == K3XB_ROUTING_FIXED) {
        unfloored = args.fixed_k;
        chosen = max(args.fixed_k, args.floor_k);
    } else if (args.mode == K3XB_ROUTING_ADAPTIVE) {
        unfloored = routing_adaptive(probs, K, support, args, 0);
        chosen = routing_adaptive(probs, K, support, args, args.floor_k);
    }
    float mass = 0.0f, sel = 0.0f;
    for (uint32_t slot = 0; slot < chosen; ++slot) {
        mass = __fadd_rn(mass, probs[slot]);
        sel = __fadd_rn(sel, sel_score[slot]);
    }
    if (!isfinite(sel) || sel <= 0.0f) {
        atomicExch(status, K3XB_INVALID_STATE);
        return;
    }
    const size_t o = static_cast<size_t>(token) * K;
    for (uint32_t slot = 0; slot < K; ++slot) {
        ids[o + slot] = slot < chosen ? sel_id[slot] : 0xffffffffu;
        weights[o + slot] = slot < chosen ? __fdiv_rn(sel_score[slot], sel) : 0.0f;
    }
    selected[token] = chosen;
    if (escalated) escalated[token] = chosen > unfloored ? 1u : 0u;
    if (stats) {
        float* st = stats + static_cast<size_t>(token) * 4;
        st[0] = K == 1 ? 0.0f : __fdiv_rn(entropy, static_cast<float>(log(static_cast<double>(K))));
        st[1] = support;
        st[2] = mass;
        st[3] = routing_boundary(probs, K, chosen);
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
    const bool rows16 = H % 8 == 0 && (reinterpret_cast<uintptr_t>(W) & 15) == 0 &&
                        (reinterpret_cast<uintptr_t>(hidden) & 15) == 0;
    if (rows16) {
        // many tokens: the register-blocked kernel, 4 x 2 or 2 x 2 chains per
        // thread, once its grid gives every SM sub-partition a warp
        const uint64_t want = 4ull * ctx->sm_count;
        auto warps = [&](uint32_t ec, uint32_t tc) {
            return 2ull * ((E + ec - 1) / ec) * ((T + tc - 1) / tc);
        };
        if (warps(32, 16) >= want) {
            router_blocked_kernel<4, 2><<<dim3((E + 31) / 32, (T + 15) / 16), kBcThreads, 0, ctx->stream>>>(
                hidden, W, T, H, E, logits);
            K3XB_LAUNCHED(ctx);
            return K3XB_OK;
        }
        if (warps(16, 16) >= want) {
            router_blocked_kernel<2, 2><<<dim3((E + 15) / 16, (T + 15) / 16), kBcThreads, 0, ctx->stream>>>(
                hidden, W, T, H, E, logits);
            K3XB_LAUNCHED(ctx);
            return K3XB_OK;
        }
    }
    const bool aligned = H % 64 == 0 && (reinterpret_cast<uintptr_t>(W) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(hidden) & 15) == 0;
    // TMA kernel: the smallest TW that keeps about one warp per SM
    // sub-partition (a chain step's latency is paid once per TW FMAs)
    int tw = 0;
    for (int c : {1, 2, 4}) {
        if (rt_smem_bytes(H, c) > kRtSmemMax) break;
        tw = c;
        const uint64_t warps = static_cast<uint64_t>((E + 127) / 128) * 4 * ((T + c - 1) / c);
        if (warps <= 4ull * ctx->sm_count) break;
    }
    if (aligned && tw > 0) {
        CUtensorMap map;
        int st = make_byte_map(ctx, &map, W, static_cast<uint64_t>(H) * 2, E, 128);
        if (st) return st;
        static std::atomic<uint64_t> tma_configured{0};
        st = configure_once(ctx, tma_configured, [&]() -> int {
            K3XB_CUDA(ctx, cudaFuncSetAttribute(router_tma_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(kRtSmemMax)));
            K3XB_CUDA(ctx, cudaFuncSetAttribute(router_tma_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(kRtSmemMax)));
            K3XB_CUDA(ctx, cudaFuncSetAttribute(router_tma_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(kRtSmemMax)));
            return K3XB_OK;
        });
        if (st) return st;
        const dim3 grid((E + 127) / 128, (T + tw - 1) / tw);
        const size_t smem = rt_smem_bytes(H, tw);
        int* err = ctx->status_word;
        if (tw == 1) router_tma_kernel<1><<<grid, kRtThreads, smem, ctx->stream>>>(map, hidden, T, H, E, logits, err);
        else if (tw == 2) router_tma_kernel<2><<<grid, kRtThreads, smem, ctx->stream>>>(map, hidden, T, H, E, logits, err);
        else router_tma_kernel<4><<<grid, kRtThreads, smem, ctx->stream>>>(map, hidden, T, H, E, logits, err);
        K3XB_LAUNCHED(ctx);
        return K3XB_OK;
    }
    static std::atomic<uint64_t> configured{0};
    const int cst = configure_once(ctx, configured, [&]() -> int {
        K3XB_CUDA(ctx, cudaFuncSetAttribute(router_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(kLogitsSmem)));
        return K3XB_OK;
    });
    if (cst) return cst;
    dim3 grid((E + kExp - 1) / kExp, (T + kTokCta - 1) / kTokCta);
    router_logits_kernel<<<grid, 128, kLogitsSmem, ctx->stream>>>(hidden, W, T, H, E, logits);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_topk(k3xb_ctx* ctx, const float* logits, const float* correction, uint32_t T,
                uint32_t E, uint32_t K, uint32_t* ids, float* contrib, float* scores,
                int32_t* status) {
    if (E > 32u * kMaxPerLane || K == 0 || K > E || K > 32)
        return fail(ctx, K3XB_INVALID_EXTENT, "route: need 0 < top_k <= min(32, experts) and experts <= 1024");
    topk_kernel<<<T, kTopkThreads, 0, ctx->stream>>>(logits, correction, T, E, K, ids, contrib, scores, status);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_select_routing(k3xb_ctx* ctx, const float* scores, uint32_t T, uint32_t E, const float* bias, uint32_t K,
                          const k3xb_routing_policy& policy, uint32_t* ids, float* weights, uint32_t* selected,
                          uint32_t* escalated, float* stats) {
    const RoutingArgs args{policy.mode, policy.fixed_k, policy.quality_floor_k, policy.mass_target,
                           policy.minimum_gap};
    select_routing_kernel<<<T, kTopkThreads, 0, ctx->stream>>>(scores, bias, T, E, K, args, ids, weights, selected,
                                                               escalated, stats, ctx->status_word);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_plan(k3xb_ctx* ctx, const uint32_t* ids, const float* contrib, uint32_t T,
                uint32_t K, uint32_t E, const k3xb_plan& plan) {
    const size_t smem = plan_smem_bytes(T, E);
    if (smem > 200 * 1024)
        return fail(ctx, K3XB_INVALID_EXTENT, "expert-major plan: experts * ceil(tokens/32) too large");
    static std::atomic<uint64_t> configured{0};
    const int cst = configure_once(ctx, configured, [&]() -> int {
        K3XB_CUDA(ctx, cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        return K3XB_OK;
    });
    if (cst) return cst;
    plan_kernel<<<1, 1024, smem, ctx->stream>>>(ids, contrib, T, K, E, plan);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

}  // namespace k3xb
