// dense.cu — f32 dense matrix-vector products with the reference CPU
// backend's arithmetic (dense_matvec, runtime/src/backend_cpu.cpp:23-47):
// y[r] = float(sum over c in column order of double(W[r][c]) * x[c]).
//
// A float x float product is exact in FP64 (48 significant bits), so
// fma(w, x, acc) rounds exactly like the reference's `sum += double(w) * x`
// and each output is one FP64 chain in column order: bit-identical to the
// reference. A thread carries one (row, token) chain; a CTA of 128 threads
// covers 128 rows of one token and streams W through shared memory in
// chunks of kChunk columns (coalesced loads, the next chunk held in
// registers while the current one is summed). The bound is the larger of
// the weight bytes over HBM and the cols-long FP64 dependency chain.
#include "common.cuh"
#include "kernels.cuh"

namespace k3xb {

namespace {

constexpr int kRows = 128;                 // rows (threads) per CTA
constexpr int kChunk = 64;                 // columns per shared-memory chunk
constexpr int kPitch = kChunk + 1;         // padded row pitch: lanes read distinct banks
constexpr int kPerThread = kRows * kChunk / kRows / 4;   // float4 loads per thread per chunk (16)

__global__ void __launch_bounds__(kRows) dense_matvec_kernel(const float* __restrict__ W, uint32_t rows,
                                                             uint32_t cols, const float* __restrict__ x,
                                                             float* __restrict__ y) {
    __shared__ float ws[kRows * kPitch];
    __shared__ double xs[kChunk];
    const uint32_t tid = threadIdx.x, r0 = blockIdx.x * kRows, t = blockIdx.y;
    const float* xt = x + static_cast<size_t>(t) * cols;
    const bool vec = (cols % 4 == 0) && ((reinterpret_cast<uintptr_t>(W) & 15) == 0);
    // chunk loader: element i of the 128 x 64 tile is (i / 64, i % 64); a
    // thread takes float4 number tid + 128 k, so a warp reads 512 contiguous
    // bytes of one row pair
    float4 reg[kPerThread];
    auto fetch = [&](uint32_t c0) {
#pragma unroll
        for (int k = 0; k < kPerThread; ++k) {
            const uint32_t v = tid + kRows * k, rr = v / (kChunk / 4), cc = (v % (kChunk / 4)) * 4;
            const uint32_t row = r0 + rr, col = c0 + cc;
            float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
            if (row < rows) {
                const float* src = W + static_cast<size_t>(row) * cols + col;
                if (vec && col + 3 < cols) {
                    f = __ldg(reinterpret_cast<const float4*>(src));
                } else {
                    if (col < cols) f.x = __ldg(src);
                    if (col + 1 < cols) f.y = __ldg(src + 1);
                    if (col + 2 < cols) f.z = __ldg(src + 2);
                    if (col + 3 < cols) f.w = __ldg(src + 3);
                }
            }
            reg[k] = f;
        }
    };
    double acc = 0.0;
    fetch(0);
    for (uint32_t c0 = 0; c0 < cols; c0 += kChunk) {
        __syncthreads();   // the previous chunk is summed
#pragma unroll
        for (int k = 0; k < kPerThread; ++k) {
            const uint32_t v = tid + kRows * k, rr = v / (kChunk / 4), cc = (v % (kChunk / 4)) * 4;
            float* d = ws + rr * kPitch + cc;
            d[0] = reg[k].x;
            d[1] = reg[k].y;
            d[2] = reg[k].z;
            d[3] = reg[k].w;
        }
        if (tid < kChunk) xs[tid] = c0 + tid < cols ? static_cast<double>(xt[c0 + tid]) : 0.0;
        __syncthreads();
        if (c0 + kChunk < cols) fetch(c0 + kChunk);
        // padding columns are 0 * 0: acc + 0 leaves the chain bit-identical
        const float* wr = ws + tid * kPitch;
#pragma unroll 16
        for (int c = 0; c < kChunk; ++c) acc = fma(static_cast<double>(wr[c]), xs[c], acc);
    }
    if (r0 + tid < rows) y[static_cast<size_t>(t) * rows + r0 + tid] = static_cast<float>(acc);
}

// The same chain over an MXFP4 matrix (mxfp4_matmul, runtime/src/ops.cpp:
// 44-76): w = ldexp(e2m1[code], scale - 127), exact in float (or infinite
// where the reference's is), so double(x) * w is exact and the fma chain in
// column order is bit-identical to the reference's. A thread owns its row:
// the 32 packed bytes and 2 scales of a 64-column chunk are one 32-byte
// sector of that row, held in registers (the next chunk's prefetched), and
// the shared x chunk is read as doubles.
__global__ void __launch_bounds__(kRows) mxfp4_matvec_kernel(const uint8_t* __restrict__ packed,
                                                             const uint8_t* __restrict__ scales, uint32_t rows,
                                                             uint32_t cols, const float* __restrict__ x,
                                                             float* __restrict__ y) {
    __shared__ double xs[kChunk];
    const uint32_t tid = threadIdx.x, r = blockIdx.x * kRows + tid, t = blockIdx.y;
    const float* xt = x + static_cast<size_t>(t) * cols;
    const bool live = r < rows;
    const uint8_t* prow = packed + static_cast<size_t>(r) * (cols / 2);
    const uint8_t* srow = scales + static_cast<size_t>(r) * (cols / 32);
    const bool vec = (reinterpret_cast<uintptr_t>(packed) & 15) == 0;   // rows are cols/2 = 16k bytes apart
    uint4 nq[2];
    uint32_t ns[2];
    auto fetch = [&](uint32_t c0) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            nq[hh] = make_uint4(0, 0, 0, 0);
            ns[hh] = 127;   // padding: code 0 at scale 1
            const uint32_t c = c0 + 32 * hh;
            if (!live || c >= cols) continue;
            const uint8_t* src = prow + c / 2;
            if (vec) {
                nq[hh] = __ldg(reinterpret_cast<const uint4*>(src));
            } else {
                uint32_t w[4] = {0, 0, 0, 0};
                for (int b = 0; b < 16; ++b) w[b / 4] |= static_cast<uint32_t>(__ldg(src + b)) << (8 * (b % 4));
                nq[hh] = make_uint4(w[0], w[1], w[2], w[3]);
            }
            ns[hh] = __ldg(srow + c / 32);
        }
    };
    double acc = 0.0;
    fetch(0);
    for (uint32_t c0 = 0; c0 < cols; c0 += kChunk) {
        const uint4 q[2] = {nq[0], nq[1]};
        const uint32_t s[2] = {ns[0], ns[1]};
        __syncthreads();   // the previous chunk's x is read
        if (tid < kChunk) xs[tid] = c0 + tid < cols ? static_cast<double>(xt[c0 + tid]) : 0.0;
        __syncthreads();
        if (c0 + kChunk < cols) fetch(c0 + kChunk);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const float scale = exp2i(static_cast<int>(s[hh]) - 127);
            const uint32_t words[4] = {q[hh].x, q[hh].y, q[hh].z, q[hh].w};
#pragma unroll
            for (int j = 0; j < 32; ++j) {   // column c0 + 32 hh + j: low nibble first (ops.cpp:52)
                const uint32_t code = (words[j / 8] >> (4 * (j % 8))) & 15u;
                const float mag = __fmul_rn(e2m1_magnitude(code & 7u), scale);
                const float w = (code & 8u) ? -mag : mag;
                acc = fma(xs[32 * hh + j], static_cast<double>(w), acc);
            }
        }
    }
    if (live) y[static_cast<size_t>(t) * rows + r] = static_cast<float>(acc);
}

// The resident layer's mix and routed norm (backend_cpu.cpp:320-329, ops.cpp:
// 10-18), one CTA: mixed[i] = sum over slots in order of contribution * y in
// float; the squares one FP64 chain in index order (a float square is exact
// in FP64); inverse = 1 / sqrt(float(squares / n) + eps) in float; out =
// mixed * inverse * weight, left to right.
__global__ void __launch_bounds__(256) resident_mix_norm_kernel(const float* __restrict__ y,
                                                                const float* __restrict__ contrib, uint32_t K,
                                                                uint32_t D, const float* __restrict__ weight, float eps,
                                                                float* __restrict__ mixed, float* __restrict__ out) {
    __shared__ float inverse;
    for (uint32_t i = threadIdx.x; i < D; i += blockDim.x) {
        float m = 0.0f;
        for (uint32_t k = 0; k < K; ++k) m = __fadd_rn(m, __fmul_rn(contrib[k], y[static_cast<size_t>(k) * D + i]));
        mixed[i] = m;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double squares = 0.0;
        for (uint32_t i = 0; i < D; ++i) squares = fma(static_cast<double>(mixed[i]), static_cast<double>(mixed[i]), squares);
        const float mean = static_cast<float>(squares / static_cast<double>(D));
        inverse = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < D; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(mixed[i], inverse), weight[i]);
}

__global__ void add_f32_kernel(const float* __restrict__ a, const float* __restrict__ b, uint32_t n,
                               float* __restrict__ out) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __fadd_rn(a[i], b[i]);
}

}  // namespace

int launch_mxfp4_matvec(k3xb_ctx* ctx, const uint8_t* packed, const uint8_t* scales, uint32_t rows, uint32_t cols,
                        const float* x, uint32_t T, float* y) {
    if (!rows || !cols || cols % 32 || !T || T > 65535)
        return fail(ctx, K3XB_INVALID_MXFP4, "mxfp4 matvec: cols a multiple of 32, 1 <= tokens <= 65535");
    const dim3 grid((rows + kRows - 1) / kRows, T);
    mxfp4_matvec_kernel<<<grid, kRows, 0, ctx->stream>>>(packed, scales, rows, cols, x, y);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_dense_matvec(k3xb_ctx* ctx, const float* W, uint32_t rows, uint32_t cols, const float* x, uint32_t T,
                        float* y) {
    if (!rows || !cols || !T || T > 65535) return fail(ctx, K3XB_INVALID_EXTENT, "dense matvec: 1 <= tokens <= 65535");
    const dim3 grid((rows + kRows - 1) / kRows, T);
    dense_matvec_kernel<<<grid, kRows, 0, ctx->stream>>>(W, rows, cols, x, y);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

}  // namespace k3xb

using namespace k3xb;

extern "C" {

int k3xb_dense_matvec(k3xb_ctx* ctx, const float* W, uint32_t rows, uint32_t cols, const float* x, uint32_t tokens,
                      float* y) {
    K3XB_ENTER(ctx);
    if (!W || !x || !y) return fail(ctx, K3XB_INVALID_EXTENT, "dense matvec arguments");
    return launch_dense_matvec(ctx, W, rows, cols, x, tokens, y);
}

int k3xb_dense_matvec_host(k3xb_ctx* ctx, const float* W, uint32_t rows, uint32_t cols, const float* x_host,
                           float* y_host) {
    K3XB_ENTER(ctx);
    if (!W || !x_host || !y_host || !rows || !cols) return fail(ctx, K3XB_INVALID_EXTENT, "dense matvec arguments");
    Sizer sz;
    sz.take<float>(cols);
    sz.take<float>(rows);
    void* base;
    int st;
    if ((st = ensure_io(ctx, sz.used, &base))) return st;
    Carver c(base);
    float* x = c.take<float>(cols);
    float* y = c.take<float>(rows);
    K3XB_CUDA(ctx, cudaMemcpyAsync(x, x_host, sizeof(float) * cols, cudaMemcpyHostToDevice, ctx->stream));
    if ((st = launch_dense_matvec(ctx, W, rows, cols, x, 1, y))) return st;
    K3XB_CUDA(ctx, cudaMemcpyAsync(y_host, y, sizeof(float) * rows, cudaMemcpyDeviceToHost, ctx->stream));
    ctx->stats.h2d_bytes += sizeof(float) * cols;
    ctx->stats.d2h_bytes += sizeof(float) * rows;
    return k3xb_sync(ctx);
}

int k3xb_dense_situ_mlp_host(k3xb_ctx* ctx, const float* gate, const float* up, const float* down, uint32_t inter,
                             uint32_t cols, uint32_t out_rows, const float* x_host, float beta, float linear_beta,
                             float* y_host) {
    K3XB_ENTER(ctx);
    if (!gate || !up || !down || !x_host || !y_host || !inter || !cols || !out_rows)
        return fail(ctx, K3XB_INVALID_EXTENT, "dense SiTU MLP arguments");
    if (!(beta > 0.0f) || linear_beta < 0.0f)
        return fail(ctx, K3XB_INVALID_EXTENT, "SiTU beta must be positive (linear beta 0 = none)");
    Sizer sz;
    sz.take<float>(cols);
    for (int i = 0; i < 3; ++i) sz.take<float>(inter);
    sz.take<float>(out_rows);
    void* base;
    int st;
    if ((st = ensure_io(ctx, sz.used, &base))) return st;
    Carver c(base);
    float* x = c.take<float>(cols);
    float* g = c.take<float>(inter);
    float* u = c.take<float>(inter);
    float* a = c.take<float>(inter);
    float* y = c.take<float>(out_rows);
    K3XB_CUDA(ctx, cudaMemcpyAsync(x, x_host, sizeof(float) * cols, cudaMemcpyHostToDevice, ctx->stream));
    // dense_situ_mlp (backend_cpu.cpp:107-122): gate and up, situ_glu, down
    if ((st = launch_dense_matvec(ctx, gate, inter, cols, x, 1, g))) return st;
    if ((st = launch_dense_matvec(ctx, up, inter, cols, x, 1, u))) return st;
    if ((st = launch_act(ctx, g, u, inter, K3XB_ACT_SITU, beta, linear_beta, a))) return st;
    if ((st = launch_dense_matvec(ctx, down, out_rows, inter, a, 1, y))) return st;
    K3XB_CUDA(ctx, cudaMemcpyAsync(y_host, y, sizeof(float) * out_rows, cudaMemcpyDeviceToHost, ctx->stream));
    ctx->stats.h2d_bytes += sizeof(float) * cols;
    ctx->stats.d2h_bytes += sizeof(float) * out_rows;
    return k3xb_sync(ctx);
}

}  // extern "C"

extern "C" {

int k3xb_mxfp4_matvec(k3xb_ctx* ctx, const uint8_t* packed, const uint8_t* scales, uint32_t rows, uint32_t cols,
                      const float* x, uint32_t tokens, float* y) {
    K3XB_ENTER(ctx);
    if (!packed || !scales || !x || !y) return fail(ctx, K3XB_INVALID_EXTENT, "mxfp4 matvec arguments");
    return launch_mxfp4_matvec(ctx, packed, scales, rows, cols, x, tokens, y);
}

int k3xb_mxfp4_matvec_host(k3xb_ctx* ctx, const uint8_t* packed, const uint8_t* scales, uint32_t rows, uint32_t cols,
                           const float* x_host, float* y_host) {
    K3XB_ENTER(ctx);
    if (!packed || !scales || !x_host || !y_host || !rows || !cols)
        return fail(ctx, K3XB_INVALID_EXTENT, "mxfp4 matvec arguments");
    Sizer sz;
    sz.take<float>(cols);
    sz.take<float>(rows);
    void* base;
    int st;
    if ((st = ensure_io(ctx, sz.used, &base))) return st;
    Carver c(base);
    float* x = c.take<float>(cols);
    float* y = c.take<float>(rows);
    K3XB_CUDA(ctx, cudaMemcpyAsync(x, x_host, sizeof(float) * cols, cudaMemcpyHostToDevice, ctx->stream));
    if ((st = launch_mxfp4_matvec(ctx, packed, scales, rows, cols, x, 1, y))) return st;
    K3XB_CUDA(ctx, cudaMemcpyAsync(y_host, y, sizeof(float) * rows, cudaMemcpyDeviceToHost, ctx->stream));
    ctx->stats.h2d_bytes += sizeof(float) * cols;
    ctx->stats.d2h_bytes += sizeof(float) * rows;
    return k3xb_sync(ctx);
}

int k3xb_resident_moe_layer_host(k3xb_ctx* ctx, uint32_t H, uint32_t D, uint32_t I, uint32_t Hs,
                                 const float* routed_down, const float* routed_norm, const float* routed_up,
                                 const float* shared_gate, const float* shared_up, const float* shared_down,
                                 const k3xb_mxfp4_expert* experts, uint32_t K, const float* contrib_host, float eps,
                                 float beta, float linear_beta, const float* x_host, float* y_host) {
    K3XB_ENTER(ctx);
    if (!H || !D || !I || !Hs || !routed_down || !routed_norm || !routed_up || !shared_gate || !shared_up ||
        !shared_down || !experts || !K || !contrib_host || !x_host || !y_host)
        return fail(ctx, K3XB_INVALID_EXTENT, "resident moe layer arguments");
    if (D % 32 || I % 32) return fail(ctx, K3XB_INVALID_MXFP4, "resident moe layer: latent and inter multiples of 32");
    if (!(eps > 0.0f) || !(beta > 0.0f) || linear_beta < 0.0f)
        return fail(ctx, K3XB_INVALID_EXTENT, "resident moe layer: eps and SiTU beta positive");
    for (uint32_t k = 0; k < K; ++k) {
        const k3xb_mxfp4_expert& e = experts[k];
        if (!e.gate_packed || !e.gate_scales || !e.up_packed || !e.up_scales || !e.down_packed || !e.down_scales)
            return fail(ctx, K3XB_INVALID_EXTENT, "resident moe layer: missing expert weights");
    }
    Sizer sz;
    sz.take<float>(H);                    // x
    sz.take<float>(K);                    // contributions
    sz.take<float>(D);                    // latent
    for (int i = 0; i < 3; ++i) sz.take<float>(I);    // expert gate, up, activation
    sz.take<float>(static_cast<size_t>(K) * D);       // expert outputs
    for (int i = 0; i < 2; ++i) sz.take<float>(D);    // mixed, normalized
    for (int i = 0; i < 3; ++i) sz.take<float>(Hs);   // shared gate, up, activation
    for (int i = 0; i < 3; ++i) sz.take<float>(H);    // routed, shared, out
    void* base;
    int st;
    if ((st = ensure_io(ctx, sz.used, &base))) return st;
    Carver c(base);
    float* x = c.take<float>(H);
    float* contrib = c.take<float>(K);
    float* latent = c.take<float>(D);
    float* g = c.take<float>(I);
    float* u = c.take<float>(I);
    float* a = c.take<float>(I);
    float* y = c.take<float>(static_cast<size_t>(K) * D);
    float* mixed = c.take<float>(D);
    float* normed = c.take<float>(D);
    float* sg = c.take<float>(Hs);
    float* su = c.take<float>(Hs);
    float* sa = c.take<float>(Hs);
    float* routed = c.take<float>(H);
    float* shared = c.take<float>(H);
    float* out = c.take<float>(H);
    K3XB_CUDA(ctx, cudaMemcpyAsync(x, x_host, sizeof(float) * H, cudaMemcpyHostToDevice, ctx->stream));
    K3XB_CUDA(ctx, cudaMemcpyAsync(contrib, contrib_host, sizeof(float) * K, cudaMemcpyHostToDevice, ctx->stream));
    ctx->stats.h2d_bytes += sizeof(float) * (H + K);
    // backend_cpu.cpp:316-338: latent, the experts (mxfp4_situ_mlp_group, :132-153), mix, routed norm, up, shared
    if ((st = launch_dense_matvec(ctx, routed_down, D, H, x, 1, latent))) return st;
    for (uint32_t k = 0; k < K; ++k) {
        const k3xb_mxfp4_expert& e = experts[k];
        if ((st = launch_mxfp4_matvec(ctx, e.gate_packed, e.gate_scales, I, D, latent, 1, g))) return st;
        if ((st = launch_mxfp4_matvec(ctx, e.up_packed, e.up_scales, I, D, latent, 1, u))) return st;
        if ((st = launch_act(ctx, g, u, I, K3XB_ACT_SITU, beta, linear_beta, a))) return st;
        if ((st = launch_mxfp4_matvec(ctx, e.down_packed, e.down_scales, D, I, a, 1, y + static_cast<size_t>(k) * D)))
            return st;
    }
    resident_mix_norm_kernel<<<1, 256, 0, ctx->stream>>>(y, contrib, K, D, routed_norm, eps, mixed, normed);
    K3XB_LAUNCHED(ctx);
    if ((st = launch_dense_matvec(ctx, routed_up, H, D, normed, 1, routed))) return st;
    if ((st = launch_dense_matvec(ctx, shared_gate, Hs, H, x, 1, sg))) return st;
    if ((st = launch_dense_matvec(ctx, shared_up, Hs, H, x, 1, su))) return st;
    if ((st = launch_act(ctx, sg, su, Hs, K3XB_ACT_SITU, beta, linear_beta, sa))) return st;
    if ((st = launch_dense_matvec(ctx, shared_down, H, Hs, sa, 1, shared))) return st;
    add_f32_kernel<<<(H + 255) / 256, 256, 0, ctx->stream>>>(routed, shared, H, out);
    K3XB_LAUNCHED(ctx);
    K3XB_CUDA(ctx, cudaMemcpyAsync(y_host, out, sizeof(float) * H, cudaMemcpyDeviceToHost, ctx->stream));
    ctx->stats.d2h_bytes += sizeof(float) * H;
    ++ctx->stats.moe_layer_calls;
    return k3xb_sync(ctx);
}

}  // extern "C"
