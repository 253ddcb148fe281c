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

}  // namespace

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
