// synth.cu — seeded synthetic data and the MXFP4 quantiser.
//
// The generator is counter-based (SplitMix64 of (seed, stream, pair index)
// -> two 24-bit uniforms -> Box-Muller), so any element can be regenerated
// independently and weights of any size are produced in place on the GPU.
// The quantiser matches oracle/k3x_oracle.c:k3xo_quantize_mxfp4 bit for
// bit: per 32-block s = smallest integer with amax <= 6*2^s, E2M1 codes by
// round-to-nearest-even (scaling by 2^-s is exact).
#include "common.cuh"
#include "kernels.cuh"

namespace k3xb {

namespace {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

// Standard normal pair for pair index i.
__device__ __forceinline__ float2 normal_pair(uint64_t seed, uint64_t stream, uint64_t i) {
    const uint64_t r = mix64(mix64(mix64(seed) ^ stream) ^ i);
    const float u1 = (static_cast<float>(r >> 40) + 1.0f) * 0x1.0p-24f;   // (0, 1]
    const float u2 = static_cast<float>((r >> 16) & 0xffffffu) * 0x1.0p-24f;
    const float rad = sqrtf(-2.0f * logf(u1));
    float sn, cs;
    sincospif(2.0f * u2, &sn, &cs);
    return make_float2(rad * cs, rad * sn);
}

__global__ void fill_normal_kernel(float* out, size_t n, uint64_t seed, uint64_t stream, float mean,
                                   float sigma) {
    const size_t pair = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (2 * pair >= n) return;
    const float2 z = normal_pair(seed, stream, pair);
    out[2 * pair] = mean + sigma * z.x;
    if (2 * pair + 1 < n) out[2 * pair + 1] = mean + sigma * z.y;
}

__global__ void fill_normal_bf16_kernel(uint16_t* out, size_t n, uint64_t seed, uint64_t stream,
                                        float sigma) {
    const size_t pair = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (2 * pair >= n) return;
    const float2 z = normal_pair(seed, stream, pair);
    out[2 * pair] = encode_bf16(sigma * z.x);
    if (2 * pair + 1 < n) out[2 * pair + 1] = encode_bf16(sigma * z.y);
}

__device__ __forceinline__ void quantize_block32(const float (&x)[32], uint8_t* packed, uint8_t* scale) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
    const int s = amax > 0.0f ? e2m1_block_exponent(amax) : 0;
    *scale = static_cast<uint8_t>(s + 127);
    const float inv = exp2i(-s);
    uint32_t words[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        uint32_t acc = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float v = x[8 * w + i];
            const uint32_t code = e2m1_code(fabsf(v) * inv);
            const uint32_t nib = code | ((signbit(v) && code) ? 8u : 0u);
            acc |= nib << (4 * i);
        }
        words[w] = acc;
    }
    *reinterpret_cast<uint4*>(packed) = make_uint4(words[0], words[1], words[2], words[3]);
}

__global__ void quantize_mxfp4_kernel(const float* __restrict__ x, size_t blocks, uint8_t* packed,
                                      uint8_t* scales) {
    const size_t b = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (b >= blocks) return;
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
        const float4 q = *reinterpret_cast<const float4*>(x + b * 32 + i);
        v[i] = q.x; v[i + 1] = q.y; v[i + 2] = q.z; v[i + 3] = q.w;
    }
    quantize_block32(v, packed + b * 16, scales + b);
}

__global__ void fill_normal_mxfp4_kernel(size_t blocks, uint64_t seed, uint64_t stream, float sigma,
                                         uint8_t* packed, uint8_t* scales) {
    const size_t b = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (b >= blocks) return;
    float v[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float2 z = normal_pair(seed, stream, b * 16 + i);
        v[2 * i] = sigma * z.x;
        v[2 * i + 1] = sigma * z.y;
    }
    quantize_block32(v, packed + b * 16, scales + b);
}

}  // namespace

int launch_fill_normal_f32(k3xb_ctx* ctx, float* out, size_t n, uint64_t seed, uint64_t stream,
                           float mean, float sigma) {
    const size_t pairs = (n + 1) / 2;
    fill_normal_kernel<<<static_cast<unsigned>((pairs + 255) / 256), 256, 0, ctx->stream>>>(
        out, n, seed, stream, mean, sigma);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_fill_normal_bf16(k3xb_ctx* ctx, uint16_t* out, size_t n, uint64_t seed, uint64_t stream,
                            float sigma) {
    const size_t pairs = (n + 1) / 2;
    fill_normal_bf16_kernel<<<static_cast<unsigned>((pairs + 255) / 256), 256, 0, ctx->stream>>>(
        out, n, seed, stream, sigma);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_quantize_mxfp4(k3xb_ctx* ctx, const float* x, size_t rows, size_t cols, uint8_t* packed,
                          uint8_t* scales) {
    const size_t blocks = rows * cols / 32;
    quantize_mxfp4_kernel<<<static_cast<unsigned>((blocks + 255) / 256), 256, 0, ctx->stream>>>(
        x, blocks, packed, scales);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

int launch_fill_normal_mxfp4(k3xb_ctx* ctx, uint8_t* packed, uint8_t* scales, size_t rows, size_t cols,
                             uint64_t seed, uint64_t stream, float sigma) {
    const size_t blocks = rows * cols / 32;
    fill_normal_mxfp4_kernel<<<static_cast<unsigned>((blocks + 255) / 256), 256, 0, ctx->stream>>>(
        blocks, seed, stream, sigma, packed, scales);
    K3XB_LAUNCHED(ctx);
    return K3XB_OK;
}

}  // namespace k3xb
