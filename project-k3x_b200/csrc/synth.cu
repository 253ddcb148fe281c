// synth.cu — seeded synthetic data and the MXFP4 quantiser.
//
// The generator is counter-based (SplitMix64 of (seed, stream, pair index)
// -> two 24-bit uniforms -> Box-Muller), so any element can be regenerated
// independently and weights of any size are produced in place on the GPU.
// Box-Muller's log and sine/cosine are this file's own short series in
// float, every operation rounded to nearest (no contraction), so a host
// restatement with the same operations (oracle/k3x_oracle.c:k3xo_normal_pair)
// gives the same bits and a CPU can rebuild any slice of a workload.
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

// ln(k * 2^-24) for k in [1, 2^24]: k = m * 2^e with m in [sqrt(1/2), sqrt(2)),
// ln m = 2 atanh(s) with s = (m - 1) / (m + 1), |s| < 0.172, by its series to
// s^11 (truncation below 1e-10); e * ln 2 with ln 2 rounded to float. The
// coefficients are the floats nearest 1/3, 1/5, ..., 1/11.
__device__ __forceinline__ float synth_log(uint32_t k) {
    int e = 31 - __clz(k);                         // k in [2^e, 2^(e+1))
    const uint32_t mant = e <= 23 ? k << (23 - e) : k >> (e - 23);
    float m = __uint_as_float((mant & 0x7fffffu) | 0x3f800000u);
    if (m > 0x1.6a09e6p+0f) {                      // sqrt(2)
        m = __fmul_rn(m, 0.5f);
        ++e;
    }
    const float s = __fdiv_rn(__fadd_rn(m, -1.0f), __fadd_rn(m, 1.0f));
    const float s2 = __fmul_rn(s, s);
    float p = 0x1.745d18p-4f;                      // 1/11
    p = __fadd_rn(__fmul_rn(p, s2), 0x1.c71c72p-4f);   // 1/9
    p = __fadd_rn(__fmul_rn(p, s2), 0x1.24924ap-3f);   // 1/7
    p = __fadd_rn(__fmul_rn(p, s2), 0x1.99999ap-3f);   // 1/5
    p = __fadd_rn(__fmul_rn(p, s2), 0x1.555556p-2f);   // 1/3
    p = __fadd_rn(__fmul_rn(p, s2), 1.0f);
    const float lnm = __fmul_rn(__fmul_rn(2.0f, s), p);
    return __fadd_rn(__fmul_rn(static_cast<float>(e - 24), 0x1.62e430p-1f), lnm);   // ln 2
}

// cos and sin of 2*pi*k*2^-24 for k in [0, 2^24): the quadrant from k's top
// two bits, x = 2*pi*f with f in [0, 1/4) exact, Taylor series to x^14 and
// x^15 (truncation below 1e-11 on [0, pi/2)); the coefficients are the
// floats nearest +-1/n!.
__device__ __forceinline__ float2 synth_cos_sin(uint32_t k) {
    const uint32_t q = k >> 22;
    const float f = static_cast<float>(k & 0x3fffffu) * 0x1.0p-24f;
    const float x = __fmul_rn(f, 0x1.921fb6p+2f), x2 = __fmul_rn(x, x);   // 2 pi
    float c = -0x1.93974cp-37f, sn = -0x1.ae7f3ep-41f;                    // -1/14!, -1/15!
    c = __fadd_rn(__fmul_rn(c, x2), 0x1.1eed8ep-29f);    // 1/12!
    c = __fadd_rn(__fmul_rn(c, x2), -0x1.27e4fcp-22f);   // -1/10!
    c = __fadd_rn(__fmul_rn(c, x2), 0x1.a01a02p-16f);    // 1/8!
    c = __fadd_rn(__fmul_rn(c, x2), -0x1.6c16c2p-10f);   // -1/6!
    c = __fadd_rn(__fmul_rn(c, x2), 0x1.555556p-5f);     // 1/4!
    c = __fadd_rn(__fmul_rn(c, x2), -0.5f);
    c = __fadd_rn(__fmul_rn(c, x2), 1.0f);
    sn = __fadd_rn(__fmul_rn(sn, x2), 0x1.612462p-33f);  // 1/13!
    sn = __fadd_rn(__fmul_rn(sn, x2), -0x1.ae6456p-26f); // -1/11!
    sn = __fadd_rn(__fmul_rn(sn, x2), 0x1.71de3ap-19f);  // 1/9!
    sn = __fadd_rn(__fmul_rn(sn, x2), -0x1.a01a02p-13f); // -1/7!
    sn = __fadd_rn(__fmul_rn(sn, x2), 0x1.111112p-7f);   // 1/5!
    sn = __fadd_rn(__fmul_rn(sn, x2), -0x1.555556p-3f);  // -1/3!
    sn = __fadd_rn(__fmul_rn(__fmul_rn(sn, x2), x), x);
    switch (q) {
        case 0: return make_float2(c, sn);
        case 1: return make_float2(-sn, c);
        case 2: return make_float2(-c, -sn);
        default: return make_float2(sn, -c);
    }
}

// Standard normal pair for pair index i.
__device__ __forceinline__ float2 normal_pair(uint64_t seed, uint64_t stream, uint64_t i) {
    const uint64_t r = mix64(mix64(mix64(seed) ^ stream) ^ i);
    const uint32_t k1 = static_cast<uint32_t>(r >> 40) + 1u;           // u1 = k1 * 2^-24 in (0, 1]
    const uint32_t k2 = static_cast<uint32_t>((r >> 16) & 0xffffffu);  // u2 = k2 * 2^-24 in [0, 1)
    const float rad = __fsqrt_rn(__fmul_rn(-2.0f, synth_log(k1)));
    const float2 cs = synth_cos_sin(k2);
    return make_float2(__fmul_rn(rad, cs.x), __fmul_rn(rad, cs.y));
}

__global__ void fill_normal_kernel(float* out, size_t n, uint64_t seed, uint64_t stream, float mean,
                                   float sigma) {
    const size_t pair = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (2 * pair >= n) return;
    const float2 z = normal_pair(seed, stream, pair);
    out[2 * pair] = __fadd_rn(mean, __fmul_rn(sigma, z.x));
    if (2 * pair + 1 < n) out[2 * pair + 1] = __fadd_rn(mean, __fmul_rn(sigma, z.y));
}

__global__ void fill_normal_bf16_kernel(uint16_t* out, size_t n, uint64_t seed, uint64_t stream,
                                        float sigma) {
    const size_t pair = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (2 * pair >= n) return;
    const float2 z = normal_pair(seed, stream, pair);
    out[2 * pair] = encode_bf16(__fmul_rn(sigma, z.x));
    if (2 * pair + 1 < n) out[2 * pair + 1] = encode_bf16(__fmul_rn(sigma, z.y));
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
        v[2 * i] = __fmul_rn(sigma, z.x);
        v[2 * i + 1] = __fmul_rn(sigma, z.y);
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
