/*
 * k3x_oracle.c — CPU restatement of the K3X speculative-verification path.
 *
 * TEST INFRASTRUCTURE ONLY (see k3x_oracle.h). Plain C99, no threads, no
 * allocation beyond scratch buffers. Each function names the reference
 * file:line it restates; the restatement is checked against the
 * reference's own compiled code in tests/test_oracle_pin.py.
 *
 * Compile with strict IEEE semantics (no -ffast-math, no FMA contraction):
 * the reference is built for baseline x86-64 (no FMA), so every a*b+c in
 * it rounds twice, and so must this file.
 */
#include "k3x_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* scalar numerics                                                           */
/* ------------------------------------------------------------------------ */

static uint32_t f2u(float v) { uint32_t u; memcpy(&u, &v, 4); return u; }
static float u2f(uint32_t u) { float v; memcpy(&v, &u, 4); return v; }

/* official_moe.cpp:18-26 */
float k3xo_round_bf16(float value)
{
    uint32_t bits = f2u(value);
    if ((bits & 0x7f800000u) == 0x7f800000u) {
        if (bits & 0x007fffffu) bits |= 0x00400000u;
        return u2f(bits & 0xffff0000u);
    }
    bits += 0x7fffu + ((bits >> 16) & 1u);
    return u2f(bits & 0xffff0000u);
}

/* official_kda.cpp:31-39 */
uint16_t k3xo_encode_bf16(float value)
{
    uint32_t bits = f2u(value);
    if ((bits & 0x7f800000u) == 0x7f800000u) {
        if (bits & 0x007fffffu) bits |= 0x00400000u;
        return (uint16_t)(bits >> 16);
    }
    bits += 0x7fffu + ((bits >> 16) & 1u);
    return (uint16_t)(bits >> 16);
}

/* official_moe.cpp:135-137 */
float k3xo_decode_bf16(uint16_t word) { return u2f((uint32_t)word << 16); }

static const float kE2m1[16] = {
    0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
    -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f,
};

/* ops.cpp:40-43 */
float k3xo_e2m1_value(uint8_t code) { return kE2m1[code & 15u]; }

static int all_finite(const float* v, size_t n)
{
    for (size_t i = 0; i < n; ++i)
        if (!isfinite(v[i])) return 0;
    return 1;
}

/* ------------------------------------------------------------------------ */
/* MXFP4                                                                     */
/* ------------------------------------------------------------------------ */

static int mxfp4_shape_ok(size_t rows, size_t cols, size_t group)
{
    return rows && cols && group && cols % group == 0 && cols % 2 == 0;
}

/* ops.cpp:32-55 */
int k3xo_decode_mxfp4(const uint8_t* packed, const uint8_t* scales,
                      size_t rows, size_t cols, size_t group, float* out)
{
    if (!mxfp4_shape_ok(rows, cols, group)) return K3XO_INVALID_MXFP4;
    for (size_t i = 0; i < rows * cols / group; ++i)
        if (scales[i] == 0xffu) return K3XO_INVALID_MXFP4;
    for (size_t i = 0; i < rows * cols; ++i) {
        uint8_t pair = packed[i / 2];
        uint8_t code = (i % 2) ? (uint8_t)(pair >> 4) : (uint8_t)(pair & 15u);
        out[i] = ldexpf(kE2m1[code], (int)scales[i / group] - 127);
    }
    return K3XO_OK;
}

/* ops.cpp:57-76. The reference decodes the whole matrix first and then
 * sums double(x[c]) * decoded[r][c] left to right; decoding on the fly
 * gives the same float operands in the same order. */
int k3xo_mxfp4_matmul(const float* x, const uint8_t* packed,
                      const uint8_t* scales, size_t rows, size_t cols,
                      size_t group, float* out)
{
    if (!mxfp4_shape_ok(rows, cols, group)) return K3XO_INVALID_MXFP4;
    for (size_t i = 0; i < rows * cols / group; ++i)
        if (scales[i] == 0xffu) return K3XO_INVALID_MXFP4;
    for (size_t r = 0; r < rows; ++r) {
        const uint8_t* prow = packed + r * (cols / 2);
        const uint8_t* srow = scales + r * (cols / group);
        double sum = 0.0;
        for (size_t c = 0; c < cols; ++c) {
            uint8_t pair = prow[c / 2];
            uint8_t code = (c % 2) ? (uint8_t)(pair >> 4) : (uint8_t)(pair & 15u);
            float w = ldexpf(kE2m1[code], (int)srow[c / group] - 127);
            sum += (double)x[c] * (double)w;
        }
        out[r] = (float)sum;
    }
    return K3XO_OK;
}

/* E2M1 round-to-nearest, ties to the even code, saturating at 6. */
uint8_t k3xo_e2m1_code(float a)
{
    if (a <= 0.25f) return 0;
    if (a < 0.75f) return 1;
    if (a <= 1.25f) return 2;
    if (a < 1.75f) return 3;
    if (a <= 2.5f) return 4;
    if (a < 3.5f) return 5;
    if (a <= 5.0f) return 6;
    return 7;
}

/* Smallest s with amax <= 6 * 2^s (amax > 0, finite): with
 * amax = m * 2^E, m in [0.5, 1): s = E-3 when m <= 0.75, else E-2. */
static int e2m1_block_exponent(float amax)
{
    int e = 0;
    float m = frexpf(amax, &e);
    int s = (m <= 0.75f) ? e - 3 : e - 2;
    if (s < -127) s = -127;
    if (s > 127) s = 127;
    return s;
}

void k3xo_quantize_mxfp4(const float* x, size_t rows, size_t cols,
                         uint8_t* packed, uint8_t* scales)
{
    for (size_t r = 0; r < rows; ++r) {
        for (size_t b = 0; b < cols / 32; ++b) {
            const float* blk = x + r * cols + b * 32;
            float amax = 0.0f;
            for (int i = 0; i < 32; ++i) {
                float a = fabsf(blk[i]);
                if (a > amax) amax = a;
            }
            int s = amax > 0.0f ? e2m1_block_exponent(amax) : 0;
            scales[r * (cols / 32) + b] = (uint8_t)(s + 127);
            uint8_t* out = packed + r * (cols / 2) + b * 16;
            for (int i = 0; i < 16; ++i) {
                uint8_t nib[2];
                for (int h = 0; h < 2; ++h) {
                    float v = blk[2 * i + h];
                    uint8_t code = k3xo_e2m1_code(ldexpf(fabsf(v), -s));
                    nib[h] = (uint8_t)(code | (signbit(v) && code ? 8u : 0u));
                }
                out[i] = (uint8_t)(nib[0] | (nib[1] << 4));
            }
        }
    }
}

float k3xo_e2m1_terms(const float* x32, int nterms, uint8_t* packed,
                      uint8_t* scales)
{
    float r[32];
    memcpy(r, x32, sizeof r);
    for (int t = 0; t < nterms; ++t) {
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) {
            float a = fabsf(r[i]);
            if (a > amax) amax = a;
        }
        int s = amax > 0.0f ? e2m1_block_exponent(amax) : 0;
        scales[t] = (uint8_t)(s + 127);
        for (int i = 0; i < 16; ++i) {
            uint8_t nib[2];
            for (int h = 0; h < 2; ++h) {
                float v = r[2 * i + h];
                uint8_t code = k3xo_e2m1_code(ldexpf(fabsf(v), -s));
                int neg = signbit(v) && code;
                nib[h] = (uint8_t)(code | (neg ? 8u : 0u));
                float q = ldexpf(kE2m1[code], s);
                r[2 * i + h] = v - (neg ? -q : q);
            }
            packed[t * 16 + i] = (uint8_t)(nib[0] | (nib[1] << 4));
        }
    }
    float res = 0.0f;
    for (int i = 0; i < 32; ++i)
        if (fabsf(r[i]) > res) res = fabsf(r[i]);
    return res;
}

/* ------------------------------------------------------------------------ */
/* elementwise / small                                                       */
/* ------------------------------------------------------------------------ */

/* ops.cpp:20-30 */
void k3xo_situ_glu(float* out, const float* gate, const float* up, size_t n,
                   float beta, float linear_beta)
{
    for (size_t i = 0; i < n; ++i) {
        float sigmoid = 1.0f / (1.0f + expf(-gate[i]));
        float bounded_gate = beta * tanhf(gate[i] / beta) * sigmoid;
        float bounded_up = linear_beta > 0.0f
            ? linear_beta * tanhf(up[i] / linear_beta) : up[i];
        out[i] = bounded_gate * bounded_up;
    }
}

void k3xo_swiglu(float* out, const float* gate, const float* up, size_t n)
{
    for (size_t i = 0; i < n; ++i) {
        float sigmoid = 1.0f / (1.0f + expf(-gate[i]));
        float g = gate[i] * sigmoid;
        out[i] = g * up[i];
    }
}

static void activate(float* out, const float* g, const float* u, size_t n,
                     int activation, float beta, float linear_beta)
{
    if (activation == K3XO_ACT_SITU)
        k3xo_situ_glu(out, g, u, n, beta, linear_beta);
    else
        k3xo_swiglu(out, g, u, n);
}

/* official_moe.cpp:39-59 */
int k3xo_bf16_matvec(const float* x, const uint16_t* w, size_t rows,
                     size_t cols, float* out)
{
    if (!rows || !cols || !all_finite(x, cols)) return K3XO_INVALID_EXTENT;
    for (size_t r = 0; r < rows; ++r) {
        double sum = 0.0;
        for (size_t c = 0; c < cols; ++c) {
            float v = k3xo_decode_bf16(w[r * cols + c]);
            if (!isfinite(v)) return K3XO_INVALID_EXTENT;
            sum += (double)v * x[c];
        }
        out[r] = k3xo_round_bf16((float)sum);
    }
    return K3XO_OK;
}

/* backend_cpu.cpp:23-47: the CPU backend's f32 dense product, one double
 * chain per row in column order (its validity check, :368-377, is shapes
 * only: non-finite values pass through). */
int k3xo_dense_matvec(const float* x, const float* w, size_t rows, size_t cols,
                      float* out)
{
    for (size_t r = 0; r < rows; ++r) {
        double sum = 0.0;
        for (size_t c = 0; c < cols; ++c) sum += (double)w[r * cols + c] * x[c];
        out[r] = (float)sum;
    }
    return K3XO_OK;
}

/* official_layer.cpp:104-125 (== official_moe.cpp:61-80 for finite input) */
int k3xo_rms_norm_bf16(const float* x, const uint16_t* weight, size_t n,
                       float eps, float* out)
{
    if (!n || !all_finite(x, n) || !isfinite(eps) || eps <= 0.0f)
        return K3XO_INVALID_EXTENT;
    double squares = 0.0;
    for (size_t i = 0; i < n; ++i) squares += (double)x[i] * x[i];
    float inverse = 1.0f / sqrtf((float)(squares / n) + eps);
    for (size_t i = 0; i < n; ++i) {
        out[i] = k3xo_round_bf16(x[i] * inverse * k3xo_decode_bf16(weight[i]));
        if (!isfinite(out[i])) return K3XO_INVALID_EXTENT;
    }
    return K3XO_OK;
}

static float residual_score(const float* v, const uint16_t* norm,
                            const uint16_t* proj, size_t n, float eps)
{
    double squares = 0.0;
    for (size_t i = 0; i < n; ++i) squares += (double)v[i] * v[i];
    float inverse = 1.0f / sqrtf((float)(squares / n) + eps);
    double result = 0.0;
    for (size_t i = 0; i < n; ++i)
        result += (double)(v[i] * inverse) * k3xo_decode_bf16(norm[i]) *
                  k3xo_decode_bf16(proj[i]);
    return (float)result;
}

/* official_layer.cpp:42-102 */
int k3xo_attention_residual(const float* prefix, const float* block,
                            const uint16_t* norm, const uint16_t* proj,
                            size_t n, float eps, float* out)
{
    if (!n || !all_finite(prefix, n) || !all_finite(block, n))
        return K3XO_INVALID_EXTENT;
    float* rp = (float*)malloc(n * sizeof(float));
    float* rb = (float*)malloc(n * sizeof(float));
    for (size_t i = 0; i < n; ++i) {
        rp[i] = k3xo_round_bf16(prefix[i]);
        rb[i] = k3xo_round_bf16(block[i]);
    }
    float block_score = residual_score(rb, norm, proj, n, eps);
    float prefix_score = residual_score(rp, norm, proj, n, eps);
    float maximum = block_score > prefix_score ? block_score : prefix_score;
    float block_exp = expf(block_score - maximum);
    float prefix_exp = expf(prefix_score - maximum);
    float denominator = block_exp + prefix_exp;
    float pb = block_exp / denominator;
    float pp = prefix_exp / denominator;
    for (size_t i = 0; i < n; ++i) out[i] = k3xo_round_bf16(pb * rb[i] + pp * rp[i]);
    free(rp);
    free(rb);
    return K3XO_OK;
}

/* ops.cpp:10-18 */
void k3xo_rms_norm_f32(const float* x, const float* weight, size_t n,
                       float eps, float* out)
{
    double squares = 0.0;
    for (size_t i = 0; i < n; ++i) squares += (double)x[i] * x[i];
    float inverse = 1.0f / sqrtf((float)(squares / n) + eps);
    for (size_t i = 0; i < n; ++i) out[i] = x[i] * inverse * weight[i];
}

/* model.cpp:645-666: values = the S sources in push order, then the prefix;
 * key = rms_norm(value, norm); score = float inner product of key and
 * projection (std::inner_product from 0.0F); softmax in float with the sum
 * taken in depth order; out = sum_d p_d * value_d from 0, in depth order. */
int k3xo_block_attention_residual(const float* prefix, const float* sources,
                                  size_t S, size_t T, size_t H,
                                  const float* norm, const float* proj,
                                  float eps, float* out)
{
    if (!H || !T || (S && !sources)) return K3XO_INVALID_EXTENT;
    float* key = (float*)malloc(H * sizeof(float));
    float* scores = (float*)malloc((S + 1) * sizeof(float));
    if (!key || !scores) {
        free(key);
        free(scores);
        return K3XO_INVALID_EXTENT;
    }
    for (size_t t = 0; t < T; ++t) {
        for (size_t d = 0; d <= S; ++d) {
            const float* v = d < S ? sources + (d * T + t) * H : prefix + t * H;
            k3xo_rms_norm_f32(v, norm, H, eps, key);
            float score = 0.0f;
            for (size_t i = 0; i < H; ++i) score = score + key[i] * proj[i];
            scores[d] = score;
        }
        float maximum = scores[0];
        for (size_t d = 1; d <= S; ++d)
            if (scores[d] > maximum) maximum = scores[d];
        float denominator = 0.0f;
        for (size_t d = 0; d <= S; ++d) {
            scores[d] = expf(scores[d] - maximum);
            denominator += scores[d];
        }
        float* o = out + t * H;
        for (size_t i = 0; i < H; ++i) o[i] = 0.0f;
        for (size_t d = 0; d <= S; ++d) {
            const float p = scores[d] / denominator;
            const float* v = d < S ? sources + (d * T + t) * H : prefix + t * H;
            for (size_t i = 0; i < H; ++i) o[i] += p * v[i];
        }
    }
    free(key);
    free(scores);
    return K3XO_OK;
}

/* ------------------------------------------------------------------------ */
/* router (a)                                                                */
/* ------------------------------------------------------------------------ */

/* official_moe.cpp:255-267 */
int k3xo_router_logits(const float* hidden, const uint16_t* w, size_t experts,
                       size_t hidden_size, float* logits)
{
    if (!experts || !hidden_size || !all_finite(hidden, hidden_size))
        return K3XO_INVALID_EXTENT;
    for (size_t e = 0; e < experts; ++e) {
        double sum = 0.0;
        for (size_t h = 0; h < hidden_size; ++h) {
            float weight = k3xo_decode_bf16(w[e * hidden_size + h]);
            if (!isfinite(weight)) return K3XO_INVALID_EXTENT;
            sum += (double)weight * hidden[h];
        }
        logits[e] = (float)sum;
    }
    return K3XO_OK;
}

/* official_moe.cpp:211-245. The reference's partial_sort uses the strict
 * total order (adjusted desc, index asc); any exact selection under that
 * order yields the same ids, so a simple insertion selection is used. */
int k3xo_route_logits(const float* logits, const float* correction,
                      size_t experts, size_t top_k, uint32_t* ids,
                      float* contributions, float* scores_out)
{
    if (!experts || !top_k || top_k > experts || !all_finite(logits, experts) ||
        !all_finite(correction, experts))
        return K3XO_INVALID_EXTENT;
    float* scores = (float*)malloc(experts * sizeof(float));
    float* adjusted = (float*)malloc(experts * sizeof(float));
    for (size_t e = 0; e < experts; ++e) {
        scores[e] = 1.0f / (1.0f + expf(-logits[e]));
        adjusted[e] = scores[e] + correction[e];
    }
    for (size_t slot = 0; slot < top_k; ++slot) {
        size_t best = (size_t)-1;
        for (size_t e = 0; e < experts; ++e) {
            int taken = 0;
            for (size_t j = 0; j < slot; ++j)
                if (ids[j] == e) { taken = 1; break; }
            if (taken) continue;
            if (best == (size_t)-1 || adjusted[e] > adjusted[best]) best = e;
        }
        ids[slot] = (uint32_t)best;
    }
    double total = 0.0;
    for (size_t slot = 0; slot < top_k; ++slot) total += scores[ids[slot]];
    int status = K3XO_OK;
    if (!isfinite(total) || total <= 0.0) {
        status = K3XO_INVALID_EXTENT;
    } else {
        for (size_t slot = 0; slot < top_k; ++slot)
            contributions[slot] = (float)(scores[ids[slot]] / total);
        if (scores_out) memcpy(scores_out, scores, experts * sizeof(float));
    }
    free(scores);
    free(adjusted);
    return status;
}

/* routing_policy.cpp:12-29 */
static int routing_k_allowed(size_t k)
{
    return k == 4 || k == 6 || k == 8 || k == 12 || k == 16;
}

static float routing_boundary(const float* probs, size_t n, size_t k)
{
    if (k >= n) return 1.0f;
    float gap = probs[k - 1] - probs[k];
    if (gap < 0.0f) gap = 0.0f;
    float top = probs[0] > FLT_MIN ? probs[0] : FLT_MIN;
    return gap / top;
}

/* routing_policy.cpp:109-128: first ladder K past the floor that reaches the
 * mass target, the entropy support and the boundary gap; else natural_k */
static size_t routing_adaptive_k(const float* probs, size_t n, float support, float mass_target,
                                 float minimum_gap, size_t floor_k)
{
    const float eps = 1.0e-5f;
    float cumulative = 0.0f;
    for (size_t slot = 0; slot < n; ++slot) {
        cumulative += probs[slot];
        size_t k = slot + 1;
        if (!routing_k_allowed(k) || k < floor_k) continue;
        float confidence = routing_boundary(probs, n, k);
        if (cumulative + eps >= mass_target && (float)k + eps >= support && confidence + eps >= minimum_gap)
            return k;
    }
    return n;
}

/* routing_policy.cpp:31-159 */
int k3xo_select_routing(const float* scores, const float* bias, size_t E, size_t K, int mode,
                        size_t fixed_k, float mass_target, float minimum_gap, size_t floor_k,
                        uint32_t* full_order, uint32_t* expert_ids, float* weights,
                        size_t* selected_k, float* stats, int* escalated)
{
    if (!E || !K || K > E) return K3XO_INVALID_STATE;
    for (size_t e = 0; e < E; ++e)
        if (!isfinite(scores[e]) || scores[e] < 0.0f || scores[e] > 1.0f || !isfinite(bias[e]))
            return K3XO_INVALID_STATE;
    if (!isfinite(mass_target) || mass_target <= 0.0f || mass_target > 1.0f || !isfinite(minimum_gap) ||
        minimum_gap < 0.0f || minimum_gap > 1.0f)
        return K3XO_INVALID_STATE;
    if (floor_k != 0 && (!routing_k_allowed(floor_k) || (mode != 0 && floor_k > K))) return K3XO_INVALID_STATE;
    if (mode == 1 && (!routing_k_allowed(fixed_k) || fixed_k > K)) return K3XO_INVALID_STATE;
    if (mode == 2 && K != 16) return K3XO_INVALID_STATE;
    if (mode < 0 || mode > 2) return K3XO_INVALID_STATE;
    float* adjusted = (float*)malloc(E * sizeof(float));
    uint32_t* order = (uint32_t*)malloc(E * sizeof(uint32_t));
    float* probs = (float*)malloc(K * sizeof(float));
    int status = K3XO_OK;
    for (size_t e = 0; e < E; ++e) {
        adjusted[e] = scores[e] + bias[e];
        if (!isfinite(adjusted[e])) status = K3XO_INVALID_STATE;
    }
    if (status == K3XO_OK) {
        /* stable order: adjusted descending, index ascending on ties */
        for (size_t e = 0; e < E; ++e) {
            size_t pos = e;
            order[e] = (uint32_t)e;
            while (pos > 0 && adjusted[order[pos - 1]] < adjusted[e]) {
                order[pos] = order[pos - 1];
                --pos;
            }
            order[pos] = (uint32_t)e;
        }
        float denom = 0.0f;
        for (size_t slot = 0; slot < K; ++slot) denom += scores[order[slot]];
        if (!isfinite(denom) || denom <= 0.0f) status = K3XO_INVALID_STATE;
    }
    if (status == K3XO_OK) {
        float denom = 0.0f;
        for (size_t slot = 0; slot < K; ++slot) denom += scores[order[slot]];
        float entropy = 0.0f;
        for (size_t slot = 0; slot < K; ++slot) {
            probs[slot] = scores[order[slot]] / denom;
            if (probs[slot] > 0.0f) entropy -= probs[slot] * logf(probs[slot]);
        }
        float support = expf(entropy);
        size_t chosen = K, unfloored = K;
        if (mode == 1) {
            unfloored = fixed_k;
            chosen = fixed_k > floor_k ? fixed_k : floor_k;
        } else if (mode == 2) {
            unfloored = routing_adaptive_k(probs, K, support, mass_target, minimum_gap, 0);
            chosen = routing_adaptive_k(probs, K, support, mass_target, minimum_gap, floor_k);
        }
        float mass = 0.0f, sel = 0.0f;
        for (size_t slot = 0; slot < chosen; ++slot) {
            mass += probs[slot];
            sel += scores[order[slot]];
        }
        if (!isfinite(sel) || sel <= 0.0f) {
            status = K3XO_INVALID_STATE;
        } else {
            for (size_t slot = 0; slot < chosen; ++slot) {
                expert_ids[slot] = order[slot];
                weights[slot] = scores[order[slot]] / sel;
            }
            *selected_k = chosen;
            stats[0] = K == 1 ? 0.0f : entropy / logf((float)K);
            stats[1] = support;
            stats[2] = mass;
            stats[3] = routing_boundary(probs, K, chosen);
            *escalated = chosen > unfloored;
            if (full_order) memcpy(full_order, order, E * sizeof(uint32_t));
        }
    }
    free(adjusted);
    free(order);
    free(probs);
    return status;
}

/* expert_major.cpp:10-54 */
int k3xo_expert_major_plan(const uint32_t* ids, const float* contributions,
                           size_t tokens, size_t top_k,
                           uint32_t* group_expert, uint32_t* group_offset,
                           uint32_t* assign_token, uint32_t* assign_slot,
                           float* assign_contrib, size_t* group_count)
{
    if (!tokens || !top_k) return K3XO_INVALID_EXTENT;
    size_t n = tokens * top_k;
    for (size_t t = 0; t < tokens; ++t) {
        for (size_t s = 0; s < top_k; ++s) {
            if (!isfinite(contributions[t * top_k + s])) return K3XO_INVALID_STATE;
            for (size_t j = 0; j < s; ++j)
                if (ids[t * top_k + j] == ids[t * top_k + s]) return K3XO_INVALID_STATE;
        }
    }
    /* first-use order of experts */
    size_t groups = 0;
    uint32_t* first = (uint32_t*)malloc(n * sizeof(uint32_t));
    for (size_t f = 0; f < n; ++f) {
        size_t g = 0;
        while (g < groups && group_expert[g] != ids[f]) ++g;
        if (g == groups) group_expert[groups++] = ids[f];
        first[f] = (uint32_t)g;
    }
    size_t pos = 0;
    for (size_t g = 0; g < groups; ++g) {
        group_offset[g] = (uint32_t)pos;
        for (size_t f = 0; f < n; ++f) {
            if (first[f] != g) continue;
            assign_token[pos] = (uint32_t)(f / top_k);
            assign_slot[pos] = (uint32_t)(f % top_k);
            assign_contrib[pos] = contributions[f];
            ++pos;
        }
    }
    group_offset[groups] = (uint32_t)pos;
    *group_count = groups;
    free(first);
    return K3XO_OK;
}

/* ------------------------------------------------------------------------ */
/* expert FFN (b) and combine (c)                                            */
/* ------------------------------------------------------------------------ */

/* official_moe.cpp:82-103 */
int k3xo_expert_ffn(const float* x, k3xo_mxfp4 gate, k3xo_mxfp4 up,
                    k3xo_mxfp4 down, size_t hidden, size_t inter,
                    int activation, float beta, float linear_beta, float* y)
{
    float* g = (float*)malloc(inter * sizeof(float));
    float* u = (float*)malloc(inter * sizeof(float));
    float* a = (float*)malloc(inter * sizeof(float));
    int st = k3xo_mxfp4_matmul(x, gate.packed, gate.scales, inter, hidden, 32, g);
    if (st == K3XO_OK) st = k3xo_mxfp4_matmul(x, up.packed, up.scales, inter, hidden, 32, u);
    if (st == K3XO_OK) {
        activate(a, g, u, inter, activation, beta, linear_beta);
        st = k3xo_mxfp4_matmul(a, down.packed, down.scales, hidden, inter, 32, y);
    }
    if (st == K3XO_OK)
        for (size_t i = 0; i < hidden; ++i) y[i] = k3xo_round_bf16(y[i]);
    free(g);
    free(u);
    free(a);
    return st;
}

/* official_moe.cpp:313-322 */
void k3xo_routed_combine(const float* y, const float* contributions,
                         size_t top_k, size_t hidden, float* mixed)
{
    for (size_t i = 0; i < hidden; ++i) mixed[i] = 0.0f;
    for (size_t slot = 0; slot < top_k; ++slot)
        for (size_t i = 0; i < hidden; ++i) {
            float p = contributions[slot] * y[slot * hidden + i];
            mixed[i] = mixed[i] + p;
        }
    for (size_t i = 0; i < hidden; ++i) mixed[i] = k3xo_round_bf16(mixed[i]);
}

/* official_moe.cpp:105-117 */
int k3xo_shared_ffn(const float* x, const uint16_t* gate, const uint16_t* up,
                    const uint16_t* down, size_t hidden, size_t inter,
                    int activation, float beta, float linear_beta, float* y)
{
    float* g = (float*)malloc(inter * sizeof(float));
    float* u = (float*)malloc(inter * sizeof(float));
    float* a = (float*)malloc(inter * sizeof(float));
    int st = k3xo_bf16_matvec(x, gate, inter, hidden, g);
    if (st == K3XO_OK) st = k3xo_bf16_matvec(x, up, inter, hidden, u);
    if (st == K3XO_OK) {
        activate(a, g, u, inter, activation, beta, linear_beta);
        st = k3xo_bf16_matvec(a, down, hidden, inter, y);
    }
    free(g);
    free(u);
    free(a);
    return st;
}

int k3xo_moe_layer_forward(const k3xo_moe_layer* L, const float* hidden,
                           size_t tokens, float* out, uint32_t* ids,
                           float* contributions)
{
    const size_t H = L->hidden, I = L->inter, E = L->experts, K = L->top_k;
    const size_t D = L->latent ? L->latent : H;   /* the experts' width */
    float* logits = (float*)malloc(E * sizeof(float));
    float* y = (float*)malloc(K * D * sizeof(float));
    float* mixed = (float*)malloc(D * sizeof(float));
    float* shared = (float*)malloc(H * sizeof(float));
    float* lat = (float*)malloc(D * sizeof(float));
    float* normed = (float*)malloc(D * sizeof(float));
    float* routed = (float*)malloc(H * sizeof(float));
    int st = K3XO_OK;
    for (size_t t = 0; t < tokens && st == K3XO_OK; ++t) {
        const float* x = hidden + t * H;
        const float* xe = x;
        st = k3xo_router_logits(x, L->router, E, H, logits);
        if (st == K3XO_OK)
            st = k3xo_route_logits(logits, L->correction, E, K, ids + t * K,
                                   contributions + t * K, NULL);
        if (st == K3XO_OK && L->latent) {   /* official_moe.cpp:296 */
            st = k3xo_bf16_matvec(x, L->routed_down, D, H, lat);
            xe = lat;
        }
        for (size_t s = 0; s < K && st == K3XO_OK; ++s) {
            size_t e = ids[t * K + s];
            k3xo_mxfp4 g = {L->gate_packed + e * I * D / 2, L->gate_scales + e * I * D / 32};
            k3xo_mxfp4 u = {L->up_packed + e * I * D / 2, L->up_scales + e * I * D / 32};
            k3xo_mxfp4 d = {L->down_packed + e * D * I / 2, L->down_scales + e * D * I / 32};
            st = k3xo_expert_ffn(xe, g, u, d, D, I, L->activation, L->situ_beta,
                                 L->situ_linear_beta, y + s * D);
        }
        if (st != K3XO_OK) break;
        k3xo_routed_combine(y, contributions + t * K, K, D, mixed);
        if (L->latent) {   /* :323-331: normalized(mixed, routed_norm), routed_up */
            st = k3xo_rms_norm_bf16(mixed, L->routed_norm, D, L->latent_eps, normed);
            if (st == K3XO_OK) st = k3xo_bf16_matvec(normed, L->routed_up, H, D, routed);
            if (st != K3XO_OK) break;
        } else {
            for (size_t i = 0; i < H; ++i) routed[i] = mixed[i];
        }
        if (L->shared_gate) {
            st = k3xo_shared_ffn(x, L->shared_gate, L->shared_up, L->shared_down, H,
                                 L->shared_inter, L->activation, L->situ_beta,
                                 L->situ_linear_beta, shared);
        } else {
            for (size_t i = 0; i < H; ++i) shared[i] = 0.0f;
        }
        /* official_moe.cpp:336: combined = round_bf16(routed + shared) */
        for (size_t i = 0; i < H; ++i) out[t * H + i] = k3xo_round_bf16(routed[i] + shared[i]);
    }
    free(logits);
    free(y);
    free(mixed);
    free(shared);
    free(lat);
    free(normed);
    free(routed);
    return st;
}

/* ------------------------------------------------------------------------ */
/* KDA (d)                                                                   */
/* ------------------------------------------------------------------------ */

/* official_kda.cpp:324-368 (body of the token loop) */
int k3xo_kda_step(float* state, const float* q, const float* k,
                  const float* v, const float* log_decay, const float* beta,
                  size_t heads, size_t d, float* out)
{
    float* decayed = (float*)malloc(d * d * sizeof(float));
    float* prediction = (float*)malloc(d * sizeof(float));
    float* delta = (float*)malloc(d * sizeof(float));
    int st = K3XO_OK;
    for (size_t h = 0; h < heads && st == K3XO_OK; ++h) {
        const size_t vb = h * d;
        float* S = state + h * d * d;
        for (size_t i = 0; i < d; ++i) prediction[i] = 0.0f;
        for (size_t key = 0; key < d; ++key) {
            float alpha = expf(log_decay[vb + key]);
            for (size_t value = 0; value < d; ++value) {
                float dv = alpha * S[value * d + key];
                decayed[key * d + value] = dv;
                prediction[value] += k[vb + key] * dv;
            }
        }
        for (size_t value = 0; value < d; ++value)
            delta[value] = (v[vb + value] - prediction[value]) * beta[h];
        for (size_t key = 0; key < d; ++key)
            for (size_t value = 0; value < d; ++value) {
                float updated = decayed[key * d + value] + k[vb + key] * delta[value];
                if (!isfinite(updated)) st = K3XO_INVALID_EXTENT;
                S[value * d + key] = updated;
            }
        for (size_t value = 0; value < d; ++value) {
            float o = 0.0f;
            for (size_t key = 0; key < d; ++key) o += q[vb + key] * S[value * d + key];
            out[vb + value] = o;
        }
    }
    free(decayed);
    free(prediction);
    free(delta);
    return st;
}

int k3xo_kda_tree(const float* prefix_state, const int32_t* parent,
                  size_t nodes, const float* q, const float* k,
                  const float* v, const float* log_decay, const float* beta,
                  size_t heads, size_t d, float* out, float* node_states)
{
    const size_t hd = heads * d, ss = heads * d * d;
    for (size_t n = 0; n < nodes; ++n)
        if (parent[n] < -1 || parent[n] >= (int32_t)n) return K3XO_INVALID_EXTENT;
    float* states = node_states ? node_states : (float*)malloc(nodes * ss * sizeof(float));
    int st = K3XO_OK;
    for (size_t n = 0; n < nodes && st == K3XO_OK; ++n) {
        const float* src = parent[n] < 0 ? prefix_state : states + (size_t)parent[n] * ss;
        memcpy(states + n * ss, src, ss * sizeof(float));
        st = k3xo_kda_step(states + n * ss, q + n * hd, k + n * hd, v + n * hd,
                           log_decay + n * hd, beta + n * heads, heads, d, out + n * hd);
    }
    if (!node_states) free(states);
    return st;
}

/* official_kda.cpp:58-88 */
static void matmul_sequence(const float* in, size_t seq, size_t width,
                            const uint16_t* w, size_t rows, float* out)
{
    for (size_t t = 0; t < seq; ++t)
        for (size_t r = 0; r < rows; ++r) {
            double sum = 0.0;
            for (size_t c = 0; c < width; ++c)
                sum += (double)in[t * width + c] * k3xo_decode_bf16(w[r * width + c]);
            out[t * rows + r] = k3xo_round_bf16((float)sum);
        }
}

/* official_kda.cpp:95-143 */
static void short_conv(const float* projected, uint16_t* state,
                       const float* weight, size_t seq, size_t proj,
                       size_t width, float* out)
{
    for (size_t t = 0; t < seq; ++t) {
        for (size_t c = 0; c < proj; ++c) {
            float sum = 0.0f;
            for (size_t h = 0; h + 1 < width; ++h)
                sum += k3xo_decode_bf16(state[h * proj + c]) * weight[c * width + h];
            sum += projected[t * proj + c] * weight[c * width + width - 1];
            float activated = sum / (1.0f + expf(-sum));
            out[t * proj + c] = k3xo_round_bf16(activated);
        }
        for (size_t h = 0; h + 2 < width; ++h)
            for (size_t c = 0; c < proj; ++c) state[h * proj + c] = state[(h + 1) * proj + c];
        for (size_t c = 0; c < proj; ++c)
            state[(width - 2) * proj + c] = k3xo_encode_bf16(projected[t * proj + c]);
    }
}

/* official_kda.cpp:198-426 */
int k3xo_kda_block(const k3xo_kda_weights* w, const float* hidden,
                   size_t T, uint16_t* conv_q, uint16_t* conv_k,
                   uint16_t* conv_v, float* recurrent, float* out)
{
    const size_t H = w->hidden, h = w->heads, d = w->head_dim, P = h * d;
    if (!T || !all_finite(hidden, T * H)) return K3XO_INVALID_EXTENT;
    float* x = (float*)malloc(T * H * sizeof(float));
    for (size_t i = 0; i < T * H; ++i) x[i] = k3xo_round_bf16(hidden[i]);
    float* pq = (float*)malloc(T * P * sizeof(float));
    float* pk = (float*)malloc(T * P * sizeof(float));
    float* pv = (float*)malloc(T * P * sizeof(float));
    float* fl = (float*)malloc(T * d * sizeof(float));
    float* bp = (float*)malloc(T * h * sizeof(float));
    float* og = (float*)malloc(T * P * sizeof(float));
    float* fg = (float*)malloc(T * P * sizeof(float));
    float* cq = (float*)malloc(T * P * sizeof(float));
    float* ck = (float*)malloc(T * P * sizeof(float));
    float* cv = (float*)malloc(T * P * sizeof(float));
    float* qn = (float*)malloc(T * P * sizeof(float));
    float* kn = (float*)malloc(T * P * sizeof(float));
    float* ld = (float*)malloc(T * P * sizeof(float));
    float* be = (float*)malloc(T * h * sizeof(float));
    float* ro = (float*)malloc(T * P * sizeof(float));
    float* gt = (float*)malloc(T * P * sizeof(float));
    int st = K3XO_OK;
    matmul_sequence(x, T, H, w->q_proj, P, pq);
    matmul_sequence(x, T, H, w->k_proj, P, pk);
    matmul_sequence(x, T, H, w->v_proj, P, pv);
    matmul_sequence(x, T, H, w->f_a_proj, d, fl);
    matmul_sequence(x, T, H, w->b_proj, h, bp);
    matmul_sequence(x, T, H, w->g_proj, P, og);
    matmul_sequence(fl, T, d, w->f_b_proj, P, fg);
    short_conv(pq, conv_q, w->q_conv, T, P, w->conv_width, cq);
    short_conv(pk, conv_k, w->k_conv, T, P, w->conv_width, ck);
    short_conv(pv, conv_v, w->v_conv, T, P, w->conv_width, cv);
    /* :259-290 */
    const float q_scale = 1.0f / sqrtf((float)d);
    for (size_t t = 0; t < T; ++t)
        for (size_t hh = 0; hh < h; ++hh) {
            size_t base = t * P + hh * d;
            float qs = 0.0f, ks = 0.0f;
            for (size_t c = 0; c < d; ++c) {
                qs += cq[base + c] * cq[base + c];
                ks += ck[base + c] * ck[base + c];
            }
            float qn_ = sqrtf(qs), kn_ = sqrtf(ks);
            float qi = 1.0f / (qn_ > 1.0e-12f ? qn_ : 1.0e-12f);
            float ki = 1.0f / (kn_ > 1.0e-12f ? kn_ : 1.0e-12f);
            for (size_t c = 0; c < d; ++c) {
                qn[base + c] = k3xo_round_bf16(cq[base + c] * qi * q_scale);
                kn[base + c] = k3xo_round_bf16(ck[base + c] * ki);
            }
        }
    /* :292-309 */
    for (size_t t = 0; t < T; ++t)
        for (size_t hh = 0; hh < h; ++hh)
            for (size_t c = 0; c < d; ++c) {
                size_t i = t * P + hh * d + c;
                float arg = expf(w->a_log[c]) * (fg[i] + w->dt_bias[hh * d + c]);
                ld[i] = w->gate_lower_bound / (1.0f + expf(-arg));
            }
    /* :310-314 */
    for (size_t i = 0; i < T * h; ++i) be[i] = 1.0f / (1.0f + expf(-bp[i]));
    /* :319-369 */
    for (size_t t = 0; t < T && st == K3XO_OK; ++t)
        st = k3xo_kda_step(recurrent, qn + t * P, kn + t * P, cv + t * P, ld + t * P,
                           be + t * h, h, d, ro + t * P);
    /* :371-395 */
    for (size_t t = 0; t < T; ++t)
        for (size_t hh = 0; hh < h; ++hh) {
            size_t base = t * P + hh * d;
            float squares = 0.0f;
            for (size_t c = 0; c < d; ++c) squares += ro[base + c] * ro[base + c];
            float inverse = 1.0f / sqrtf(squares / (float)d + w->eps);
            for (size_t c = 0; c < d; ++c) {
                float gate = 1.0f / (1.0f + expf(-og[base + c]));
                gt[base + c] = k3xo_round_bf16(ro[base + c] * inverse * w->o_norm[c] * gate);
            }
        }
    /* :396-397 */
    matmul_sequence(gt, T, P, w->o_proj, H, out);
    free(x); free(pq); free(pk); free(pv); free(fl); free(bp); free(og); free(fg);
    free(cq); free(ck); free(cv); free(qn); free(kn); free(ld); free(be); free(ro);
    free(gt);
    return st;
}

/* ------------------------------------------------------------------------ */
/* acceptance (e)                                                            */
/* ------------------------------------------------------------------------ */

/* model.cpp:1174-1176 (std::max_element: first maximum) */
uint32_t k3xo_argmax(const float* logits, size_t vocab)
{
    size_t best = 0;
    for (size_t i = 1; i < vocab; ++i)
        if (logits[best] < logits[i]) best = i;
    return (uint32_t)best;
}

/* speculative.cpp:74-112 */
int k3xo_verify_greedy_block(uint32_t anchor, const uint32_t* drafts,
                             size_t p, size_t max_draft, size_t vocab,
                             const uint32_t* targets, size_t* accepted,
                             uint32_t* committed, size_t* ncommitted,
                             int* all_accepted)
{
    if (vocab == 0 || anchor >= vocab || p > max_draft) return K3XO_INVALID_EXTENT;
    for (size_t i = 0; i < p; ++i)
        if (drafts[i] >= vocab) return K3XO_INVALID_EXTENT;
    for (size_t i = 0; i <= p; ++i)
        if (targets[i] >= vocab) return K3XO_INVALID_STATE;
    *accepted = 0;
    *ncommitted = 0;
    *all_accepted = 0;
    for (size_t i = 0; i < p; ++i) {
        if (drafts[i] != targets[i]) {
            committed[(*ncommitted)++] = targets[i];
            return K3XO_OK;
        }
        committed[(*ncommitted)++] = drafts[i];
        ++*accepted;
    }
    committed[(*ncommitted)++] = targets[p];
    *all_accepted = 1;
    return K3XO_OK;
}

/* SplitMix64 finaliser (Steele, Lea, Flood, OOPSLA 2014). */
static uint64_t splitmix64(uint64_t z)
{
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

double k3xo_uniform(uint64_t seed, uint64_t sequence, uint64_t position,
                    uint64_t purpose)
{
    uint64_t key = splitmix64(seed);
    key = splitmix64(key ^ sequence);
    key = splitmix64(key ^ position);
    key = splitmix64(key ^ purpose);
    return (double)(key >> 11) * 0x1.0p-53;
}

/*
 * Canonical reduction order for a length-V vector w (shared with the CUDA
 * acceptance kernels so that decisions agree bit for bit):
 *   1024 chunks of L = ceil(V/1024) consecutive entries (tail chunks may be
 *   short or empty); chunk sums are sequential from 0.0; 32 group sums, each
 *   the sequential sum of 32 consecutive chunk sums; the total is the
 *   sequential sum of the 32 group sums. Sampling looks for the first group
 *   whose running total exceeds the target, then the first chunk inside it
 *   (running from the previous groups' running total), then the first entry
 *   inside that chunk; at each level, if rounding leaves no crossing, the
 *   last candidate with positive weight is taken.
 */
#define RS_CHUNKS 1024
#define RS_GROUPS 32

typedef struct {
    double chunk[RS_CHUNKS];
    double group[RS_GROUPS];
    double total;
    size_t len;
} rs_sums;

static void rs_reduce(const double* w, size_t V, rs_sums* s)
{
    s->len = (V + RS_CHUNKS - 1) / RS_CHUNKS;
    for (size_t c = 0; c < RS_CHUNKS; ++c) {
        double acc = 0.0;
        size_t lo = c * s->len, hi = lo + s->len;
        if (hi > V) hi = V;
        for (size_t j = lo; j < hi; ++j) acc += w[j];
        s->chunk[c] = acc;
    }
    for (size_t g = 0; g < RS_GROUPS; ++g) {
        double acc = 0.0;
        for (size_t c = 0; c < RS_CHUNKS / RS_GROUPS; ++c) acc += s->chunk[g * 32 + c];
        s->group[g] = acc;
    }
    double acc = 0.0;
    for (size_t g = 0; g < RS_GROUPS; ++g) acc += s->group[g];
    s->total = acc;
}

static uint32_t rs_sample(const double* w, size_t V, const rs_sums* s, double target)
{
    double run = 0.0;
    size_t g_sel = RS_GROUPS, g_last = 0;
    for (size_t g = 0; g < RS_GROUPS; ++g) {
        if (s->group[g] > 0.0) g_last = g;
        double next = run + s->group[g];
        if (next > target) { g_sel = g; break; }
        run = next;
    }
    if (g_sel == RS_GROUPS) {
        g_sel = g_last;
        run = 0.0;
        for (size_t g = 0; g < g_sel; ++g) run += s->group[g];
    }
    size_t c_sel = RS_CHUNKS, c_last = g_sel * 32;
    for (size_t c = g_sel * 32; c < g_sel * 32 + 32; ++c) {
        if (s->chunk[c] > 0.0) c_last = c;
        double next = run + s->chunk[c];
        if (next > target) { c_sel = c; break; }
        run = next;
    }
    if (c_sel == RS_CHUNKS) {
        c_sel = c_last;
        run = 0.0;
        for (size_t g = 0; g < g_sel; ++g) run += s->group[g];
        for (size_t c = g_sel * 32; c < c_sel; ++c) run += s->chunk[c];
    }
    size_t lo = c_sel * s->len, hi = lo + s->len;
    if (hi > V) hi = V;
    size_t j_last = lo;
    for (size_t j = lo; j < hi; ++j) {
        if (w[j] > 0.0) j_last = j;
        double next = run + w[j];
        if (next > target) return (uint32_t)j;
        run = next;
    }
    return (uint32_t)j_last;
}

static float row_max(const float* l, size_t V)
{
    float m = l[0];
    for (size_t j = 1; j < V; ++j)
        if (l[j] > m) m = l[j];
    return m;
}

/* w[j] = exp((l[j] - max) / tau) in double */
static void softmax_weights(const float* l, size_t V, double tau, double* w)
{
    double m = row_max(l, V);
    for (size_t j = 0; j < V; ++j) w[j] = exp(((double)l[j] - m) / tau);
}

int k3xo_verify_rejection(const float* target_logits,
                          const float* draft_logits, const uint32_t* drafts,
                          size_t p, size_t V, float temperature,
                          uint64_t seed, uint64_t sequence, size_t* accepted,
                          uint32_t* committed, size_t* ncommitted)
{
    if (!V || !(temperature > 0.0f)) return K3XO_INVALID_EXTENT;
    for (size_t i = 0; i < p; ++i)
        if (drafts[i] >= V) return K3XO_INVALID_EXTENT;
    const double tau = temperature;
    double* wp = (double*)malloc(V * sizeof(double));
    double* wq = (double*)malloc(V * sizeof(double));
    rs_sums* sp = (rs_sums*)malloc(sizeof(rs_sums));
    rs_sums* sq = (rs_sums*)malloc(sizeof(rs_sums));
    *accepted = 0;
    *ncommitted = 0;
    size_t i = 0;
    for (; i < p; ++i) {
        softmax_weights(target_logits + i * V, V, tau, wp);
        softmax_weights(draft_logits + i * V, V, tau, wq);
        rs_reduce(wp, V, sp);
        rs_reduce(wq, V, sq);
        double pd = wp[drafts[i]] / sp->total;
        double qd = wq[drafts[i]] / sq->total;
        double u = k3xo_uniform(seed, sequence, i, 0);
        if (u * qd < pd) {
            committed[(*ncommitted)++] = drafts[i];
            ++*accepted;
            continue;
        }
        /* rejected: sample from norm(max(0, p - q)) */
        double* r = (double*)malloc(V * sizeof(double));
        for (size_t j = 0; j < V; ++j) {
            double diff = wp[j] / sp->total - wq[j] / sq->total;
            r[j] = diff > 0.0 ? diff : 0.0;
        }
        rs_sums* sr = (rs_sums*)malloc(sizeof(rs_sums));
        rs_reduce(r, V, sr);
        double u2 = k3xo_uniform(seed, sequence, i, 1);
        uint32_t tok = sr->total > 0.0 ? rs_sample(r, V, sr, u2 * sr->total)
                                       : rs_sample(wp, V, sp, u2 * sp->total);
        committed[(*ncommitted)++] = tok;
        free(r);
        free(sr);
        break;
    }
    if (i == p) {
        softmax_weights(target_logits + p * V, V, tau, wp);
        rs_reduce(wp, V, sp);
        double u2 = k3xo_uniform(seed, sequence, p, 1);
        committed[(*ncommitted)++] = rs_sample(wp, V, sp, u2 * sp->total);
    }
    free(wp);
    free(wq);
    free(sp);
    free(sq);
    return K3XO_OK;
}

/* ------------------------------------------------------------------------ */
/* seeded synthetic workloads: the library's generator (csrc/synth.cu)       */
/* ------------------------------------------------------------------------ */

static uint64_t mix64(uint64_t z)
{
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

/* ln(k * 2^-24), k in [1, 2^24]: k = m * 2^e, m in [sqrt(1/2), sqrt(2)),
 * ln m = 2 atanh((m - 1) / (m + 1)) by its series to s^11. */
static float synth_log(uint32_t k)
{
    int e = 31;
    while (!(k >> e)) --e;
    const uint32_t mant = e <= 23 ? k << (23 - e) : k >> (e - 23);
    float m = u2f((mant & 0x7fffffu) | 0x3f800000u);
    if (m > 0x1.6a09e6p+0f) {
        m = m * 0.5f;
        ++e;
    }
    const float s = (m + -1.0f) / (m + 1.0f);
    const float s2 = s * s;
    float p = 0x1.745d18p-4f;
    p = p * s2 + 0x1.c71c72p-4f;
    p = p * s2 + 0x1.24924ap-3f;
    p = p * s2 + 0x1.99999ap-3f;
    p = p * s2 + 0x1.555556p-2f;
    p = p * s2 + 1.0f;
    const float lnm = (2.0f * s) * p;
    return (float)(e - 24) * 0x1.62e430p-1f + lnm;
}

/* cos and sin of 2*pi*k*2^-24, k in [0, 2^24): quadrant from the top two
 * bits, Taylor series to x^14 / x^15 on [0, pi/2). */
static void synth_cos_sin(uint32_t k, float* c_out, float* s_out)
{
    const uint32_t q = k >> 22;
    const float f = (float)(k & 0x3fffffu) * 0x1.0p-24f;
    const float x = f * 0x1.921fb6p+2f, x2 = x * x;
    float c = -0x1.93974cp-37f, sn = -0x1.ae7f3ep-41f;
    c = c * x2 + 0x1.1eed8ep-29f;
    c = c * x2 + -0x1.27e4fcp-22f;
    c = c * x2 + 0x1.a01a02p-16f;
    c = c * x2 + -0x1.6c16c2p-10f;
    c = c * x2 + 0x1.555556p-5f;
    c = c * x2 + -0.5f;
    c = c * x2 + 1.0f;
    sn = sn * x2 + 0x1.612462p-33f;
    sn = sn * x2 + -0x1.ae6456p-26f;
    sn = sn * x2 + 0x1.71de3ap-19f;
    sn = sn * x2 + -0x1.a01a02p-13f;
    sn = sn * x2 + 0x1.111112p-7f;
    sn = sn * x2 + -0x1.555556p-3f;
    sn = (sn * x2) * x + x;
    switch (q) {
    case 0: *c_out = c; *s_out = sn; break;
    case 1: *c_out = -sn; *s_out = c; break;
    case 2: *c_out = -c; *s_out = -sn; break;
    default: *c_out = sn; *s_out = -c; break;
    }
}

void k3xo_normal_pair(uint64_t seed, uint64_t stream, uint64_t pair, float* z0, float* z1)
{
    const uint64_t r = mix64(mix64(mix64(seed) ^ stream) ^ pair);
    const uint32_t k1 = (uint32_t)(r >> 40) + 1u;
    const uint32_t k2 = (uint32_t)((r >> 16) & 0xffffffu);
    const float rad = sqrtf(-2.0f * synth_log(k1));
    float c, s;
    synth_cos_sin(k2, &c, &s);
    *z0 = rad * c;
    *z1 = rad * s;
}

static float synth_normal(uint64_t seed, uint64_t stream, uint64_t element)
{
    float z0, z1;
    k3xo_normal_pair(seed, stream, element >> 1, &z0, &z1);
    return (element & 1u) ? z1 : z0;
}

void k3xo_fill_normal_f32(float* out, size_t n, uint64_t first, uint64_t seed, uint64_t stream,
                          float mean, float sigma)
{
    for (size_t j = 0; j < n; ++j) out[j] = mean + sigma * synth_normal(seed, stream, first + j);
}

void k3xo_fill_normal_bf16(uint16_t* out, size_t n, uint64_t first, uint64_t seed, uint64_t stream,
                           float sigma)
{
    for (size_t j = 0; j < n; ++j) out[j] = k3xo_encode_bf16(sigma * synth_normal(seed, stream, first + j));
}

void k3xo_fill_normal_mxfp4(uint8_t* packed, uint8_t* scales, size_t blocks, uint64_t first,
                            uint64_t seed, uint64_t stream, float sigma)
{
    float v[32];
    for (size_t b = 0; b < blocks; ++b) {
        for (int i = 0; i < 16; ++i) {
            float z0, z1;
            k3xo_normal_pair(seed, stream, (first + b) * 16 + (uint64_t)i, &z0, &z1);
            v[2 * i] = sigma * z0;
            v[2 * i + 1] = sigma * z1;
        }
        k3xo_quantize_mxfp4(v, 1, 32, packed + b * 16, scales + b);
    }
}

/* ------------------------------------------------------------------------ */
/* gated MLA (model.cpp:755-811) and KV crop (model.cpp:1235-1251)           */
/* ------------------------------------------------------------------------ */

static float mla_sigmoid(float v) { return 1.0f / (1.0f + expf(-v)); }   /* model.cpp:60 */

/* model.cpp:758-772: one position's query [heads][q_main + q_extra], its
 * key [heads][q_main], value [heads][value_dim] and shared key [q_extra]. */
static int mla_project(const k3xo_mla_weights* w, const float* x, float* query, float* key,
                       float* value, float* shared_key)
{
    const size_t H = w->hidden, nh = w->heads, qm = w->q_main, qe = w->q_extra, vd = w->value_dim;
    float* q_latent = (float*)malloc(w->q_rank * sizeof(float));
    float* q_normed = (float*)malloc(w->q_rank * sizeof(float));
    float* compressed = (float*)malloc((w->kv_rank + qe) * sizeof(float));
    float* latent = (float*)malloc(w->kv_rank * sizeof(float));
    float* expanded = (float*)malloc(nh * (qm + vd) * sizeof(float));
    int st = K3XO_INVALID_EXTENT;
    if (q_latent && q_normed && compressed && latent && expanded) {
        k3xo_dense_matvec(x, w->q_a_proj, w->q_rank, H, q_latent);
        k3xo_rms_norm_f32(q_latent, w->q_a_norm, w->q_rank, w->eps, q_normed);
        k3xo_dense_matvec(q_normed, w->q_b_proj, nh * (qm + qe), w->q_rank, query);
        k3xo_dense_matvec(x, w->kv_a_proj, w->kv_rank + qe, H, compressed);
        k3xo_rms_norm_f32(compressed, w->kv_a_norm, w->kv_rank, w->eps, latent);
        k3xo_dense_matvec(latent, w->kv_b_proj, nh * (qm + vd), w->kv_rank, expanded);
        memcpy(shared_key, compressed + w->kv_rank, qe * sizeof(float));
        for (size_t h = 0; h < nh; ++h) {
            memcpy(key + h * qm, expanded + h * (qm + vd), qm * sizeof(float));
            memcpy(value + h * vd, expanded + h * (qm + vd) + qm, vd * sizeof(float));
        }
        st = K3XO_OK;
    }
    free(q_latent);
    free(q_normed);
    free(compressed);
    free(latent);
    free(expanded);
    return st;
}

/* model.cpp:785-810: attention of one query over n positions in the given
 * order (position p's key rows kp[p] [heads][q_main], values vp[p]
 * [heads][value_dim], shared key sp[p] [q_extra]), FP64 sums of float
 * products, float softmax, the output gate and o_proj. */
static int mla_attend(const k3xo_mla_weights* w, const float* x, const float* query,
                      const float* const* kp, const float* const* vp, const float* const* sp,
                      size_t n, float* out)
{
    const size_t H = w->hidden, nh = w->heads, qm = w->q_main, qe = w->q_extra, vd = w->value_dim;
    const size_t qw = qm + qe;
    float* merged = (float*)calloc(nh * vd, sizeof(float));
    float* gate = (float*)malloc(nh * vd * sizeof(float));
    float* scores = (float*)malloc(n * sizeof(float));
    int st = K3XO_INVALID_EXTENT;
    if (merged && gate && scores && n) {
        const float scale = 1.0f / sqrtf((float)qw);
        for (size_t h = 0; h < nh; ++h) {
            for (size_t p = 0; p < n; ++p) {
                double score = 0.0;
                for (size_t i = 0; i < qm; ++i) score += query[h * qw + i] * kp[p][h * qm + i];
                for (size_t i = 0; i < qe; ++i) score += query[h * qw + qm + i] * sp[p][i];
                scores[p] = (float)score * scale;
            }
            float maximum = scores[0];
            for (size_t p = 1; p < n; ++p)
                if (scores[p] > maximum) maximum = scores[p];
            float denominator = 0.0f;
            for (size_t p = 0; p < n; ++p) {
                scores[p] = expf(scores[p] - maximum);
                denominator += scores[p];
            }
            for (size_t p = 0; p < n; ++p)
                for (size_t i = 0; i < vd; ++i)
                    merged[h * vd + i] += scores[p] / denominator * vp[p][h * vd + i];
        }
        k3xo_dense_matvec(x, w->g_proj, nh * vd, H, gate);
        for (size_t i = 0; i < nh * vd; ++i) merged[i] *= mla_sigmoid(gate[i]);
        k3xo_dense_matvec(merged, w->o_proj, H, nh * vd, out);
        st = K3XO_OK;
    }
    free(merged);
    free(gate);
    free(scores);
    return st;
}

int k3xo_mla_step(const k3xo_mla_weights* w, const float* x, float* keys, float* values,
                  float* shared, size_t capacity, size_t* length, float* out)
{
    if (!w || !x || !keys || !values || !shared || !length || !out || *length >= capacity)
        return K3XO_INVALID_EXTENT;
    const size_t nh = w->heads, qm = w->q_main, qe = w->q_extra, vd = w->value_dim;
    const size_t p0 = *length, n = p0 + 1;
    float* query = (float*)malloc(nh * (qm + qe) * sizeof(float));
    const float** kp = (const float**)malloc(n * sizeof(float*));
    const float** vp = (const float**)malloc(n * sizeof(float*));
    const float** sp = (const float**)malloc(n * sizeof(float*));
    int st = K3XO_INVALID_EXTENT;
    if (query && kp && vp && sp) {
        /* model.cpp:773-784: append this position, then attend over all */
        st = mla_project(w, x, query, keys + p0 * nh * qm, values + p0 * nh * vd, shared + p0 * qe);
        if (st == K3XO_OK) {
            *length = n;
            for (size_t p = 0; p < n; ++p) {
                kp[p] = keys + p * nh * qm;
                vp[p] = values + p * nh * vd;
                sp[p] = shared + p * qe;
            }
            st = mla_attend(w, x, query, kp, vp, sp, n, out);
        }
    }
    free(query);
    free(kp);
    free(vp);
    free(sp);
    return st;
}

int k3xo_mla_tree(const k3xo_mla_weights* w, const float* keys, const float* values,
                  const float* shared, size_t length, const int32_t* parent, size_t nodes,
                  const float* x, float* node_keys, float* node_values, float* node_shared,
                  float* out)
{
    if (!w || (length && (!keys || !values || !shared)) || !parent || !nodes || !x || !node_keys ||
        !node_values || !node_shared || !out)
        return K3XO_INVALID_EXTENT;
    for (size_t i = 0; i < nodes; ++i)
        if (parent[i] < -1 || parent[i] >= (int32_t)i) return K3XO_INVALID_EXTENT;
    const size_t H = w->hidden, nh = w->heads, qm = w->q_main, qe = w->q_extra, vd = w->value_dim;
    const size_t cap = length + nodes;
    float* query = (float*)malloc(nh * (qm + qe) * sizeof(float));
    size_t* path = (size_t*)malloc(nodes * sizeof(size_t));
    const float** kp = (const float**)malloc(cap * sizeof(float*));
    const float** vp = (const float**)malloc(cap * sizeof(float*));
    const float** sp = (const float**)malloc(cap * sizeof(float*));
    int st = (query && path && kp && vp && sp) ? K3XO_OK : K3XO_INVALID_EXTENT;
    for (size_t p = 0; st == K3XO_OK && p < length; ++p) {
        kp[p] = keys + p * nh * qm;
        vp[p] = values + p * nh * vd;
        sp[p] = shared + p * qe;
    }
    for (size_t i = 0; st == K3XO_OK && i < nodes; ++i) {
        st = mla_project(w, x + i * H, query, node_keys + i * nh * qm, node_values + i * nh * vd,
                         node_shared + i * qe);
        if (st != K3XO_OK) break;
        /* the committed positions, then the node's ancestors root first and
         * the node itself: on a chain, the order a sequential prefill sees */
        size_t depth = 0;
        for (int32_t a = (int32_t)i; a >= 0; a = parent[a]) path[depth++] = (size_t)a;
        for (size_t k = 0; k < depth; ++k) {
            const size_t a = path[depth - 1 - k];
            kp[length + k] = node_keys + a * nh * qm;
            vp[length + k] = node_values + a * nh * vd;
            sp[length + k] = node_shared + a * qe;
        }
        st = mla_attend(w, x + i * H, query, kp, vp, sp, length + depth, out + i * H);
    }
    free(query);
    free(path);
    free(kp);
    free(vp);
    free(sp);
    return st;
}

int k3xo_mla_crop(size_t* length, size_t keep)
{
    if (!length || keep > *length) return K3XO_INVALID_EXTENT;
    *length = keep;
    return K3XO_OK;
}
