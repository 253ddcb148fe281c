/*
 * k3x_oracle.h — CPU restatement of the K3X speculative-verification path.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the shipped library links, loads or
 * calls this code: it is the checker that tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg compare the CUDA path against.
 *
 * Every function restates one reference function (file:line under the
 * rsb1813/project-k3x tree) or, where the reference has no counterpart
 * (MXFP4 quantizer, E2M1 term split, draft-tree recurrence, rejection
 * sampling), defines the algorithm that the CUDA kernels must reproduce.
 * The restatement is pinned against the reference's own compiled CPU code
 * (oracle/_ref, built by oracle/Makefile) and its golden literals in
 * tests/test_oracle_pin.py.
 */
#ifndef K3X_ORACLE_H
#define K3X_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status values mirror k3x::ErrorCode (runtime/include/k3x/status.hpp:9-30). */
enum {
    K3XO_OK = 0,
    K3XO_INVALID_EXTENT = 9,
    K3XO_INVALID_MXFP4 = 15,
    K3XO_INVALID_STATE = 16,
};

/* Activations used by the expert / shared FFN. */
enum { K3XO_ACT_SWIGLU = 0, K3XO_ACT_SITU = 1 };

/* ---- scalar numerics ---------------------------------------------------- */
float k3xo_round_bf16(float value);            /* official_moe.cpp:18-26 */
uint16_t k3xo_encode_bf16(float value);        /* official_kda.cpp:31-39 */
float k3xo_decode_bf16(uint16_t word);         /* official_moe.cpp:135-137 */
float k3xo_e2m1_value(uint8_t code);           /* ops.cpp:40-43 table */

/* ---- MXFP4 -------------------------------------------------------------- */
/* ops.cpp:32-55: decode packed [rows][cols/2] (low nibble = even column)
 * with E8M0 scales [rows][cols/group]; 0xFF scale -> INVALID_MXFP4. */
int k3xo_decode_mxfp4(const uint8_t* packed, const uint8_t* scales,
                      size_t rows, size_t cols, size_t group, float* out);
/* ops.cpp:57-76: y[r] = float(sum_c double(x[c]) * w[r][c]), sequential. */
int k3xo_mxfp4_matmul(const float* x, const uint8_t* packed,
                      const uint8_t* scales, size_t rows, size_t cols,
                      size_t group, float* out);
/* New (the reference only decodes): per 32-block scale s = smallest integer
 * with amax <= 6*2^s, codes = round-to-nearest-even onto the E2M1 grid. */
void k3xo_quantize_mxfp4(const float* x, size_t rows, size_t cols,
                         uint8_t* packed, uint8_t* scales);
/* The E2M1 rounding used by the quantizer (ties to the even code). */
uint8_t k3xo_e2m1_code(float magnitude);
/* Exact multi-term split used for the tensor-core activation operand:
 * x[0..31] = sum_t code_t * 2^(scale_t-127) + residual. Writes nterms*16
 * packed bytes and nterms scale bytes; returns max |residual|. */
float k3xo_e2m1_terms(const float* x32, int nterms, uint8_t* packed,
                      uint8_t* scales);

/* ---- elementwise / small ------------------------------------------------ */
/* ops.cpp:20-30 (linear_beta <= 0 means "no linear bound"). */
void k3xo_situ_glu(float* out, const float* gate, const float* up, size_t n,
                   float beta, float linear_beta);
/* SwiGLU = the beta -> infinity limit of situ_glu without a linear bound:
 * (g * sigmoid(g)) * u, all float. */
void k3xo_swiglu(float* out, const float* gate, const float* up, size_t n);
/* official_moe.cpp:39-59: FP64 accumulation, output rounded to bf16. */
int k3xo_dense_matvec(const float* x, const float* w, size_t rows, size_t cols,
                      float* out);   /* backend_cpu.cpp:23-47 */
int k3xo_bf16_matvec(const float* x, const uint16_t* w, size_t rows,
                     size_t cols, float* out);
/* official_moe.cpp:61-80 / official_layer.cpp:104-125 (bf16 weight). */
int k3xo_rms_norm_bf16(const float* x, const uint16_t* weight, size_t n,
                       float eps, float* out);
/* official_layer.cpp:42-102: two-source attention residual. */
int k3xo_attention_residual(const float* prefix, const float* block,
                            const uint16_t* norm, const uint16_t* proj,
                            size_t n, float eps, float* out);
/* ops.cpp:10-18: rms_norm with float weights (FP64 squares, float
 * inverse, (x * inverse) * weight). */
void k3xo_rms_norm_f32(const float* x, const float* weight, size_t n,
                       float eps, float* out);
/* model.cpp:645-666: block attention residual over S sources [S][T][H]
 * (depth-major) and the prefix [T][H]; float norm and projection [H]. */
int k3xo_block_attention_residual(const float* prefix, const float* sources,
                                  size_t S, size_t T, size_t H,
                                  const float* norm, const float* proj,
                                  float eps, float* out);

/* ---- router (a) --------------------------------------------------------- */
/* official_moe.cpp:255-267: logits[e] = float(sum_h double(bf16 W[e][h]) * x[h]). */
int k3xo_router_logits(const float* hidden, const uint16_t* w, size_t experts,
                       size_t hidden_size, float* logits);
/* official_moe.cpp:211-245: sigmoid, +correction, Top-k (adjusted desc,
 * index asc), contributions = score / double total. scores may be NULL. */
int k3xo_route_logits(const float* logits, const float* correction,
                      size_t experts, size_t top_k, uint32_t* ids,
                      float* contributions, float* scores);
/* select_routing (routing_policy.cpp:31-159): the synthetic engine's
 * routing policy over sigmoid scores in [0,1]. mode 0 natural (Top-k),
 * 1 fixed (fixed_k from the ladder {4,6,8,12,16}), 2 adaptive (natural
 * Top-16 cut at the first ladder K that reaches the mass target, covers the
 * entropy support and clears the boundary gap); quality_floor_k (0 = none)
 * raises the choice. Outputs: full_order [E] (may be NULL), expert_ids and
 * weights [selected_k] (room for natural_k), *selected_k, stats[4] =
 * {normalized entropy, entropy support, selected mass, boundary
 * confidence}, *escalated. Invalid input: K3XO_INVALID_STATE. */
int k3xo_select_routing(const float* scores, const float* bias, size_t experts,
                        size_t natural_k, int mode, size_t fixed_k,
                        float mass_target, float minimum_gap,
                        size_t quality_floor_k, uint32_t* full_order,
                        uint32_t* expert_ids, float* weights,
                        size_t* selected_k, float* stats, int* escalated);

/* expert_major.cpp:10-54: stable first-use grouping. Outputs:
 * group_expert[g], group_offset[g..g+1] into the assignment arrays,
 * assign_token/assign_slot/assign_contrib in (token, slot) order per group. */
int k3xo_expert_major_plan(const uint32_t* ids, const float* contributions,
                           size_t tokens, size_t top_k,
                           uint32_t* group_expert, uint32_t* group_offset,
                           uint32_t* assign_token, uint32_t* assign_slot,
                           float* assign_contrib, size_t* group_count);

/* ---- expert FFN (b) and combine (c) ------------------------------------- */
typedef struct {
    const uint8_t* packed;
    const uint8_t* scales;
} k3xo_mxfp4;

/* official_moe.cpp:82-103: y = round_bf16(W_d * act(W_g x, W_u x)). */
int k3xo_expert_ffn(const float* x, k3xo_mxfp4 gate, k3xo_mxfp4 up,
                    k3xo_mxfp4 down, size_t hidden, size_t inter,
                    int activation, float beta, float linear_beta, float* y);
/* official_moe.cpp:313-322: mixed = sum_slot c[slot]*y[slot] (float, slot
 * order), then round_bf16. */
void k3xo_routed_combine(const float* y, const float* contributions,
                         size_t top_k, size_t hidden, float* mixed);
/* official_moe.cpp:105-117: bf16 shared expert (each matvec rounded). */
int k3xo_shared_ffn(const float* x, const uint16_t* gate, const uint16_t* up,
                    const uint16_t* down, size_t hidden, size_t inter,
                    int activation, float beta, float linear_beta, float* y);

/* MoE layer of official_moe.cpp:271-344 after the input preparation: route
 * on the hidden row, experts, slot-ordered combine, shared expert,
 * out[t] = round_bf16(routed + shared) (the prefix residual, :337-341, is
 * the caller's). latent == 0: the plain hidden-space MoE (routed = mixed,
 * no :296 / :323-331). latent = L: LatentMoE — latent = bf16_matvec(hidden,
 * routed_down) (:296), experts on the latent row, mixed rounded (:322),
 * normalized by routed_norm with latent_eps (:323), routed =
 * bf16_matvec(normalized, routed_up) (:328). Experts are stacked over their
 * width D (H, or L): gate/up [E][inter][D/2], down [E][D][inter/2], scales
 * likewise with /32. shared_* may be NULL (no shared expert). ids/contrib
 * (T*k) receive the routes. */
typedef struct {
    size_t hidden, inter, experts, top_k, shared_inter;
    const uint16_t* router;       /* [E][H] bf16 */
    const float* correction;      /* [E] */
    const uint8_t* gate_packed;   /* [E][I][H/2] */
    const uint8_t* gate_scales;   /* [E][I][H/32] */
    const uint8_t* up_packed;
    const uint8_t* up_scales;
    const uint8_t* down_packed;   /* [E][H][I/2] */
    const uint8_t* down_scales;   /* [E][H][I/32] */
    const uint16_t* shared_gate;  /* [Is][H] */
    const uint16_t* shared_up;    /* [Is][H] */
    const uint16_t* shared_down;  /* [H][Is] */
    int activation;
    float situ_beta, situ_linear_beta;
    size_t latent;                /* 0: plain MoE */
    const uint16_t* routed_down;  /* [L][H] */
    const uint16_t* routed_norm;  /* [L] */
    const uint16_t* routed_up;    /* [H][L] */
    float latent_eps;
} k3xo_moe_layer;

int k3xo_moe_layer_forward(const k3xo_moe_layer* layer, const float* hidden,
                           size_t tokens, float* out, uint32_t* ids,
                           float* contributions);

/* ---- KDA (d) ------------------------------------------------------------ */
/* official_kda.cpp:319-369 for one token, all heads. state is V-first
 * [heads][d(value)][d(key)] float, updated in place. */
int k3xo_kda_step(float* state, const float* q, const float* k,
                  const float* v, const float* log_decay, const float* beta,
                  size_t heads, size_t head_dim, float* out);
/* Draft-tree verification (new): node n's state = step(parent's state),
 * parent[n] = -1 means the prefix state. parent[n] < n is required.
 * q/k/v/log_decay are [nodes][heads*d], beta [nodes][heads], out
 * [nodes][heads*d]. node_states (optional) receives every node's state. */
int k3xo_kda_tree(const float* prefix_state, const int32_t* parent,
                  size_t nodes, const float* q, const float* k,
                  const float* v, const float* log_decay, const float* beta,
                  size_t heads, size_t head_dim, float* out,
                  float* node_states);

/* Full official KDA block (official_kda.cpp:198-426). Weights bf16 words,
 * conv/a_log/dt_bias/o_norm float. State: conv_{q,k,v} [(w-1)][h*d] bf16
 * words, recurrent [h][d][d] float; all updated in place. */
typedef struct {
    size_t hidden, heads, head_dim, conv_width;
    float eps, gate_lower_bound;
    const uint16_t *q_proj, *k_proj, *v_proj;   /* [h*d][H] */
    const float *q_conv, *k_conv, *v_conv;      /* [h*d][w] */
    const uint16_t* f_a_proj;                   /* [d][H] */
    const uint16_t* f_b_proj;                   /* [h*d][d] */
    const float* a_log;                         /* [d] */
    const float* dt_bias;                       /* [h*d] */
    const uint16_t* b_proj;                     /* [h][H] */
    const uint16_t* g_proj;                     /* [h*d][H] */
    const float* o_norm;                        /* [d] */
    const uint16_t* o_proj;                     /* [H][h*d] */
} k3xo_kda_weights;

int k3xo_kda_block(const k3xo_kda_weights* w, const float* hidden,
                   size_t tokens, uint16_t* conv_q, uint16_t* conv_k,
                   uint16_t* conv_v, float* recurrent, float* out);

/* ---- acceptance (e) ----------------------------------------------------- */
/* model.cpp:1174-1176: first index of the maximum. */
uint32_t k3xo_argmax(const float* logits, size_t vocab);
/* speculative.cpp:74-112 (verify_greedy_target_block). committed must hold
 * drafts+1 entries. */
int k3xo_verify_greedy_block(uint32_t anchor, const uint32_t* drafts,
                             size_t draft_count, size_t max_draft,
                             size_t vocab, const uint32_t* targets,
                             size_t* accepted, uint32_t* committed,
                             size_t* committed_count, int* all_accepted);
/* New: counter-based uniform in [0,1) (SplitMix64 finaliser, 53 bits). */
double k3xo_uniform(uint64_t seed, uint64_t sequence, uint64_t position,
                    uint64_t purpose);
/* New: speculative rejection sampling over target logits [p+1][V] and
 * draft logits [p][V] at temperature tau, with the canonical reduction
 * order documented in k3x_oracle.c. */
int k3xo_verify_rejection(const float* target_logits,
                          const float* draft_logits, const uint32_t* drafts,
                          size_t draft_count, size_t vocab, float temperature,
                          uint64_t seed, uint64_t sequence, size_t* accepted,
                          uint32_t* committed, size_t* committed_count);

/* ---- seeded synthetic workloads (restates the library's generator) ------ */
/* The library's counter-based generator (project-k3x_b200/csrc/synth.cu):
 * pair i of (seed, stream) = SplitMix64 -> two 24-bit uniforms -> Box-Muller
 * with its own float series for log and sine/cosine, every operation
 * rounded to nearest, so the same bits come out here. Not a reference
 * function: it lets a CPU rebuild any slice of a workload that the GPU
 * generates in place (bench.py's reference arm). */
void k3xo_normal_pair(uint64_t seed, uint64_t stream, uint64_t pair, float* z0, float* z1);
/* out[j] = mean + sigma * z for global element first + j (element e uses
 * component e & 1 of pair e >> 1), as k3xb_fill_normal_f32. */
void k3xo_fill_normal_f32(float* out, size_t n, uint64_t first, uint64_t seed, uint64_t stream,
                          float mean, float sigma);
/* bf16 words of sigma * z, as k3xb_fill_normal_bf16. */
void k3xo_fill_normal_bf16(uint16_t* out, size_t n, uint64_t first, uint64_t seed, uint64_t stream,
                           float sigma);
/* MXFP4 32-blocks first .. first + blocks - 1 of sigma * z (block b holds
 * pairs 16b .. 16b + 15), quantised as k3xo_quantize_mxfp4, as
 * k3xb_fill_normal_mxfp4: packed [blocks][16] bytes, scales [blocks]. */
void k3xo_fill_normal_mxfp4(uint8_t* packed, uint8_t* scales, size_t blocks, uint64_t first,
                            uint64_t seed, uint64_t stream, float sigma);

/* ---- gated MLA (model.cpp:755-811) and its KV crop (model.cpp:1235-1251) -- */
/* Weights are f32 [rows][cols]; the products are the CPU backend's FP64
 * dense_matvec (backend_cpu.cpp:23-47), the norms ops.cpp:10-18. */
typedef struct {
    size_t hidden, heads, q_rank, kv_rank, q_main, q_extra, value_dim;
    float eps;
    const float* q_a_proj;    /* [q_rank][hidden] */
    const float* q_a_norm;    /* [q_rank] */
    const float* q_b_proj;    /* [heads * (q_main + q_extra)][q_rank] */
    const float* kv_a_proj;   /* [kv_rank + q_extra][hidden] */
    const float* kv_a_norm;   /* [kv_rank] */
    const float* kv_b_proj;   /* [heads * (q_main + value_dim)][kv_rank] */
    const float* g_proj;      /* [heads * value_dim][hidden] */
    const float* o_proj;      /* [hidden][heads * value_dim] */
} k3xo_mla_weights;
/* One position: appends its key, value and shared key at *length (the
 * state is position-major: keys [cap][heads][q_main], values
 * [cap][heads][value_dim], shared [cap][q_extra]), attends over positions
 * 0 .. *length, writes out [hidden] and increments *length. */
int k3xo_mla_step(const k3xo_mla_weights* w, const float* x, float* keys, float* values,
                  float* shared, size_t capacity, size_t* length, float* out);
/* A draft tree verified against a committed state of `length` positions:
 * node i (parent[i] < i, -1 = a root on the committed state) is projected
 * like a position of k3xo_mla_step and attends to the committed positions,
 * then its ancestors root first, then itself; on a chain this is the
 * sequential prefill bit for bit. Writes each node's key, value and shared
 * key (node_* [nodes][...], for the commit) and its output out [nodes][H].
 * New: the reference verifies chains only. */
int k3xo_mla_tree(const k3xo_mla_weights* w, const float* keys, const float* values,
                  const float* shared, size_t length, const int32_t* parent, size_t nodes,
                  const float* x, float* node_keys, float* node_values, float* node_shared,
                  float* out);
/* Crop to `keep` positions (a rejected draft's rollback); keep > *length
 * is invalid, as the reference's restore refuses it. */
int k3xo_mla_crop(size_t* length, size_t keep);

#ifdef __cplusplus
}
#endif
#endif
