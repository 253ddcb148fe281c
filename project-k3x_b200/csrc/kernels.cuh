// kernels.cuh — host-side launchers implemented by the .cu files of libk3xb.
#pragma once

#include "common.cuh"

namespace k3xb {

// router.cu
size_t plan_smem_bytes(uint32_t T, uint32_t E);
int launch_router_logits(k3xb_ctx* ctx, const float* hidden, uint32_t T, uint32_t H,
                         const uint16_t* W, uint32_t E, float* logits);
int launch_topk(k3xb_ctx* ctx, const float* logits, const float* correction, uint32_t T,
                uint32_t E, uint32_t K, uint32_t* ids, float* contrib, float* scores,
                int32_t* status);
int launch_select_routing(k3xb_ctx* ctx, const float* scores, uint32_t T, uint32_t E, const float* bias, uint32_t K,
                          const k3xb_routing_policy& policy, uint32_t* ids, float* weights, uint32_t* selected,
                          uint32_t* escalated, float* stats);
int launch_plan(k3xb_ctx* ctx, const uint32_t* ids, const float* contrib, uint32_t T,
                uint32_t K, uint32_t E, const k3xb_plan& plan);

// experts_simt.cu
int launch_simt_experts(k3xb_ctx* ctx, const k3xb_moe_layer& L, const float* hidden, uint32_t T,
                        const k3xb_plan& plan, float* act_buf, float* slot_out);
int launch_combine(k3xb_ctx* ctx, const float* slot_out, const float* contrib, const float* shared,
                   uint32_t T, uint32_t K, uint32_t H, float* out);
// the same over bf16 expert rows [T*k][H]
int launch_combine16(k3xb_ctx* ctx, const uint16_t* slot_out16, const float* contrib, const float* shared,
                     uint32_t T, uint32_t K, uint32_t H, float* out);
int launch_bf16_rows(k3xb_ctx* ctx, const float* x, const uint16_t* W, uint32_t T, uint32_t rows,
                     uint32_t cols, float* out);
int launch_act(k3xb_ctx* ctx, const float* g, const float* u, size_t n, int act, float beta,
               float lbeta, float* out);

// kda.cu
int launch_kda(k3xb_ctx* ctx, const float* state, const int32_t* order, const int32_t* depth,
               const int32_t* from_stack, uint32_t visit, uint32_t nodes, uint32_t sequences,
               uint32_t heads, uint32_t head_dim, const float* q, const float* k, const float* v,
               const float* log_decay, const float* beta, float* out, float* state_out,
               uint32_t levels, const int32_t* commit = nullptr);

// accept.cu
int launch_accept_greedy(k3xb_ctx* ctx, const float* logits, const uint32_t* drafts, uint32_t S,
                         uint32_t p, uint32_t V, uint32_t* targets, uint32_t* accepted,
                         uint32_t* committed, uint32_t* count);
int launch_accept_rejection(k3xb_ctx* ctx, const float* tl, const float* dl, const uint32_t* drafts,
                            uint32_t S, uint32_t p, uint32_t V, float temperature, uint64_t seed,
                            uint64_t seq_base, double* pd, double* qd, uint32_t* accepted,
                            uint32_t* committed, uint32_t* count);

// anchors[s] = committed[s][count[s] - 1] (the next round's anchor)
int launch_next_anchor(k3xb_ctx* ctx, const uint32_t* committed, const uint32_t* count, uint32_t S, uint32_t stride,
                       uint32_t* anchors);

// synth.cu
int launch_fill_normal_f32(k3xb_ctx* ctx, float* out, size_t n, uint64_t seed, uint64_t stream,
                           float mean, float sigma);
int launch_fill_normal_bf16(k3xb_ctx* ctx, uint16_t* out, size_t n, uint64_t seed, uint64_t stream,
                            float sigma);
int launch_quantize_mxfp4(k3xb_ctx* ctx, const float* x, size_t rows, size_t cols, uint8_t* packed,
                          uint8_t* scales);
int launch_fill_normal_mxfp4(k3xb_ctx* ctx, uint8_t* packed, uint8_t* scales, size_t rows, size_t cols,
                             uint64_t seed, uint64_t stream, float sigma);

}  // namespace k3xb

namespace k3xb {
// Where an expert-parallel call's down projection puts its outputs: received
// row r is token r % home_rows of home rank g = r / home_rows, and its
// (token, slot) output row goes to win[g] + y_off, row token * top_k + slot,
// as bf16 words. When every CTA is done, the last one stores `epoch` into
// flag word `rank` at win[g] + flag_off of every rank g (ep.cu).
struct EpTarget {
    uint8_t* win[8];        // each rank's exchange window as mapped in this process
    uint64_t y_off;         // byte offset of this call's output rows in every window
    uint64_t flag_off;      // byte offset of the return flags in every window
    uint32_t* done;         // this rank's grid-completion counter (device, zero between calls)
    uint32_t home_rows;     // rows each home rank sent (its token count)
    uint32_t rank, world, epoch;   // world 0: not expert parallel
};
// experts_tc.cu — tcgen05 block-scaled expert engine
size_t mxf4_scratch_bytes(const k3xb_moe_layer& L, uint32_t T);
// E2M1 activation terms when a layer leaves act_terms 0, from the whole
// batch's assignments (tokens x top_k) and its experts
uint32_t mxf4_default_terms(uint64_t assignments, uint32_t experts);
void set_mxf4_scratch(k3xb_ctx* ctx, void* region);
// slot_out [T*k][H] float, or bf16 words in slot_out16 when that is given, or
// (expert parallel) the home ranks' windows; rows are floats, or bf16 words
// in hidden16 when that is given
int launch_mxf4_experts(k3xb_ctx* ctx, const k3xb_moe_layer& L, const float* hidden, uint32_t T,
                        const k3xb_plan& plan, float* slot_out, uint16_t* slot_out16 = nullptr,
                        const EpTarget* ep = nullptr, const uint16_t* hidden16 = nullptr);
void release_mxf4_resources(k3xb_ctx* ctx);
int prepare_mxfp4_scales(k3xb_ctx* ctx, const uint8_t* scales, size_t rows, size_t cols, uint8_t* out);
// 2-D byte tensor map (128B swizzle, box {128 B, box_rows}); map is a CUtensorMap*
int make_byte_map(k3xb_ctx* ctx, void* map, const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_rows);
// linear_tc.cu — out[T][rows] = (round_bf16)(W . x), x split into two bf16 terms
size_t linear_scratch_bytes(uint32_t T, uint32_t K);
int launch_linear_bf16(k3xb_ctx* ctx, const float* x, const uint16_t* W, uint32_t T, uint32_t rows, uint32_t K,
                       int round_out, uint16_t* xterms, float* out);
// the same with the two-term split done once for several weights of one x
// terms = 1: x is bf16-valued (one row per token); 2: hi/lo split of any float
int launch_split_terms(k3xb_ctx* ctx, const float* x, uint32_t T, uint32_t K, uint32_t terms, uint16_t* xterms);
int launch_linear_terms(k3xb_ctx* ctx, const uint16_t* xterms, uint32_t terms, const uint16_t* W, uint32_t T,
                        uint32_t rows, uint32_t K, int round_out, float* out);
// up to 8 products of the same split x in one launch: out_j[T][rows_j] = W_j . x
struct LinearJob {
    const uint16_t* W;   // [rows][K] bf16 words
    uint32_t rows;
    float* out;
};
int launch_linear_group(k3xb_ctx* ctx, const uint16_t* xterms, uint32_t terms, uint32_t T, uint32_t K,
                        const LinearJob* jobs, uint32_t njobs, int round_out);
// dense.cu — f32 dense products in the reference CPU backend's FP64 column order
int launch_dense_matvec(k3xb_ctx* ctx, const float* W, uint32_t rows, uint32_t cols, const float* x, uint32_t T,
                        float* y);
int launch_mxfp4_matvec(k3xb_ctx* ctx, const uint8_t* packed, const uint8_t* scales, uint32_t rows, uint32_t cols,
                        const float* x, uint32_t T, float* y);
// resident.cu — the resident weight table
void release_resident(k3xb_ctx* ctx);
void resident_stats(const k3xb_ctx* ctx, k3xb_stats* out);
// attnres.cu — block attention residual over many sources
constexpr uint32_t kBlockAttnResMaxDepth = 64;   // sources + the prefix
int launch_block_attnres(k3xb_ctx* ctx, const float* prefix, const float* sources, uint32_t S, uint32_t T, uint32_t H,
                         const float* norm, const float* proj, float eps, float* out);
// layer.cu — KDA block and layer steps around the GEMMs
size_t attnres_smem_bytes(uint32_t H);
int launch_attnres_norm(k3xb_ctx* ctx, const float* a, const float* delta, const float* block, const uint16_t* rnorm,
                        const uint16_t* rproj, const uint16_t* post, uint32_t T, uint32_t H, float eps,
                        float* prefix_out, float* out);
int launch_short_conv(k3xb_ctx* ctx, const float* const proj[3], const float* const weight[3], const uint16_t* conv,
                      const int32_t* anc, uint32_t S, uint32_t N, uint32_t P, uint32_t w, float* const out[3]);
int launch_qk_gates(k3xb_ctx* ctx, const float* cq, const float* ck, const float* fg, const float* bp,
                    const float* a_log, const float* dt_bias, float glb, uint32_t T, uint32_t h, uint32_t d,
                    float* qn, float* kn, float* ld, float* be);
int launch_gated_norm(k3xb_ctx* ctx, const float* ro, const float* og, const float* o_norm, float eps, uint32_t T,
                      uint32_t h, uint32_t d, float* gt);
int launch_residual(k3xb_ctx* ctx, const float* a, const float* b, size_t n, float* out);
int launch_residual_round(k3xb_ctx* ctx, const float* a, size_t n, float* out);   // out = round_bf16(a)
int launch_conv_commit(k3xb_ctx* ctx, const float* const proj[3], const uint16_t* conv_in, const int32_t* anc_commit,
                       uint32_t S, uint32_t N, uint32_t P, uint32_t w, uint16_t* conv_out);
int launch_conv_commit_linear(k3xb_ctx* ctx, const float* const proj[3], const uint16_t* conv_in,
                              const uint32_t* commit, uint32_t S, uint32_t N, uint32_t P, uint32_t w,
                              uint16_t* conv_out);
int launch_rms_norm(k3xb_ctx* ctx, const float* x, const uint16_t* w, uint32_t T, uint32_t H, float eps, float* out);
int launch_embed(k3xb_ctx* ctx, const uint32_t* tokens, const uint16_t* table, uint32_t V, uint32_t T, uint32_t H,
                 float* out);
// ep.cu — expert parallelism (rows and expert outputs through peer-memory windows)
void release_ep(k3xb_ctx* ctx);
size_t ep_scratch_bytes(uint32_t G, uint32_t T, uint32_t K, uint32_t H, uint32_t E_r);
// rows_bf16: the rows are bf16-valued, so they travel as bf16 words
int ep_moe_forward(k3xb_ctx* ctx, const k3xb_moe_layer& local, uint32_t E, const float* hidden, uint32_t T,
                   const uint32_t* ids, const float* contrib, const float* shared, void* region, float* out,
                   bool rows_bf16);
// Sizes the exchange window for T tokens x K slots of width D before a
// sequence of calls is queued (collective; growing drains the stream).
int ep_reserve(k3xb_ctx* ctx, uint32_t T, uint32_t K, uint32_t D);
// After a drain: a bounded device wait that gave up aborts the exchange.
int ep_check_waits(k3xb_ctx* ctx);
int ep_world(const k3xb_ctx* ctx);   // 0 when expert parallelism is not initialised
// Waits for ctx->stream with the communicator's bound (ep_guard.hpp); OK at
// once without expert parallelism.
int ep_drain(k3xb_ctx* ctx);
// shared expert on kind::f16 tensor cores; xb [2T][H], bd [2T][Is] bf16 scratch
int launch_shared_tc(k3xb_ctx* ctx, const k3xb_moe_layer& L, const float* hidden, uint32_t T, uint16_t* xb,
                     uint16_t* bd, float* out);
}  // namespace k3xb
