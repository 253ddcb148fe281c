/*
 * k3xb.h — C ABI of the B200-native K3X speculative-verification library
 * (libk3xb.so, built from project-k3x_b200/csrc for sm_100a).
 *
 * Plain pointers and sizes only. Every array argument is DEVICE memory on
 * the context's GPU and the call is asynchronous on the context's current
 * stream (k3xb_set_stream), except where a name ends in _host and for the
 * resident-weight uploads (k3xb_acquire_*), which read HOST arrays. A call
 * makes the context's GPU the calling thread's current device; a context is
 * used by one thread at a time. All
 * entry points return a status that mirrors k3x::ErrorCode
 * (runtime/include/k3x/status.hpp:9-30); k3xb_last_error() gives the
 * message of the last failure on a context. There is no CPU fallback: a
 * missing or unsupported device returns K3XB_BACKEND_UNAVAILABLE or
 * K3XB_UNSUPPORTED_ARCHITECTURE.
 *
 * Each entry point names the reference interface it replaces. The C++20
 * adapter project-k3x_b200/adapter/backend_b200.cpp maps
 * k3x::ComputeBackend (runtime/include/k3x/backend.hpp:326-462) onto these
 * calls for the reference runtime; include/k3xb.hpp is the C++20 host
 * layer over them.
 */
#ifndef K3XB_H
#define K3XB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes: runtime/include/k3x/status.hpp:9-30 ---------------- */
enum {
    K3XB_OK = 0,
    K3XB_INVALID_EXTENT = 9,
    K3XB_INVALID_MXFP4 = 15,
    K3XB_INVALID_STATE = 16,
    K3XB_BACKEND_UNAVAILABLE = 17,
    K3XB_UNSUPPORTED_ARCHITECTURE = 19,
};

/* Expert / shared-expert activation. SwiGLU is situ_glu's beta -> inf limit
 * without a linear bound; SiTU is runtime/src/ops.cpp:20-30. */
enum { K3XB_ACT_SWIGLU = 0, K3XB_ACT_SITU = 1 };

/* Expert GEMM engine. MXF4 = tcgen05 block-scaled kind::mxf4 tensor cores
 * (E2M1 weights and activation terms, E8M0 per-32 scales, TMEM
 * accumulators); SIMT = CUDA-core FP4 decode + FP32 FMA (cross-check). */
enum { K3XB_ENGINE_MXF4 = 0, K3XB_ENGINE_SIMT = 1 };

typedef struct k3xb_ctx k3xb_ctx;

/* ---- context ------------------------------------------------------------ */
/* Replaces make_cuda_backend (runtime/include/k3x/backend.hpp:465-466):
 * requires compute capability 10.x (B200) and returns
 * K3XB_UNSUPPORTED_ARCHITECTURE otherwise. */
int k3xb_create(int device, k3xb_ctx** out);
int k3xb_destroy(k3xb_ctx* ctx);
/* Copies the last error message (NUL-terminated, truncated to len). */
int k3xb_last_error(const k3xb_ctx* ctx, char* buf, size_t len);
/* Stream for subsequent calls (a cudaStream_t); NULL = the context's own
 * non-blocking stream (backend_cuda.cu:5344-5348 keeps one stream too). */
int k3xb_set_stream(k3xb_ctx* ctx, void* stream);
int k3xb_sync(k3xb_ctx* ctx);

/* Counters in the spirit of k3x::BackendRuntimeStats (backend.hpp:50-129). */
typedef struct {
    uint64_t kernel_launches;
    uint64_t route_calls;
    uint64_t moe_layer_calls;
    uint64_t moe_layer_experts;
    uint64_t kda_calls;
    uint64_t accept_calls;
    uint64_t scratch_bytes;
    uint64_t peak_scratch_bytes;
    uint64_t h2d_bytes;
    uint64_t d2h_bytes;
    /* resident weights (k3xb_acquire_weight / k3xb_acquire_expert_stack) */
    uint64_t weight_cache_hits;
    uint64_t weight_cache_misses;
    uint64_t weight_cache_bypasses;
    uint64_t resident_weight_bytes;
    uint64_t peak_resident_weight_bytes;
    uint64_t weight_h2d_bytes;
} k3xb_stats;
int k3xb_get_stats(const k3xb_ctx* ctx, k3xb_stats* out);

/* Device time per phase of the path (the reference's Profiler,
 * runtime/include/k3x/profile.hpp:32-63, and the CUDA events its backend
 * records around each operation). Every phase is also an NVTX range. With
 * profiling on, each phase records a pair of CUDA events on its stream
 * (none while a stream is captured into a graph); k3xb_get_profile waits
 * for them and adds their elapsed time to the phase's total. Phases on the
 * side stream (the shared expert) overlap others, so totals can sum to more
 * than the call's wall time. */
enum {
    K3XB_PHASE_ROUTE = 0,          /* router logits + Top-k */
    K3XB_PHASE_PLAN,               /* expert-major bucketing */
    K3XB_PHASE_EXPERT_PREP,        /* work list, activation split, row gather */
    K3XB_PHASE_EXPERT_GATEUP,      /* gate/up grouped GEMM + activation */
    K3XB_PHASE_EXPERT_DOWN,        /* down grouped GEMM + scatter */
    K3XB_PHASE_SHARED,             /* shared expert */
    K3XB_PHASE_COMBINE,            /* slot-ordered combine (+ shared) */
    K3XB_PHASE_EP_DISPATCH,        /* expert parallelism: send buffers */
    K3XB_PHASE_EP_EXCHANGE,        /* rows + metadata all-to-all */
    K3XB_PHASE_EP_RETURN,          /* expert outputs back to their tokens */
    K3XB_PHASE_ATTN_RESIDUAL,      /* attention residual + RMSNorm */
    K3XB_PHASE_KDA_PROJECT,        /* q/k/v/f/b/g projections */
    K3XB_PHASE_KDA_CONV,           /* short conv, q/k norm, gates */
    K3XB_PHASE_KDA_RECURRENCE,     /* gated delta rule over the draft tree */
    K3XB_PHASE_KDA_OUTPUT,         /* gated norm + output projection */
    K3XB_PHASE_EMBED,              /* token embedding */
    K3XB_PHASE_LM_HEAD,            /* final norm + LM head */
    K3XB_PHASE_ACCEPT,             /* greedy / rejection acceptance */
    K3XB_PHASE_COMMIT,             /* state commit of the accepted path */
    K3XB_PHASE_LATENT,             /* LatentMoE projections and routed norm */
    K3XB_PHASE_COUNT
};
typedef struct {
    double device_ms;   /* summed over calls */
    uint64_t calls;
} k3xb_phase_time;
/* enable != 0 starts recording; either way the totals are cleared. */
int k3xb_set_profiling(k3xb_ctx* ctx, int enable);
/* Synchronises with the recorded events and copies K3XB_PHASE_COUNT totals
 * to out. dropped (may be NULL): phases not timed because more than 4096
 * were pending; read the profile at least every few thousand phases. */
int k3xb_get_profile(k3xb_ctx* ctx, k3xb_phase_time* out, uint64_t* dropped);
/* Name of a K3XB_PHASE_* value ("route", "expert_gateup", ...), or NULL. */
const char* k3xb_phase_name(int phase);

/* ---- (a) router ---------------------------------------------------------- */
/* route_official_moe (runtime/src/official_moe.cpp:247-269) for T tokens:
 * logits = float(sum_h double(bf16 W[e][h]) * hidden[t][h]) summed in h
 * order (bit-identical to the reference), scores = sigmoid, Top-k by
 * (score + correction) desc / index asc, contributions = score / double
 * sum. ids/contributions are [T][k]; scores [T][E] may be NULL. */
int k3xb_route(k3xb_ctx* ctx, const float* hidden, uint32_t tokens,
               uint32_t hidden_size, const uint16_t* router,
               const float* correction, uint32_t experts, uint32_t top_k,
               uint32_t* ids, float* contributions, float* scores);

/* The logits of route_official_moe alone (official_moe.cpp:255-267): the
 * [T][E] floats k3xb_route feeds to its Top-k, for a caller that routes them
 * itself (route_official_moe_logits, official_moe.cpp:211-245, takes
 * them). Bit-identical to the reference's sequential double sums. */
int k3xb_router_logits(k3xb_ctx* ctx, const float* hidden, uint32_t tokens,
                       uint32_t hidden_size, const uint16_t* router,
                       uint32_t experts, float* logits);

/* Same routing as k3xb_route for callers that may not allocate device
 * memory while they run (a serving loop that reserved all of HBM up front,
 * an application whose own allocator owns the device, a latency-critical
 * loop where cudaMalloc/cudaFree would synchronise the device). No
 * counterpart in the reference. Needs no context: the logits live in a
 * 1 MiB array compiled into the library (one per GPU, held until exit), so
 * tokens * experts must be <= 262144, else K3XB_INVALID_EXTENT. Runs on
 * `stream` (a cudaStream_t, NULL = legacy default stream) of the current
 * device and returns before the work finishes. `status` (device int32)
 * receives K3XB_INVALID_EXTENT for non-finite inputs and
 * K3XB_BACKEND_UNAVAILABLE when a bounded wait in the logits kernel ran out;
 * with status NULL those device-side failures are dropped (the call still
 * returns K3XB_OK and ids/contributions are then undefined), so callers
 * that cannot rule them out should pass a status word. All calls on a
 * device share the array, so calls that overlap on the GPU race. The first
 * call on each device looks the array up once; make it before any stream
 * capture starts. */
int k3xb_route_static(const float* hidden, uint32_t tokens, uint32_t hidden_size,
                      const uint16_t* router, const float* correction,
                      uint32_t experts, uint32_t top_k, uint32_t* ids,
                      float* contributions, int32_t* status, void* stream);

/* select_routing (runtime/src/routing_policy.cpp:31-159), the synthetic
 * engine's routing policy (model.cpp:245, :925) over sigmoid scores:
 * natural Top-k, a fixed K from the ladder {4, 6, 8, 12, 16}, or an
 * adaptive K (natural Top-16 cut at the first ladder K that reaches
 * mass_target, covers the entropy support exp(H) and clears
 * minimum_boundary_gap), raised to quality_floor_k (0 = none). */
enum { K3XB_ROUTING_NATURAL = 0, K3XB_ROUTING_FIXED = 1, K3XB_ROUTING_ADAPTIVE = 2 };
typedef struct {
    int32_t mode;              /* K3XB_ROUTING_* */
    uint32_t fixed_k;
    float mass_target;         /* (0, 1] */
    float minimum_gap;         /* [0, 1] */
    uint32_t quality_floor_k;
} k3xb_routing_policy;
/* scores [T][E] in [0, 1], bias [E]; natural_k <= min(32, E), E <= 1024.
 * Outputs [T][natural_k]: expert_ids (UINT32_MAX past the selected K) and
 * normalized weights (0 there); selected_k [T]; escalated [T] (may be NULL:
 * the floor raised K); stats [T][4] (may be NULL): normalized entropy,
 * entropy support, selected mass, boundary confidence. Policy errors return
 * K3XB_INVALID_STATE; invalid scores set the device status word to it. */
int k3xb_select_routing(k3xb_ctx* ctx, const float* scores, uint32_t tokens,
                        uint32_t experts, const float* bias, uint32_t natural_k,
                        const k3xb_routing_policy* policy, uint32_t* expert_ids,
                        float* weights, uint32_t* selected_k, uint32_t* escalated,
                        float* stats);

/* build_expert_major_plan (runtime/src/expert_major.cpp:10-54): groups in
 * first-use order, assignments in (token, slot) order inside a group.
 * group_offset has room for experts+1 entries; the used prefix is
 * group_count[0]+1. Duplicate ids in a token or non-finite contributions
 * set status[0] = K3XB_INVALID_STATE (device-side; read it after sync). */
typedef struct {
    uint32_t* group_expert;    /* [experts] */
    uint32_t* group_offset;    /* [experts + 1] */
    uint32_t* assign_token;    /* [T * k] */
    uint32_t* assign_slot;     /* [T * k] */
    float* assign_contrib;     /* [T * k] */
    uint32_t* group_count;     /* [1] */
    int32_t* status;           /* [1] */
} k3xb_plan;
int k3xb_expert_major_plan(k3xb_ctx* ctx, const uint32_t* ids,
                           const float* contributions, uint32_t tokens,
                           uint32_t top_k, uint32_t experts,
                           const k3xb_plan* plan);

/* ---- (b)+(c) resident MoE layer ----------------------------------------- */
/* Plain (hidden-space) MoE layer over device-resident weights: route ->
 * expert-major plan -> grouped expert FFN -> slot-ordered weighted combine
 * -> + shared expert. Replaces resident_mxfp4_moe_layer /
 * official_mxfp4_moe_ffn (backend.hpp:369-397; official_moe.cpp:271-344
 * without the latent projections). Expert weights are stacked:
 * gate/up [E][I][H/2] (+ scales [E][I][H/32]), down [E][H][I/2] (+ scales
 * [E][H][I/32]), reference MXFP4 layout (low nibble = even column). */
typedef struct {
    uint32_t hidden, inter, experts, top_k, shared_inter;
    const uint16_t* router;        /* [E][H] bf16 */
    const float* correction;       /* [E] */
    const uint8_t* gate_packed;
    const uint8_t* gate_scales;
    const uint8_t* up_packed;
    const uint8_t* up_scales;
    const uint8_t* down_packed;
    const uint8_t* down_scales;
    const uint16_t* shared_gate;   /* [Is][H] bf16, or NULL */
    const uint16_t* shared_up;     /* [Is][H] */
    const uint16_t* shared_down;   /* [H][Is] */
    int32_t activation;            /* K3XB_ACT_* */
    float situ_beta, situ_linear_beta;  /* linear_beta <= 0: none */
    int32_t engine;                /* K3XB_ENGINE_* */
    int32_t act_terms;             /* E2M1 activation terms (MXF4 engine); 0 = the
                                      library default: 6 (exact for bf16 rows)
                                      while the batch gives experts fewer than 12
                                      tokens on average (tokens x top_k / experts),
                                      4 from there on (k3xb_default_act_terms) */
    /* Optional copies of the three scale arrays in the tcgen05 layout made by
     * k3xb_prepare_mxfp4_scales (same byte count). When NULL the MXF4 engine
     * re-lays the scales into its scratch on every call. */
    const uint8_t* gate_scales_tc;
    const uint8_t* up_scales_tc;
    const uint8_t* down_scales_tc;
    /* LatentMoE (official_moe_cpu, official_moe.cpp:271-344 with :296 and
     * :322-331): latent = round_bf16(routed_down . hidden) [L]; the experts
     * work on the latent row (their stacks are gate/up [E][I][L/2], down
     * [E][L][I/2]); mixed = round_bf16(slot-ordered combine) [L]; routed =
     * round_bf16(routed_up . rms_norm(mixed, routed_norm, latent_eps)) [H];
     * out = round_bf16(routed + shared). latent = 0: the plain MoE above.
     * The router still reads the hidden row. */
    uint32_t latent;
    const uint16_t* routed_down;   /* [L][H] bf16 */
    const uint16_t* routed_norm;   /* [L] bf16 */
    const uint16_t* routed_up;     /* [H][L] bf16 */
    float latent_eps;
    /* Expert placement for the expert-parallel entry points (device array
     * [experts_total], or NULL): entry e = rank << 16 | local, the rank that
     * holds expert e and its index in that rank's stacks. Every (rank,
     * local) with rank < world and local < E / world appears exactly once.
     * NULL: rank r holds experts [r*E/world, (r+1)*E/world) in order.
     * Placement moves no result: the outputs are bit-identical for any
     * table (k3xb_ep_balance makes one from expected loads). Ignored by the
     * one-GPU entry points. */
    const uint32_t* ep_owner;
} k3xb_moe_layer;

/* bf16_matvec (runtime/src/official_moe.cpp:39-59) for many tokens on
 * tcgen05 kind::f16 tensor cores: out[t][r] = sum_k W[r][k] * x[t][k],
 * rounded to bf16 when round_output != 0. W [out_features][in_features]
 * bf16 words, x [tokens][in_features] float, out [tokens][out_features].
 * FP32 accumulation (the reference accumulates in FP64); x is carried as
 * two bf16 terms, exact for bf16-valued x. in_features % 8 == 0. Used for
 * the LM head and the KDA projections. */
int k3xb_linear_bf16(k3xb_ctx* ctx, const float* x, uint32_t tokens,
                     uint32_t in_features, const uint16_t* weight,
                     uint32_t out_features, int32_t round_output, float* out);

/* Re-lays MXFP4 scales [rows][cols/32] (rows % 128 == 0, cols % 128 == 0)
 * into the layout the tcgen05 block-scaled MMA reads: 512-byte atoms of 128
 * rows x 4 scale blocks, atoms[rows/128][cols/128]. Done once per resident
 * weight, like the reference's one-time resident upload (resident_weights.cuh). */
int k3xb_prepare_mxfp4_scales(k3xb_ctx* ctx, const uint8_t* scales, size_t rows,
                              size_t cols, uint8_t* out);

/* out [T][H] = round_bf16(mixed + shared); ids/contributions [T][k] and
 * plan_out may be NULL. */
int k3xb_moe_layer_forward(k3xb_ctx* ctx, const k3xb_moe_layer* layer,
                           const float* hidden, uint32_t tokens, float* out,
                           uint32_t* ids, float* contributions);
/* Same with HOST hidden/out/ids/contributions: copies in, runs, copies out
 * and synchronises (the reference's resident layer returns by value). */
int k3xb_moe_layer_forward_host(k3xb_ctx* ctx, const k3xb_moe_layer* layer,
                                const float* hidden_host, uint32_t tokens,
                                float* out_host, uint32_t* ids_host,
                                float* contributions_host);

/* The E2M1 activation term count the MXF4 engine uses for a layer whose
 * act_terms is 0, for a batch of `assignments` (tokens x top_k) over
 * `experts` routed experts (the whole batch for an expert-parallel layer).
 * No reference counterpart (the reference multiplies float activations). */
uint32_t k3xb_default_act_terms(uint64_t assignments, uint32_t experts);

/* Expert FFN only, for an existing plan (mxfp4_situ_mlp_grid,
 * backend.hpp:357-363): y[t][slot][D] = round_bf16(expert(hidden[t])), D the
 * experts' width (the latent width of a LatentMoE layer, whose rows the
 * caller then passes as `hidden`). */
int k3xb_moe_experts(k3xb_ctx* ctx, const k3xb_moe_layer* layer,
                     const float* hidden, uint32_t tokens,
                     const k3xb_plan* plan, float* slot_out);

/* ---- resident weights ------------------------------------------------------ */
/* Device copies of HOST weights, kept by the context and keyed by tensor id:
 * the reference's ResidentWeightTable (runtime/cuda/resident_weights.cuh:
 * 17-47, acquire in resident_weights.cu:104-166), which its CUDA backend
 * fills from the host views Bf16WeightView / Mxfp4WeightView
 * (backend.hpp:131-158). Same rules: a payload that does not match its key
 * or a tensor id seen with another shape is K3XB_INVALID_EXTENT; a held key
 * is a HIT (no copy); a new entry that would pass the capacity is a BYPASS
 * (K3XB_OK, null pointers, nothing kept); otherwise ADMITTED. In addition,
 * MXFP4 scales are checked at admission (0xFF -> K3XB_INVALID_MXFP4) and
 * MXFP4 entries with rows and cols multiples of 128 also hold the scales in
 * the tcgen05 layout (scales_tc). Copies are issued on the context's stream;
 * the host arrays may be reused when the call returns. */
enum {
    K3XB_WEIGHT_F32 = 0,           /* values [rows][cols] float */
    K3XB_WEIGHT_BF16 = 1,          /* values [rows][cols] bf16 words */
    K3XB_WEIGHT_MXFP4 = 2,         /* packed [rows][cols/2] + scales [rows][cols/group] */
    K3XB_WEIGHT_EXPERT_STACK = 3   /* k3xb_acquire_expert_stack */
};
enum { K3XB_RESIDENT_HIT = 0, K3XB_RESIDENT_ADMITTED = 1, K3XB_RESIDENT_BYPASS = 2 };

typedef struct {
    int32_t disposition;           /* K3XB_RESIDENT_* */
    const void* primary;           /* values / MXFP4 packed (device) */
    const void* secondary;         /* MXFP4 scales (device), else NULL */
    const void* scales_tc;         /* MXFP4 scales in the tcgen05 layout, or NULL */
    uint64_t uploaded_bytes;       /* host->device bytes of this call */
} k3xb_resident;

/* Bytes the table may hold (default: no bound but device memory). Entries
 * already held stay. */
int k3xb_set_resident_capacity(k3xb_ctx* ctx, uint64_t bytes);
/* primary_bytes / secondary_bytes must be what (representation, rows,
 * cols, group_size) imply: f32 rows*cols*4, bf16 rows*cols*2 (group 0, no
 * secondary), MXFP4 rows*cols/2 and rows*cols/group_size. */
int k3xb_acquire_weight(k3xb_ctx* ctx, uint64_t tensor_id, int32_t representation,
                        uint64_t rows, uint64_t cols, uint64_t group_size,
                        const void* primary, size_t primary_bytes,
                        const void* secondary, size_t secondary_bytes,
                        k3xb_resident* out);

/* One expert's HOST MXFP4 arrays (gate/up [I][H/2] + [I][H/32], down
 * [H][I/2] + [H][I/32]): an element of the Mxfp4MlpView list the
 * reference's MoE methods take (backend.hpp:315-319). */
typedef struct {
    const uint8_t* gate_packed;
    const uint8_t* gate_scales;
    const uint8_t* up_packed;
    const uint8_t* up_scales;
    const uint8_t* down_packed;
    const uint8_t* down_scales;
} k3xb_mxfp4_expert_host;

/* Device pointers of a resident expert stack, ready for the expert fields
 * of k3xb_moe_layer (including the *_scales_tc copies). */
typedef struct {
    int32_t disposition;           /* K3XB_RESIDENT_* */
    const uint8_t* gate_packed;
    const uint8_t* gate_scales;
    const uint8_t* up_packed;
    const uint8_t* up_scales;
    const uint8_t* down_packed;
    const uint8_t* down_scales;
    const uint8_t* gate_scales_tc;
    const uint8_t* up_scales_tc;
    const uint8_t* down_scales_tc;
    uint64_t uploaded_bytes;
} k3xb_resident_stack;

/* Uploads `experts` experts into one resident stack in the stacked layout
 * of k3xb_moe_layer, keyed by stack_id (same table, capacity and
 * counters; hidden and inter multiples of 128). A BYPASS leaves the
 * pointers NULL. */
int k3xb_acquire_expert_stack(k3xb_ctx* ctx, uint64_t stack_id, uint32_t experts,
                              uint32_t hidden, uint32_t inter,
                              const k3xb_mxfp4_expert_host* host,
                              k3xb_resident_stack* out);
/* Frees every resident entry (pointers handed out before become invalid). */
int k3xb_release_resident(k3xb_ctx* ctx);

/* mxfp4_situ_mlp_grid (backend.hpp:357-363, CPU semantics
 * backend_cpu.cpp:191-262) over a stack of experts (rows of the experts'
 * width H: the latent width for a LatentMoE layer): out[j][t][H] =
 * expert_{expert_ids[j]}(inputs[t]) for j < n, t < tokens: gate/up MXFP4
 * products, the layer's activation, down product rounded to bf16 as
 * expert_ffn (official_moe.cpp:82-103) does (the reference backend's
 * per-token methods return it unrounded, a difference inside their 2e-2
 * CUDA tolerance). Only the dims, expert arrays, activation, act_terms and
 * engine of `layer` are read; expert ids must be distinct (at most 32).
 * HOST inputs [tokens][H], out [n][tokens][H] and expert_ids; returns after
 * the results are on the host. */
int k3xb_expert_grid_host(k3xb_ctx* ctx, const k3xb_moe_layer* layer,
                          const uint32_t* expert_ids, uint32_t n,
                          const float* inputs_host, uint32_t tokens,
                          float* out_host);

/* official_mxfp4_moe_ffn (backend.hpp:376-381; the reference's CUDA
 * backend_cuda.cu:3717-4172) for ONE position with its route given: the
 * LatentMoE tail of official_moe_cpu (official_moe.cpp:296-341).
 *   latent   = bf16_matvec(hidden, routed_down)
 *   y_k      = expert of slot k on the latent row (bf16-rounded down product)
 *   mixed    = round_bf16(sum_k contributions[k] * y_k, in slot order)
 *   routed   = bf16_matvec(normalized(mixed, routed_norm, latent_eps), routed_up)
 *   combined = round_bf16(routed + shared(hidden))   (no shared expert: round_bf16(routed))
 *   out      = round_bf16(round_bf16(prefix) + combined)
 * `tail` gives hidden, latent, shared_inter, the routed_* and shared_*
 * weights, latent_eps and the activation (shared and experts alike); its
 * expert fields are not read. slots[k] (K <= 64) is one expert (experts =
 * 1 of the latent width: latent, or hidden when latent is 0; one inter and
 * engine for all; MXF4 needs
 * the *_scales_tc copies), e.g. a resident stack of one
 * (k3xb_acquire_expert_stack) or single resident MXFP4 weights for the SIMT
 * engine. The shared expert runs on the tensor cores with the MXF4 engine
 * when hidden and shared_inter are multiples of 128 (as in
 * k3xb_moe_layer_forward), else on the CUDA cores, so the result equals the
 * layer path's bit for bit. hidden is the prepared (bf16-valued) MoE input; HOST
 * contributions [K], hidden [H], prefix [H] and out [H]; returns after out
 * is on the host. */
int k3xb_official_moe_ffn_host(k3xb_ctx* ctx, const k3xb_moe_layer* tail,
                               const k3xb_moe_layer* slots, uint32_t K,
                               const float* contributions, const float* hidden,
                               const float* prefix, float* out);

/* dense_matvec (backend.hpp:332-334; CPU semantics backend_cpu.cpp:23-47)
 * for `tokens` inputs: y[t][r] = float(sum over c in column order of
 * double(W[r][c]) * x[t][c]), bit-identical to the reference CPU backend.
 * Device W [rows][cols] float, x [tokens][cols], y [tokens][rows]. */
int k3xb_dense_matvec(k3xb_ctx* ctx, const float* W, uint32_t rows,
                      uint32_t cols, const float* x, uint32_t tokens,
                      float* y);
/* The same for one HOST input x [cols] and HOST y [rows] (W on the device,
 * e.g. resident); returns after y is on the host. */
int k3xb_dense_matvec_host(k3xb_ctx* ctx, const float* W, uint32_t rows,
                           uint32_t cols, const float* x_host, float* y_host);
/* dense_situ_mlp (backend.hpp:344-347; CPU semantics backend_cpu.cpp:
 * 107-122): down(situ_glu(gate x, up x)) with the products above; device
 * gate/up [inter][cols], down [out_rows][inter]; linear_beta 0 = no linear
 * bound. situ_glu uses the device's tanhf/expf, so the activation can differ
 * from the host's libm in the last bit. HOST x [cols], y [out_rows]. */
int k3xb_dense_situ_mlp_host(k3xb_ctx* ctx, const float* gate, const float* up,
                             const float* down, uint32_t inter, uint32_t cols,
                             uint32_t out_rows, const float* x_host, float beta,
                             float linear_beta, float* y_host);

/* mxfp4_matvec (backend.hpp:335-337; CPU semantics mxfp4_matmul,
 * ops.cpp:44-76) for `tokens` inputs: y[t][r] = float(sum over c in column
 * order of double(x[t][c]) * w[r][c]), w the decoded MXFP4 value
 * (ldexp(e2m1, scale - 127)), bit-identical to the reference. Device packed
 * [rows][cols/2], scales [rows][cols/32] (group 32, 0xFF refused at
 * admission, e.g. k3xb_acquire_weight), x [tokens][cols], y [tokens][rows]. */
int k3xb_mxfp4_matvec(k3xb_ctx* ctx, const uint8_t* packed, const uint8_t* scales,
                      uint32_t rows, uint32_t cols, const float* x, uint32_t tokens,
                      float* y);
/* The same for one HOST x [cols] and HOST y [rows]. */
int k3xb_mxfp4_matvec_host(k3xb_ctx* ctx, const uint8_t* packed, const uint8_t* scales,
                           uint32_t rows, uint32_t cols, const float* x_host,
                           float* y_host);

/* One expert's DEVICE MXFP4 arrays (layouts of k3xb_mxfp4_expert_host). */
typedef struct {
    const uint8_t* gate_packed;
    const uint8_t* gate_scales;
    const uint8_t* up_packed;
    const uint8_t* up_scales;
    const uint8_t* down_packed;
    const uint8_t* down_scales;
} k3xb_mxfp4_expert;
/* resident_mxfp4_moe_layer (backend.hpp:369-375; CPU semantics
 * backend_cpu.cpp:305-339) for one position, f32 dense projections:
 * latent = dense(x, routed_down [D][H]); per slot k the expert's
 * gate/up [I][D] and down [D][I] MXFP4 products (k3xb_mxfp4_matvec) around
 * situ_glu, unrounded; mixed = sum over slots in order of contributions[k] *
 * y_k in float; rms_norm(mixed, routed_norm [D], eps) in float (FP64
 * squares); routed = dense(., routed_up [H][D]); plus the dense SiTU shared
 * MLP (shared_gate/up [Hs][H], shared_down [H][Hs]) in float. The products
 * and norm are bit-identical to the CPU backend; situ_glu uses the device's
 * tanhf/expf. Weights are device arrays; HOST contributions [K], x [H],
 * y [H]; returns after y is on the host. */
int k3xb_resident_moe_layer_host(k3xb_ctx* ctx, uint32_t hidden, uint32_t latent,
                                 uint32_t inter, uint32_t shared_inter,
                                 const float* routed_down, const float* routed_norm,
                                 const float* routed_up, const float* shared_gate,
                                 const float* shared_up, const float* shared_down,
                                 const k3xb_mxfp4_expert* experts, uint32_t K,
                                 const float* contributions, float eps, float beta,
                                 float linear_beta, const float* x_host, float* y_host);

/* ---- (d) KDA recurrence -------------------------------------------------- */
/* official_kda.cpp:319-369 applied over a draft tree for S sequences that
 * share the topology: node n continues from parent[n]'s state
 * (parent[n] = -1: the prefix state; parent[n] < n). A linear draft is
 * parent[n] = n - 1. parent is a HOST array. Device arrays:
 * state [S][h][d][d] (V-first), q/k/v/log_decay [S][N][h*d],
 * beta [S][N][h], out [S][N][h*d]. */
int k3xb_kda_tree(k3xb_ctx* ctx, const float* state, const int32_t* parent,
                  uint32_t nodes, uint32_t sequences, uint32_t heads,
                  uint32_t head_dim, const float* q, const float* k,
                  const float* v, const float* log_decay, const float* beta,
                  float* out);
/* Replays root..commit_node[s] and writes that node's state to state_out
 * (bit-identical to the state k3xb_kda_tree computed for it);
 * commit_node[s] = -1 copies the prefix state. commit_node is HOST. */
int k3xb_kda_commit(k3xb_ctx* ctx, const float* state, const int32_t* parent,
                    uint32_t nodes, uint32_t sequences, uint32_t heads,
                    uint32_t head_dim, const float* q, const float* k,
                    const float* v, const float* log_decay, const float* beta,
                    const int32_t* commit_node, float* state_out);

/* ---- full KDA block and the KDA + MoE layer -------------------------------- */
/* Weights of one official KDA block (official_kda.hpp / official_kda.cpp:
 * 198-426), bf16 words unless marked float. P = heads * head_dim, H the
 * model width, w = conv_width. */
typedef struct {
    uint32_t heads, head_dim, conv_width;
    float eps, gate_lower_bound;
    const uint16_t* q_proj;     /* [P][H] */
    const uint16_t* k_proj;     /* [P][H] */
    const uint16_t* v_proj;     /* [P][H] */
    const float* q_conv;        /* [P][w] float */
    const float* k_conv;        /* [P][w] float */
    const float* v_conv;        /* [P][w] float */
    const uint16_t* f_a_proj;   /* [d][H] */
    const uint16_t* f_b_proj;   /* [P][d] */
    const float* a_log;         /* [d] float */
    const float* dt_bias;       /* [P] float */
    const uint16_t* b_proj;     /* [h][H] */
    const uint16_t* g_proj;     /* [P][H] */
    const float* o_norm;        /* [d] float */
    const uint16_t* o_proj;     /* [H][P] */
} k3xb_kda_layer;

/* Device bytes of the trace k3xb_kda_block leaves for a later commit: the
 * recurrence inputs q, k, v, log-decay, beta and the projected q, k, v of
 * every node. */
size_t k3xb_kda_trace_bytes(const k3xb_kda_layer* w, uint32_t nodes,
                            uint32_t sequences);

/* official_kda_cpu (official_kda.cpp:198-426) over a draft topology shared
 * by S sequences (parent is a HOST array, as for k3xb_kda_tree): node n's
 * short-conv window and recurrent state continue from its ancestors, and
 * from the sequence's prefix state below the roots. A linear draft is
 * parent[n] = n - 1. hidden [S][N][H]; conv [S][3][w-1][P] bf16 words (the
 * q, k, v histories, oldest row first); recurrent [S][h][d][d]. Neither
 * state is modified. out [S][N][H]. trace (k3xb_kda_trace_bytes) may be
 * NULL when no commit follows. */
int k3xb_kda_block(k3xb_ctx* ctx, const k3xb_kda_layer* w, uint32_t hidden,
                   const float* x, const int32_t* parent, uint32_t nodes,
                   uint32_t sequences, const uint16_t* conv,
                   const float* recurrent, float* out, void* trace);

/* The state after node commit_node[s] (HOST; -1 keeps the prefix state)
 * from a k3xb_kda_block trace, as Engine::forward_expert_major_block's
 * commit (model.cpp:1660-1664) keeps the last committed position: the
 * recurrent state replayed along the path (bit-identical to the verify
 * pass) and the conv windows ending at that node. conv_out may alias conv;
 * recurrent_out must not alias recurrent. */
int k3xb_kda_block_commit(k3xb_ctx* ctx, const k3xb_kda_layer* w,
                          const void* trace, const int32_t* parent,
                          uint32_t nodes, uint32_t sequences,
                          const int32_t* commit_node, const uint16_t* conv,
                          const float* recurrent, uint16_t* conv_out,
                          float* recurrent_out);

/* official_kda (backend.hpp:402-408) in its host-roundtrip state mode
 * (OfficialKdaStateMode::host_roundtrip): one sequence's `tokens`
 * positions of HOST x [tokens][H] run as a chain through the KDA block;
 * out [tokens][H] (HOST); the state after the last position replaces
 * conv [3][w-1][P] (bf16 words: the q, k, v histories of
 * OfficialKdaCudaStateView, oldest row first) and recurrent [h][d][d]
 * (V-first). Weights are device arrays (e.g. resident, k3xb_acquire_weight).
 * Returns after the results are on the host. */
int k3xb_kda_block_host(k3xb_ctx* ctx, const k3xb_kda_layer* w, uint32_t hidden,
                        const float* x_host, uint32_t tokens, uint16_t* conv_host,
                        float* recurrent_host, float* out_host);

/* official_kda with the state held on the device between calls
 * (OfficialKdaStateMode device_seed / device_continue / device_publish,
 * backend.hpp:242-259; the reference's CUDA backend_cuda.cu:2564-3140): the
 * positions of k3xb_kda_block_host as a chain from the state held in
 * `slot` of the context. SEED takes the state from conv_host/rec_host
 * (layouts as k3xb_kda_block_host) and holds the new one; CONTINUE runs
 * from the held state and holds the new one (conv_host/rec_host unused,
 * may be NULL); PUBLISH runs from the held state and also copies the new
 * one to conv_host/rec_host. A slot holds one state of one shape; CONTINUE
 * and PUBLISH on a slot without a state of this block's shape are
 * INVALID_STATE. The tokens and lifetime rules of the reference's modes are
 * the caller's (the ComputeBackend adapter keeps them). HOST x [tokens][H]
 * and out; returns after the results are on the host. */
#define K3XB_KDA_HELD_SLOTS 8
enum { K3XB_KDA_SEED = 0, K3XB_KDA_CONTINUE = 1, K3XB_KDA_PUBLISH = 2 };
int k3xb_kda_block_held(k3xb_ctx* ctx, const k3xb_kda_layer* w, uint32_t hidden,
                        const float* x_host, uint32_t tokens, uint32_t slot,
                        int32_t mode, uint16_t* conv_host, float* recurrent_host,
                        float* out_host);

/* prepare_official_moe_input (official_moe.cpp:156-209) and the layer's
 * input path (official_layer.cpp:159-172): attention_residual of the two
 * sources (official_layer.cpp:42-102), then rms_norm (:104-125) with
 * post_norm. With delta != NULL the first source is round_bf16(round_bf16(a)
 * + delta) (official_layer.cpp:190-193), written to prefix_out. Rows [T][H];
 * norm/proj/post_norm [H] bf16 words. */
int k3xb_attention_residual_norm(k3xb_ctx* ctx, const float* a,
                                 const float* delta, const float* block,
                                 const uint16_t* residual_norm,
                                 const uint16_t* residual_proj,
                                 const uint16_t* post_norm, uint32_t tokens,
                                 uint32_t hidden, float eps,
                                 float* prefix_out, float* out);

/* The block attention residual of the K3 token graph with many sources
 * (Engine::attention_residual, runtime/src/model.cpp:645-666; its torch form
 * reference/k3x_ref/attn_res.py:9-23). For each row t the values are the
 * S block sources in push order, then the prefix:
 *   key_d = rms_norm(value_d, norm, eps) (ops.cpp:10-18),
 *   score_d = key_d . projection, p = softmax over the S + 1 scores,
 *   out[t] = sum_d p_d * value_d[t], summed in depth order.
 * Device pointers: prefix, out [T][H]; sources [S][T][H] (depth-major, may
 * be NULL when S = 0, which gives out = prefix); norm, projection [H]
 * floats. S <= 63, hidden <= 49152; eps finite and >= 0. Scores are FP64
 * sums rounded once to float (the reference rounds each product and chains
 * float adds), so results agree with it to float tolerance, not bit for
 * bit. */
int k3xb_block_attention_residual(k3xb_ctx* ctx, const float* prefix,
                                  const float* sources, uint32_t sources_count,
                                  uint32_t tokens, uint32_t hidden,
                                  const float* norm, const float* projection,
                                  float eps, float* out);

/* prepare_official_moe_route (backend.hpp:384-389; the reference's CUDA
 * backend_cuda.cu:3478-3699) for one position: the MoE input
 * prepare_official_moe_input makes of (a, block), as
 * k3xb_attention_residual_norm, and its router logits (float of the FP64
 * sum in h order, bit-identical to route_official_moe_logits' input). With
 * delta (may be NULL) the first source is the prefix
 * round_bf16(round_bf16(a) + delta), also written to prefix_out; this is the
 * layer front's "prefix from the KDA output" (backend_cuda.cu:3342-3359).
 * router NULL: no logits (experts and logits_out unused), which with the
 * input norm in place of post_norm is the layer's KDA input preparation.
 * HOST a, delta, block, prefix_out, hidden_out [H] and logits_out [E];
 * norms, proj and router [E][H] are device bf16 words. Returns after the
 * results are on the host. */
int k3xb_prepare_moe_route_host(k3xb_ctx* ctx, const float* a,
                                const float* delta, const float* block,
                                uint32_t hidden, const uint16_t* residual_norm,
                                const uint16_t* residual_proj,
                                const uint16_t* post_norm, float eps,
                                const uint16_t* router, uint32_t experts,
                                float* prefix_out, float* hidden_out,
                                float* logits_out);

/* One KDA + MoE layer: official_layer_cpu (official_layer.cpp:134-244) with
 * the plain hidden-space MoE (official_moe.cpp:271-344 without the latent
 * steps :296, :323-331): out = round_bf16(round_bf16(prefix) +
 * round_bf16(routed + shared)). moe.hidden must equal hidden. */
typedef struct {
    uint32_t hidden;
    float rms_eps;
    const uint16_t* self_residual_norm;   /* [H] */
    const uint16_t* self_residual_proj;   /* [H] */
    const uint16_t* input_norm;           /* [H] */
    const uint16_t* moe_residual_norm;    /* [H] */
    const uint16_t* moe_residual_proj;    /* [H] */
    const uint16_t* post_norm;            /* [H] */
    k3xb_kda_layer kda;
    k3xb_moe_layer moe;
} k3xb_layer;

/* The layer over S sequences x N draft nodes (parent HOST, as above):
 * hidden_in and block_source [S][N][H] -> hidden_out [S][N][H]; KDA state
 * as k3xb_kda_block (unchanged; commit with k3xb_kda_block_commit and the
 * trace). expert_ids [S*N][top_k] may be NULL. */
int k3xb_layer_forward(k3xb_ctx* ctx, const k3xb_layer* layer,
                       const float* hidden_in, const float* block_source,
                       const int32_t* parent, uint32_t nodes,
                       uint32_t sequences, const uint16_t* conv,
                       const float* recurrent, float* hidden_out,
                       uint32_t* expert_ids, void* kda_trace);

/* ---- the verify step: layer stack + LM head + acceptance + commit -------- */
/* A stack of KDA + MoE layers with its LM head (model.cpp:376-386,
 * :456-459, :1174-1176). layer is a HOST array of `layers` descriptors that
 * share hidden, heads, head_dim and conv_width. embedding [V][H] bf16 may be
 * NULL (the caller passes embedded hidden states); final_norm [H] bf16 may
 * be NULL (no final RMSNorm); lm_head [V][H] bf16. */
typedef struct {
    uint32_t layers, vocab;
    const k3xb_layer* layer;
    const uint16_t* embedding;
    const uint16_t* final_norm;
    float final_eps;
    const uint16_t* lm_head;
} k3xb_verify_model;

enum { K3XB_ACCEPT_GREEDY = 0, K3XB_ACCEPT_REJECTION = 1 };

/* One call's device arrays. S sequences verify p linear drafts each; node 0
 * of a sequence is its anchor, node i its draft i. tokens [S][p+1] (anchor
 * then drafts; with an embedding), hidden_in [S][p+1][H] (without one),
 * block_source [S][p+1][H] (NULL: the embedded/given input), drafts [S][p].
 * conv [layers][S][3][w-1][P] and recurrent [layers][S][h][d][d] are the
 * per-layer KDA states, advanced IN PLACE to the last accepted position
 * (node accepted[s]). logits [S][p+1][V] (may be NULL) receives the
 * bf16-rounded LM-head logits. draft_logits [S][p][V], temperature, seed and
 * sequence_base are read for K3XB_ACCEPT_REJECTION. */
typedef struct {
    uint32_t sequences, drafts;
    const uint32_t* tokens;
    const float* hidden_in;
    const float* block_source;
    const uint32_t* draft_tokens;
    uint16_t* conv;
    float* recurrent;
    int32_t mode;
    const float* draft_logits;
    float temperature;
    uint64_t seed, sequence_base;
    float* logits;
    uint32_t* accepted;
    uint32_t* committed;
    uint32_t* committed_count;
} k3xb_verify_io;

/* Engine::forward_expert_major_block + verify_greedy_target_block +
 * commit (model.cpp:133-420, :1660-1664; speculative.cpp:74-112), or the
 * seeded rejection rule (no reference counterpart), as one device-side call:
 * no host synchronisation between the layers, the LM head, the acceptance
 * and the state commit. */
int k3xb_verify_step(k3xb_ctx* ctx, const k3xb_verify_model* model,
                     const k3xb_verify_io* io);

/* The AURORA reduced-Top-K self-draft on the device (the draft side of
 * AuroraPersistentDraftProvider, aurora.cpp:206-383, with the draft
 * session's fixed routing of K in {4, 6, 8, 12}, aurora.cpp:10-12): from
 * each sequence's committed KDA state, `drafts` greedy decode steps of the
 * same layer stack with every MoE layer's top_k replaced by draft_top_k.
 * Step i feeds the token step i-1 produced (step 0 the anchor) and its
 * argmax becomes draft i. The target's state arrays are read, not changed:
 * the draft runs on its own copy, so nothing needs rolling back after
 * verification (the job of IncrementalDraftCursor, model.cpp:1179-1409).
 * The model needs its embedding. Device arrays: anchors [S], conv
 * [layers][S][3][w-1][P], recurrent [layers][S][h][d][d] (as
 * k3xb_verify_io), draft_tokens [S][drafts]. */
typedef struct {
    uint32_t sequences, drafts, draft_top_k;
    const uint32_t* anchors;
    const uint16_t* conv;
    const float* recurrent;
    uint32_t* draft_tokens;
} k3xb_draft_io;
int k3xb_draft_greedy(k3xb_ctx* ctx, const k3xb_verify_model* model,
                      const k3xb_draft_io* io);

/* One speculative round with the drafter on the device (the propose /
 * verify / update loop of generate_speculative, model.cpp:1507, with
 * AuroraPersistentDraftProvider as the drafter): k3xb_draft_greedy from
 * the anchors and the committed state, then k3xb_verify_step (greedy) of
 * anchor + drafts with the full model, which advances the state to the
 * accepted position, then anchors <- each sequence's last committed token.
 * No host synchronisation inside: rounds can be queued back to back.
 * Device arrays: anchors [S] (in/out); conv, recurrent as k3xb_verify_io
 * (in/out); draft_tokens [S][p], accepted [S], committed [S][p+1],
 * committed_count [S] (out); logits [S][p+1][V] (out, may be NULL). */
typedef struct {
    uint32_t sequences, drafts, draft_top_k;
    uint32_t* anchors;
    uint16_t* conv;
    float* recurrent;
    uint32_t* draft_tokens;
    uint32_t* accepted;
    uint32_t* committed;
    uint32_t* committed_count;
    float* logits;
} k3xb_speculative_io;
int k3xb_speculative_step(k3xb_ctx* ctx, const k3xb_verify_model* model,
                          const k3xb_speculative_io* io);

/* ---- expert parallelism (peer memory over NVLink; NCCL for set-up) ---------- */
/* 128-byte NCCL unique id, made on one rank and handed to all (any
 * transport: a store, a file, a broadcast). No reference counterpart: the
 * reference runs one process on one GPU. */
int k3xb_ep_unique_id(uint8_t* unique_id);
/* Joins this context (its GPU) to a world of `world` ranks: a blocking
 * communicator with the default bound (k3xb_ep_init_config with NULL). */
int k3xb_ep_init(k3xb_ctx* ctx, const uint8_t* unique_id, int32_t rank,
                 int32_t world);
/* Failure detection. Every wait has a bound: on the host the stream drains
 * of k3xb_sync, of scratch and window growth, of k3xb_ep_finalize and of
 * k3xb_destroy, and (nonblocking = 1) communicator creation and each NCCL
 * launch; on the device each kernel's wait for the other ranks' exchange
 * flags (5 s). A bound that passes, or an error NCCL reports (a peer that
 * failed), aborts the exchange (its kernels in flight return); the call, or
 * the next k3xb_sync after a device wait gave up, returns
 * BACKEND_UNAVAILABLE with the reason in k3xb_last_error. The context's
 * one-GPU entry points keep working; the expert-parallel ones return
 * INVALID_STATE until k3xb_ep_finalize and a new init (with a new unique id
 * on every rank). A caller that synchronises the stream itself (e.g. with
 * torch) should call k3xb_sync or k3xb_ep_status instead, or it waits on
 * NCCL's kernels without a bound. */
#define K3XB_EP_DEFAULT_TIMEOUT_MS 300000u
typedef struct {
    uint32_t timeout_ms;    /* the bound; 0 = K3XB_EP_DEFAULT_TIMEOUT_MS */
    uint32_t nonblocking;   /* 1: NCCL nonblocking communicator (creation and
                               group launch polled under the bound) */
} k3xb_ep_config;
int k3xb_ep_init_config(k3xb_ctx* ctx, const uint8_t* unique_id, int32_t rank,
                        int32_t world, const k3xb_ep_config* config);
/* OK while the communicator is healthy (an error NCCL reported since the
 * last call aborts it here); INVALID_STATE when there is none or it was
 * aborted. Does not wait. */
int k3xb_ep_status(k3xb_ctx* ctx);
/* Ends the communicator at once, without its peers (ncclCommAbort): for a
 * rank that found on the host that a peer is gone (k3xb.peers.PeerWatch),
 * or that leaves while the others may not take part in a finalize. Then
 * k3xb_ep_finalize, and k3xb_ep_init with a new unique id to go on. */
int k3xb_ep_abort(k3xb_ctx* ctx);
/* Drains the stream (bounded), then frees the communicator. */
int k3xb_ep_finalize(k3xb_ctx* ctx);
/* The MoE layer of k3xb_moe_layer_forward with the routed experts sharded:
 * this rank holds experts [rank*E/world, (rank+1)*E/world) in `local` (or,
 * with local->ep_owner, the experts that table gives this rank)
 * (local->experts == E / world; router [E][H], correction [E] and the shared
 * expert are the full, replicated ones) and `tokens` tokens of its own
 * sequences, the same count on every rank. Each rank owns an exchange
 * window that the others map (CUDA IPC handles all-gathered over the
 * communicator at the first call, and again if a call needs a larger one):
 * a token's row goes only to the ranks that own one of its experts, and
 * the down projection stores each (token, slot) output row straight into
 * the token's rank's window; epoch flags with bounded waits order the
 * steps. The combine runs on the token's rank with the one-GPU arithmetic,
 * so out/ids/contributions equal the single-GPU layer's bit for bit. Every
 * rank calls it with the same shapes (a collective). MXF4 engine only; at
 * most 8 ranks. */
int k3xb_ep_moe_layer_forward(k3xb_ctx* ctx, const k3xb_moe_layer* local,
                              uint32_t experts_total, const float* hidden,
                              uint32_t tokens, float* out, uint32_t* ids,
                              float* contributions);

/* The verify step (k3xb_verify_step) over this rank's own sequences, with
 * every layer's MoE expert parallel: each layer descriptor's experts are
 * this rank's slice of experts_total (ranks hold equal slices in rank
 * order); router, correction, shared expert, KDA, norms, embedding and LM
 * head are whole on every rank. KDA, routing, the shared expert, the LM head
 * and acceptance run on the token's rank (data parallel over sequences); the
 * routed experts run on the rank that owns them, reached through the
 * exchange windows as in k3xb_ep_moe_layer_forward. Replaces the reference's
 * one-process Engine::forward_expert_major_block (model.cpp:133-420) for
 * one box of GPUs; every rank calls it with the same shapes (a collective). */
int k3xb_ep_verify_step(k3xb_ctx* ctx, const k3xb_verify_model* model,
                        const k3xb_verify_io* io, uint32_t experts_total);

/* An expert placement for k3xb_moe_layer.ep_owner (HOST arrays, no
 * context): experts dealt in descending order of `load` (any expected
 * per-expert work, e.g. routing counts or the routing bias) over `world`
 * ranks in a snake (ranks 0..world-1, then world-1..0, ...), so the
 * heaviest experts land on different ranks and every rank gets
 * experts / world of them. Ties keep the lower expert id first. owner[e] =
 * rank << 16 | index in that rank's stacks (ascending order of dealing).
 * No counterpart in the reference (one process, one GPU). */
int k3xb_ep_balance(const float* load, uint32_t experts, uint32_t world, uint32_t* owner);

/* ---- (e) acceptance ------------------------------------------------------- */
/* verify_greedy_target_block (runtime/src/speculative.cpp:74-112) for S
 * sequences of p drafts: targets = first-max argmax of logits
 * [S][p+1][V] (model.cpp:1174-1176); accepted [S], committed [S][p+1],
 * committed_count [S], targets [S][p+1] (may be NULL). */
int k3xb_accept_greedy(k3xb_ctx* ctx, const float* logits,
                       const uint32_t* drafts, uint32_t sequences,
                       uint32_t drafts_per_sequence, uint32_t vocab,
                       uint32_t* targets, uint32_t* accepted,
                       uint32_t* committed, uint32_t* committed_count);
/* Seeded speculative rejection sampling (no reference counterpart): accept
 * draft i if u_i * q_i(d_i) < p_i(d_i) (softmax at `temperature`, FP64);
 * at the first rejection sample norm(max(0, p - q)), else a bonus from p.
 * Canonical FP64 reduction order and RNG are those of oracle/k3x_oracle.c.
 * draft_logits [S][p][V]. */
int k3xb_accept_rejection(k3xb_ctx* ctx, const float* target_logits,
                          const float* draft_logits, const uint32_t* drafts,
                          uint32_t sequences, uint32_t drafts_per_sequence,
                          uint32_t vocab, float temperature, uint64_t seed,
                          uint64_t sequence_base, uint32_t* accepted,
                          uint32_t* committed, uint32_t* committed_count);

/* ---- synthetic data and MXFP4 preparation -------------------------------- */
/* N(mean, sigma) from a counter-based generator (SplitMix64 + Box-Muller),
 * deterministic in (seed, stream, index). */
int k3xb_fill_normal_f32(k3xb_ctx* ctx, float* out, size_t count,
                         uint64_t seed, uint64_t stream, float mean,
                         float sigma);
/* Same values rounded to bf16 (as float values or as bf16 words). */
int k3xb_fill_normal_bf16(k3xb_ctx* ctx, uint16_t* out, size_t count,
                          uint64_t seed, uint64_t stream, float sigma);
/* MXFP4 quantiser (no reference counterpart; the reference only decodes):
 * per 32-block s = smallest integer with amax <= 6*2^s, E2M1 codes by
 * round-to-nearest-even. x [rows][cols] float, cols % 32 == 0. */
int k3xb_quantize_mxfp4(k3xb_ctx* ctx, const float* x, size_t rows,
                        size_t cols, uint8_t* packed, uint8_t* scales);
/* Generates N(0, sigma) weights and quantises them without a float copy. */
int k3xb_fill_normal_mxfp4(k3xb_ctx* ctx, uint8_t* packed, uint8_t* scales,
                           size_t rows, size_t cols, uint64_t seed,
                           uint64_t stream, float sigma);

#ifdef __cplusplus
}
#endif
#endif
