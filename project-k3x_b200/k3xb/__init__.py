"""Python binding of libk3xb (include/k3xb.h) over ctypes.

Device arrays are passed as torch CUDA tensors (torch supplies memory and
streams; all compute is in libk3xb.so). There is no CPU fallback: if the
library or a B200 is missing, every entry point raises K3xbError.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libk3xb.so")

OK = 0
INVALID_EXTENT = 9
INVALID_MXFP4 = 15
INVALID_STATE = 16
BACKEND_UNAVAILABLE = 17
UNSUPPORTED_ARCHITECTURE = 19

ACT_SWIGLU = 0
ACT_SITU = 1
ENGINE_MXF4 = 0
ENGINE_SIMT = 1

STATUS_NAMES = {0: "OK", 9: "INVALID_EXTENT", 15: "INVALID_MXFP4", 16: "INVALID_STATE",
                17: "BACKEND_UNAVAILABLE", 19: "UNSUPPORTED_ARCHITECTURE"}


class K3xbError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class Plan(C.Structure):
    _fields_ = [("group_expert", C.c_void_p), ("group_offset", C.c_void_p),
                ("assign_token", C.c_void_p), ("assign_slot", C.c_void_p),
                ("assign_contrib", C.c_void_p), ("group_count", C.c_void_p),
                ("status", C.c_void_p)]


class MoeLayer(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("inter", C.c_uint32), ("experts", C.c_uint32),
                ("top_k", C.c_uint32), ("shared_inter", C.c_uint32),
                ("router", C.c_void_p), ("correction", C.c_void_p),
                ("gate_packed", C.c_void_p), ("gate_scales", C.c_void_p),
                ("up_packed", C.c_void_p), ("up_scales", C.c_void_p),
                ("down_packed", C.c_void_p), ("down_scales", C.c_void_p),
                ("shared_gate", C.c_void_p), ("shared_up", C.c_void_p), ("shared_down", C.c_void_p),
                ("activation", C.c_int32), ("situ_beta", C.c_float),
                ("situ_linear_beta", C.c_float), ("engine", C.c_int32), ("act_terms", C.c_int32),
                ("gate_scales_tc", C.c_void_p), ("up_scales_tc", C.c_void_p),
                ("down_scales_tc", C.c_void_p),
                ("latent", C.c_uint32), ("routed_down", C.c_void_p), ("routed_norm", C.c_void_p),
                ("routed_up", C.c_void_p), ("latent_eps", C.c_float), ("ep_owner", C.c_void_p)]


class KdaLayer(C.Structure):
    _fields_ = [("heads", C.c_uint32), ("head_dim", C.c_uint32), ("conv_width", C.c_uint32),
                ("eps", C.c_float), ("gate_lower_bound", C.c_float)] + [
        (n, C.c_void_p) for n in ("q_proj", "k_proj", "v_proj", "q_conv", "k_conv", "v_conv", "f_a_proj",
                                  "f_b_proj", "a_log", "dt_bias", "b_proj", "g_proj", "o_norm", "o_proj")]


class Layer(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("rms_eps", C.c_float)] + [
        (n, C.c_void_p) for n in ("self_residual_norm", "self_residual_proj", "input_norm",
                                  "moe_residual_norm", "moe_residual_proj", "post_norm")] + [
        ("kda", KdaLayer), ("moe", MoeLayer)]


class VerifyModel(C.Structure):
    _fields_ = [("layers", C.c_uint32), ("vocab", C.c_uint32), ("layer", C.POINTER(Layer)),
                ("embedding", C.c_void_p), ("final_norm", C.c_void_p), ("final_eps", C.c_float),
                ("lm_head", C.c_void_p)]


class VerifyIO(C.Structure):
    _fields_ = [("sequences", C.c_uint32), ("drafts", C.c_uint32)] + [
        (n, C.c_void_p) for n in ("tokens", "hidden_in", "block_source", "draft_tokens", "conv", "recurrent")] + [
        ("mode", C.c_int32), ("draft_logits", C.c_void_p), ("temperature", C.c_float),
        ("seed", C.c_uint64), ("sequence_base", C.c_uint64)] + [
        (n, C.c_void_p) for n in ("logits", "accepted", "committed", "committed_count")]


class DraftIO(C.Structure):
    _fields_ = [("sequences", C.c_uint32), ("drafts", C.c_uint32), ("draft_top_k", C.c_uint32)] + [
        (n, C.c_void_p) for n in ("anchors", "conv", "recurrent", "draft_tokens")]


class SpeculativeIO(C.Structure):
    _fields_ = [("sequences", C.c_uint32), ("drafts", C.c_uint32), ("draft_top_k", C.c_uint32)] + [
        (n, C.c_void_p) for n in ("anchors", "conv", "recurrent", "draft_tokens", "accepted", "committed",
                                  "committed_count", "logits")]


KDA_SEED, KDA_CONTINUE, KDA_PUBLISH = 0, 1, 2   # k3xb_kda_block_held modes
KDA_HELD_SLOTS = 8

EP_DEFAULT_TIMEOUT_MS = 300000


class EpConfig(C.Structure):
    _fields_ = [("timeout_ms", C.c_uint32), ("nonblocking", C.c_uint32)]


class RoutingPolicy(C.Structure):
    _fields_ = [("mode", C.c_int32), ("fixed_k", C.c_uint32), ("mass_target", C.c_float),
                ("minimum_gap", C.c_float), ("quality_floor_k", C.c_uint32)]


ROUTING_NATURAL, ROUTING_FIXED, ROUTING_ADAPTIVE = 0, 1, 2


class Stats(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in (
        "kernel_launches", "route_calls", "moe_layer_calls", "moe_layer_experts", "kda_calls",
        "accept_calls", "scratch_bytes", "peak_scratch_bytes", "h2d_bytes", "d2h_bytes",
        "weight_cache_hits", "weight_cache_misses", "weight_cache_bypasses", "resident_weight_bytes",
        "peak_resident_weight_bytes", "weight_h2d_bytes")]


PHASE_COUNT = 20   # K3XB_PHASE_COUNT


class PhaseTime(C.Structure):
    _fields_ = [("device_ms", C.c_double), ("calls", C.c_uint64)]


WEIGHT_F32, WEIGHT_BF16, WEIGHT_MXFP4, WEIGHT_EXPERT_STACK = 0, 1, 2, 3
RESIDENT_HIT, RESIDENT_ADMITTED, RESIDENT_BYPASS = 0, 1, 2


class Resident(C.Structure):
    _fields_ = [("disposition", C.c_int32), ("primary", C.c_void_p), ("secondary", C.c_void_p),
                ("scales_tc", C.c_void_p), ("uploaded_bytes", C.c_uint64)]


class ExpertHost(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("gate_packed", "gate_scales", "up_packed", "up_scales",
                                          "down_packed", "down_scales")]


class ResidentStack(C.Structure):
    _fields_ = [("disposition", C.c_int32)] + [(n, C.c_void_p) for n in (
        "gate_packed", "gate_scales", "up_packed", "up_scales", "down_packed", "down_scales",
        "gate_scales_tc", "up_scales_tc", "down_scales_tc")] + [("uploaded_bytes", C.c_uint64)]


_lib = None


def library() -> C.CDLL:
    """Loads libk3xb.so; raises if it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise K3xbError(BACKEND_UNAVAILABLE, f"{LIB_PATH} is missing: run project-k3x_b200/build.py")
        lib = C.CDLL(LIB_PATH)
        vp, u32, u64, sz, f32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_size_t, C.c_float
        sigs = {
            "k3xb_create": [C.c_int, C.POINTER(vp)],
            "k3xb_destroy": [vp],
            "k3xb_last_error": [vp, C.c_char_p, sz],
            "k3xb_set_stream": [vp, vp],
            "k3xb_sync": [vp],
            "k3xb_get_stats": [vp, C.POINTER(Stats)],
            "k3xb_route": [vp, vp, u32, u32, vp, vp, u32, u32, vp, vp, vp],
            "k3xb_router_logits": [vp, vp, u32, u32, vp, u32, vp],
            "k3xb_ep_balance": [vp, u32, u32, vp],
            "k3xb_expert_major_plan": [vp, vp, vp, u32, u32, u32, C.POINTER(Plan)],
            "k3xb_select_routing": [vp, vp, u32, u32, vp, u32, C.POINTER(RoutingPolicy), vp, vp, vp, vp, vp],
            "k3xb_moe_layer_forward": [vp, C.POINTER(MoeLayer), vp, u32, vp, vp, vp],
            "k3xb_moe_layer_forward_host": [vp, C.POINTER(MoeLayer), vp, u32, vp, vp, vp],
            "k3xb_moe_experts": [vp, C.POINTER(MoeLayer), vp, u32, C.POINTER(Plan), vp],
            "k3xb_kda_tree": [vp, vp, vp, u32, u32, u32, u32, vp, vp, vp, vp, vp, vp],
            "k3xb_kda_commit": [vp, vp, vp, u32, u32, u32, u32, vp, vp, vp, vp, vp, vp, vp],
            "k3xb_accept_greedy": [vp, vp, vp, u32, u32, u32, vp, vp, vp, vp],
            "k3xb_accept_rejection": [vp, vp, vp, vp, u32, u32, u32, f32, u64, u64, vp, vp, vp],
            "k3xb_fill_normal_f32": [vp, vp, sz, u64, u64, f32, f32],
            "k3xb_fill_normal_bf16": [vp, vp, sz, u64, u64, f32],
            "k3xb_quantize_mxfp4": [vp, vp, sz, sz, vp, vp],
            "k3xb_fill_normal_mxfp4": [vp, vp, vp, sz, sz, u64, u64, f32],
            "k3xb_prepare_mxfp4_scales": [vp, vp, sz, sz, vp],
            "k3xb_linear_bf16": [vp, vp, u32, u32, vp, u32, C.c_int32, vp],
            "k3xb_kda_block": [vp, C.POINTER(KdaLayer), u32, vp, vp, u32, u32, vp, vp, vp, vp],
            "k3xb_kda_block_commit": [vp, C.POINTER(KdaLayer), vp, vp, u32, u32, vp, vp, vp, vp, vp],
            "k3xb_attention_residual_norm": [vp, vp, vp, vp, vp, vp, vp, u32, u32, f32, vp, vp],
            "k3xb_block_attention_residual": [vp, vp, vp, u32, u32, u32, vp, vp, f32, vp],
            "k3xb_layer_forward": [vp, C.POINTER(Layer), vp, vp, vp, u32, u32, vp, vp, vp, vp, vp],
            "k3xb_verify_step": [vp, C.POINTER(VerifyModel), C.POINTER(VerifyIO)],
            "k3xb_ep_verify_step": [vp, C.POINTER(VerifyModel), C.POINTER(VerifyIO), u32],
            "k3xb_draft_greedy": [vp, C.POINTER(VerifyModel), C.POINTER(DraftIO)],
            "k3xb_speculative_step": [vp, C.POINTER(VerifyModel), C.POINTER(SpeculativeIO)],
            "k3xb_ep_unique_id": [vp],
            "k3xb_ep_init": [vp, vp, C.c_int32, C.c_int32],
            "k3xb_ep_init_config": [vp, vp, C.c_int32, C.c_int32, C.POINTER(EpConfig)],
            "k3xb_ep_status": [vp],
            "k3xb_ep_abort": [vp],
            "k3xb_ep_finalize": [vp],
            "k3xb_ep_moe_layer_forward": [vp, C.POINTER(MoeLayer), u32, vp, u32, vp, vp, vp],
            "k3xb_set_resident_capacity": [vp, u64],
            "k3xb_acquire_weight": [vp, u64, C.c_int32, u64, u64, u64, vp, sz, vp, sz, C.POINTER(Resident)],
            "k3xb_acquire_expert_stack": [vp, u64, u32, u32, u32, C.POINTER(ExpertHost),
                                          C.POINTER(ResidentStack)],
            "k3xb_release_resident": [vp],
            "k3xb_expert_grid_host": [vp, C.POINTER(MoeLayer), vp, u32, vp, u32, vp],
            "k3xb_official_moe_ffn_host": [vp, C.POINTER(MoeLayer), C.POINTER(MoeLayer), u32, vp, vp, vp, vp],
            "k3xb_set_profiling": [vp, C.c_int],
            "k3xb_get_profile": [vp, C.POINTER(PhaseTime), C.POINTER(u64)],
            "k3xb_kda_block_host": [vp, C.POINTER(KdaLayer), u32, vp, u32, vp, vp, vp],
            "k3xb_dense_matvec": [vp, vp, u32, u32, vp, u32, vp],
            "k3xb_mxfp4_matvec": [vp, vp, vp, u32, u32, vp, u32, vp],
            "k3xb_prepare_moe_route_host": [vp, vp, vp, vp, u32, vp, vp, vp, C.c_float, vp, u32, vp, vp, vp],
            "k3xb_mxfp4_matvec_host": [vp, vp, vp, u32, u32, vp, vp],
            "k3xb_resident_moe_layer_host": [vp, u32, u32, u32, u32] + [vp] * 6 + [vp, u32, vp, C.c_float, C.c_float,
                                                                                    C.c_float, vp, vp],
            "k3xb_dense_matvec_host": [vp, vp, u32, u32, vp, vp],
            "k3xb_dense_situ_mlp_host": [vp, vp, vp, vp, u32, u32, u32, vp, C.c_float, C.c_float, vp],
            "k3xb_kda_block_held": [vp, C.POINTER(KdaLayer), u32, vp, u32, u32, C.c_int32, vp, vp, vp],
        }
        for name, args in sigs.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = C.c_int
        lib.k3xb_kda_trace_bytes.argtypes = [C.POINTER(KdaLayer), u32, u32]
        lib.k3xb_kda_trace_bytes.restype = sz
        lib.k3xb_default_act_terms.argtypes = [u64, u32]
        lib.k3xb_default_act_terms.restype = u32
        lib.k3xb_phase_name.argtypes = [C.c_int]
        lib.k3xb_phase_name.restype = C.c_char_p
        _lib = lib
    return _lib


def _p(t):
    """Device pointer of a torch tensor (None -> NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise K3xbError(INVALID_EXTENT, "expected a CUDA tensor")
    if not t.is_contiguous():
        raise K3xbError(INVALID_EXTENT, "expected a contiguous tensor")
    return C.c_void_p(t.data_ptr())


class Context:
    """One k3xb context per GPU; calls run on torch's current stream unless
    `stream` is given."""

    def __init__(self, device: int = 0):
        self.lib = library()
        h = C.c_void_p()
        st = self.lib.k3xb_create(device, C.byref(h))
        if st != OK:
            raise K3xbError(st, f"k3xb_create(device={device})")
        self.h = h
        self.device = device

    def close(self):
        if getattr(self, "h", None):
            self.lib.k3xb_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, st, where):
        if st != OK:
            buf = C.create_string_buffer(512)
            self.lib.k3xb_last_error(self.h, buf, 512)
            raise K3xbError(st, f"{where}: {buf.value.decode(errors='replace')}")

    def use_stream(self, stream=None):
        """Binds a torch.cuda.Stream (default: torch's current stream)."""
        import torch
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        # torch's default stream has handle 0, which the C ABI reads as "the
        # context's own stream"; pass cudaStreamLegacy (0x1) so work stays
        # ordered with torch's default-stream work.
        handle = s.cuda_stream if s.cuda_stream else 0x1
        self._check(self.lib.k3xb_set_stream(self.h, C.c_void_p(handle)), "set_stream")

    def sync(self):
        self._check(self.lib.k3xb_sync(self.h), "sync")

    def stats(self) -> dict:
        s = Stats()
        self._check(self.lib.k3xb_get_stats(self.h, C.byref(s)), "stats")
        return {n: getattr(s, n) for n, _ in Stats._fields_}

    # ---- (a) ------------------------------------------------------------------
    def route(self, hidden, router, correction, top_k, ids, contrib, scores=None):
        T, H = hidden.shape
        E = router.shape[0]
        self._check(self.lib.k3xb_route(self.h, _p(hidden), T, H, _p(router), _p(correction), E, top_k,
                                        _p(ids), _p(contrib), _p(scores)), "route")

    def router_logits(self, hidden, router, logits):
        T, H = hidden.shape
        self._check(self.lib.k3xb_router_logits(self.h, _p(hidden), T, H, _p(router), router.shape[0],
                                                _p(logits)), "router_logits")

    def expert_major_plan(self, ids, contrib, experts, plan: dict):
        T, K = ids.shape
        pl = Plan(*(_p(plan[k]) for k in ("group_expert", "group_offset", "assign_token", "assign_slot",
                                          "assign_contrib", "group_count", "status")))
        self._check(self.lib.k3xb_expert_major_plan(self.h, _p(ids), _p(contrib), T, K, experts,
                                                    C.byref(pl)), "expert_major_plan")

    # ---- (b)+(c) ----------------------------------------------------------------
    def moe_layer_forward(self, layer: MoeLayer, hidden, out, ids=None, contrib=None):
        self._check(self.lib.k3xb_moe_layer_forward(self.h, C.byref(layer), _p(hidden), hidden.shape[0],
                                                    _p(out), _p(ids), _p(contrib)), "moe_layer_forward")

    def moe_layer_forward_host(self, layer: MoeLayer, hidden, out, ids=None, contrib=None):
        """hidden/out/ids/contrib are CPU tensors (pinned for async copies)."""
        ptr = lambda t: None if t is None else C.c_void_p(t.data_ptr())
        self._check(self.lib.k3xb_moe_layer_forward_host(self.h, C.byref(layer), ptr(hidden),
                                                         hidden.shape[0], ptr(out), ptr(ids),
                                                         ptr(contrib)), "moe_layer_forward_host")

    # ---- (d) --------------------------------------------------------------------
    def kda_tree(self, state, parent, q, k, v, log_decay, beta, out):
        S, N = q.shape[0], q.shape[1]
        heads, d = state.shape[1], state.shape[2]
        par = (C.c_int32 * N)(*[int(x) for x in parent])
        self._check(self.lib.k3xb_kda_tree(self.h, _p(state), par, N, S, heads, d, _p(q), _p(k), _p(v),
                                           _p(log_decay), _p(beta), _p(out)), "kda_tree")

    def kda_commit(self, state, parent, q, k, v, log_decay, beta, commit_node, state_out):
        S, N = q.shape[0], q.shape[1]
        heads, d = state.shape[1], state.shape[2]
        par = (C.c_int32 * N)(*[int(x) for x in parent])
        com = (C.c_int32 * S)(*[int(x) for x in commit_node])
        self._check(self.lib.k3xb_kda_commit(self.h, _p(state), par, N, S, heads, d, _p(q), _p(k), _p(v),
                                             _p(log_decay), _p(beta), com, _p(state_out)), "kda_commit")

    def select_routing(self, scores, bias, natural_k, ids, weights, selected, escalated=None, stats=None,
                       mode=ROUTING_NATURAL, fixed_k=0, mass_target=0.9, minimum_gap=0.0, quality_floor_k=0):
        """select_routing (routing_policy.cpp:31-159) for scores [T][E]."""
        T, E = scores.shape
        pol = RoutingPolicy(mode, fixed_k, mass_target, minimum_gap, quality_floor_k)
        self._check(self.lib.k3xb_select_routing(self.h, _p(scores), T, E, _p(bias), natural_k, C.byref(pol),
                                                 _p(ids), _p(weights), _p(selected), _p(escalated), _p(stats)),
                    "select_routing")

    # ---- full KDA block and the layer ----------------------------------------
    def kda_trace_bytes(self, kda: "KdaLayer", nodes, sequences):
        return self.lib.k3xb_kda_trace_bytes(C.byref(kda), nodes, sequences)

    def kda_block(self, kda: "KdaLayer", x, parent, conv, recurrent, out, trace=None):
        """x/out [S][N][H]; conv [S][3][w-1][P] int16 (bf16 words); recurrent [S][h][d][d]."""
        S, N, H = x.shape
        par = (C.c_int32 * N)(*[int(v) for v in parent])
        self._check(self.lib.k3xb_kda_block(self.h, C.byref(kda), H, _p(x), par, N, S, _p(conv), _p(recurrent),
                                            _p(out), _p(trace)), "kda_block")

    def kda_block_commit(self, kda: "KdaLayer", trace, parent, sequences, commit_node, conv, recurrent,
                         conv_out, recurrent_out):
        N = len(parent)
        par = (C.c_int32 * N)(*[int(v) for v in parent])
        com = (C.c_int32 * sequences)(*[int(v) for v in commit_node])
        self._check(self.lib.k3xb_kda_block_commit(self.h, C.byref(kda), _p(trace), par, N, sequences, com,
                                                   _p(conv), _p(recurrent), _p(conv_out), _p(recurrent_out)),
                    "kda_block_commit")

    def attention_residual_norm(self, a, block, norm, proj, post, eps, out, delta=None, prefix_out=None):
        T, H = a.shape
        self._check(self.lib.k3xb_attention_residual_norm(self.h, _p(a), _p(delta), _p(block), _p(norm), _p(proj),
                                                          _p(post), T, H, eps, _p(prefix_out), _p(out)),
                    "attention_residual_norm")

    def block_attention_residual(self, prefix, sources, norm, proj, eps, out):
        """Depth attention over the block sources [S][T][H] (S may be 0:
        sources None) and the prefix [T][H] (model.cpp:645-666)."""
        T, H = prefix.shape
        S = 0 if sources is None else sources.shape[0]
        self._check(self.lib.k3xb_block_attention_residual(self.h, _p(prefix), _p(sources), S, T, H, _p(norm),
                                                           _p(proj), eps, _p(out)), "block_attention_residual")

    def layer_forward(self, layer: "Layer", hidden_in, block, parent, conv, recurrent, hidden_out,
                      expert_ids=None, trace=None):
        S, N, H = hidden_in.shape
        par = (C.c_int32 * N)(*[int(v) for v in parent])
        self._check(self.lib.k3xb_layer_forward(self.h, C.byref(layer), _p(hidden_in), _p(block), par, N, S,
                                                _p(conv), _p(recurrent), _p(hidden_out), _p(expert_ids),
                                                _p(trace)), "layer_forward")

    # ---- expert parallelism ------------------------------------------------
    def ep_init(self, unique_id: bytes, rank: int, world: int, timeout_ms: int = 0, nonblocking: bool = False):
        """Joins a world of `world` ranks. Every wait on the communicator is
        bounded by timeout_ms (0: EP_DEFAULT_TIMEOUT_MS); past it, or on an
        error NCCL reports, the communicator is aborted and the call raises
        (BACKEND_UNAVAILABLE), later expert-parallel calls raise
        INVALID_STATE until ep_finalize and a new ep_init."""
        buf = (C.c_uint8 * 128).from_buffer_copy(unique_id)
        cfg = EpConfig(timeout_ms, 1 if nonblocking else 0)
        self._check(self.lib.k3xb_ep_init_config(self.h, buf, rank, world, C.byref(cfg)), "ep_init")

    def ep_abort(self):
        """Ends the communicator without its peers (one is known to be gone)."""
        self._check(self.lib.k3xb_ep_abort(self.h), "ep_abort")

    def ep_status(self):
        """Raises if the communicator is gone or NCCL has reported a failure
        (which aborts it); does not wait."""
        self._check(self.lib.k3xb_ep_status(self.h), "ep_status")

    def ep_finalize(self):
        self._check(self.lib.k3xb_ep_finalize(self.h), "ep_finalize")

    def ep_moe_layer_forward(self, local: "MoeLayer", experts_total, hidden, out, ids=None, contrib=None):
        self._check(self.lib.k3xb_ep_moe_layer_forward(self.h, C.byref(local), experts_total, _p(hidden),
                                                       hidden.shape[0], _p(out), _p(ids), _p(contrib)),
                    "ep_moe_layer_forward")

    def verify_step(self, model: "VerifyModel", io: "VerifyIO"):
        self._check(self.lib.k3xb_verify_step(self.h, C.byref(model), C.byref(io)), "verify_step")

    def ep_verify_step(self, model: "VerifyModel", io: "VerifyIO", experts_total: int):
        """The verify step over this rank's sequences with every MoE layer
        expert parallel (each layer descriptor holds this rank's expert slice,
        ep_local_layer); needs ep_init first."""
        self._check(self.lib.k3xb_ep_verify_step(self.h, C.byref(model), C.byref(io), experts_total),
                    "ep_verify_step")

    def draft_greedy(self, model: "VerifyModel", anchors, conv, recurrent, draft_tokens, draft_top_k):
        """AURORA reduced-Top-K self-draft: draft_tokens [S][p] (device int32)
        from anchors [S] and the committed states (read, not changed)."""
        S, p = draft_tokens.shape
        io = DraftIO(S, p, draft_top_k, _p(anchors), _p(conv), _p(recurrent), _p(draft_tokens))
        self._check(self.lib.k3xb_draft_greedy(self.h, C.byref(model), C.byref(io)), "draft_greedy")

    def speculative_step(self, model: "VerifyModel", anchors, conv, recurrent, draft_tokens, accepted, committed,
                         committed_count, draft_top_k, logits=None):
        """One on-device round: draft, verify, advance the state, anchors <-
        last committed tokens (all device tensors)."""
        S, p = draft_tokens.shape
        io = SpeculativeIO(S, p, draft_top_k, _p(anchors), _p(conv), _p(recurrent), _p(draft_tokens), _p(accepted),
                           _p(committed), _p(committed_count), _p(logits))
        self._check(self.lib.k3xb_speculative_step(self.h, C.byref(model), C.byref(io)), "speculative_step")

    # ---- (e) --------------------------------------------------------------------
    def accept_greedy(self, logits, drafts, accepted, committed, count, targets=None):
        S, P1, V = logits.shape
        self._check(self.lib.k3xb_accept_greedy(self.h, _p(logits), _p(drafts), S, P1 - 1, V, _p(targets),
                                                _p(accepted), _p(committed), _p(count)), "accept_greedy")

    def accept_rejection(self, target_logits, draft_logits, drafts, temperature, seed, seq_base,
                         accepted, committed, count):
        S, P1, V = target_logits.shape
        self._check(self.lib.k3xb_accept_rejection(self.h, _p(target_logits), _p(draft_logits), _p(drafts),
                                                   S, P1 - 1, V, temperature, seed, seq_base,
                                                   _p(accepted), _p(committed), _p(count)),
                    "accept_rejection")

    # ---- synthetic ----------------------------------------------------------------
    def fill_normal_f32(self, out, seed, stream, mean=0.0, sigma=1.0):
        self._check(self.lib.k3xb_fill_normal_f32(self.h, _p(out), out.numel(), seed, stream, mean, sigma),
                    "fill_normal_f32")

    def fill_normal_bf16(self, out, seed, stream, sigma=1.0):
        self._check(self.lib.k3xb_fill_normal_bf16(self.h, _p(out), out.numel(), seed, stream, sigma),
                    "fill_normal_bf16")

    def quantize_mxfp4(self, x, packed, scales):
        rows, cols = x.shape
        self._check(self.lib.k3xb_quantize_mxfp4(self.h, _p(x), rows, cols, _p(packed), _p(scales)),
                    "quantize_mxfp4")

    def linear_bf16(self, x, weight, out, round_output=True):
        """out[T][rows] = (round_bf16)(weight[rows][K] . x[T][K]) on kind::f16."""
        T, K = x.shape
        rows = weight.shape[0]
        self._check(self.lib.k3xb_linear_bf16(self.h, _p(x), T, K, _p(weight), rows,
                                              1 if round_output else 0, _p(out)), "linear_bf16")

    def prepare_mxfp4_scales(self, scales, rows, cols, out):
        self._check(self.lib.k3xb_prepare_mxfp4_scales(self.h, _p(scales), rows, cols, _p(out)),
                    "prepare_mxfp4_scales")

    # ---- phase profile ----------------------------------------------------------
    def set_profiling(self, on: bool):
        """Starts (or stops) per-phase device timing; clears the totals."""
        self._check(self.lib.k3xb_set_profiling(self.h, 1 if on else 0), "set_profiling")

    def profile(self) -> dict:
        """{phase name: (device ms summed, calls)} for phases that ran, and
        "dropped": phases not timed."""
        arr = (PhaseTime * PHASE_COUNT)()
        dropped = C.c_uint64()
        self._check(self.lib.k3xb_get_profile(self.h, arr, C.byref(dropped)), "get_profile")
        out = {phase_name(i): (arr[i].device_ms, arr[i].calls) for i in range(PHASE_COUNT) if arr[i].calls}
        out["dropped"] = dropped.value
        return out

    # ---- resident weights (host arrays -> device copies keyed by tensor id) ----
    def set_resident_capacity(self, nbytes: int):
        self._check(self.lib.k3xb_set_resident_capacity(self.h, nbytes), "set_resident_capacity")

    def acquire_weight(self, tensor_id, representation, rows, cols, group_size, primary, secondary=None):
        """primary / secondary are HOST numpy arrays; returns a Resident."""
        import numpy as np
        primary = np.ascontiguousarray(primary)
        sec = None if secondary is None else np.ascontiguousarray(secondary)
        out = Resident()
        self._check(self.lib.k3xb_acquire_weight(
            self.h, tensor_id, representation, rows, cols, group_size, primary.ctypes.data, primary.nbytes,
            None if sec is None else sec.ctypes.data, 0 if sec is None else sec.nbytes, C.byref(out)),
            "acquire_weight")
        return out

    def acquire_expert_stack(self, stack_id, hidden, inter, experts):
        """experts: list of dicts of HOST uint8 arrays (gate_packed, gate_scales,
        up_packed, up_scales, down_packed, down_scales). Returns a ResidentStack."""
        import numpy as np
        keep = [{k: np.ascontiguousarray(v) for k, v in e.items()} for e in experts]
        views = (ExpertHost * len(keep))()
        for i, e in enumerate(keep):
            for name, _ in ExpertHost._fields_:
                setattr(views[i], name, e[name].ctypes.data)
        out = ResidentStack()
        self._check(self.lib.k3xb_acquire_expert_stack(self.h, stack_id, len(keep), hidden, inter, views,
                                                       C.byref(out)), "acquire_expert_stack")
        return out

    def expert_grid_host(self, layer: MoeLayer, expert_ids, inputs):
        """HOST inputs [T][H] float32 through each listed expert of the
        layer's stack -> HOST [n][T][H] (k3xb_expert_grid_host)."""
        import numpy as np
        x = np.ascontiguousarray(inputs, dtype=np.float32)
        ids = np.ascontiguousarray(expert_ids, dtype=np.uint32)
        out = np.empty((ids.size, x.shape[0], layer.hidden), np.float32)
        self._check(self.lib.k3xb_expert_grid_host(self.h, C.byref(layer), ids.ctypes.data, ids.size,
                                                   x.ctypes.data, x.shape[0], out.ctypes.data),
                    "expert_grid_host")
        return out

    def kda_block_host(self, w: KdaLayer, hidden, x, conv, recurrent):
        """One sequence through the KDA block with HOST arrays: x [T][H]
        float32 -> out [T][H]; conv [3][w-1][P] uint16 and recurrent
        [h][d][d] float32 are replaced by the state after the last position."""
        import numpy as np
        x = np.ascontiguousarray(x, dtype=np.float32)
        for a, dt in ((conv, np.uint16), (recurrent, np.float32)):
            if a.dtype != dt or not a.flags.c_contiguous:
                raise K3xbError(INVALID_EXTENT, "conv must be contiguous uint16 and recurrent float32")
        out = np.empty((x.shape[0], hidden), np.float32)
        self._check(self.lib.k3xb_kda_block_host(self.h, C.byref(w), hidden, x.ctypes.data, x.shape[0],
                                                 conv.ctypes.data, recurrent.ctypes.data, out.ctypes.data),
                    "kda_block_host")
        return out

    def dense_matvec(self, W, x, y):
        """y [T][rows] = W [rows][cols] x [T][cols] (device float32 tensors),
        the reference CPU backend's FP64 column-order sums."""
        rows, cols = W.shape
        self._check(self.lib.k3xb_dense_matvec(self.h, _p(W), rows, cols, _p(x), x.shape[0], _p(y)), "dense_matvec")

    def prepare_moe_route_host(self, a, block, norm, proj, post, eps, router=None, delta=None):
        """k3xb_prepare_moe_route_host: HOST a, block (and delta) [H]; device
        bf16 norm/proj/post [H] and router [E][H] (or None) -> HOST (prefix or
        None, prepared input [H], logits [E] or None)."""
        import numpy as np
        a = np.ascontiguousarray(a, dtype=np.float32)
        block = np.ascontiguousarray(block, dtype=np.float32)
        H = a.shape[0]
        E = router.shape[0] if router is not None else 0
        d = None if delta is None else np.ascontiguousarray(delta, dtype=np.float32)
        prefix = np.empty(H, np.float32) if d is not None else None
        hidden = np.empty(H, np.float32)
        logits = np.empty(E, np.float32) if E else None
        self._check(self.lib.k3xb_prepare_moe_route_host(
            self.h, a.ctypes.data, None if d is None else d.ctypes.data, block.ctypes.data, H, _p(norm), _p(proj),
            _p(post), eps, _p(router), E, None if prefix is None else prefix.ctypes.data, hidden.ctypes.data,
            None if logits is None else logits.ctypes.data), "prepare_moe_route_host")
        return prefix, hidden, logits

    def mxfp4_matvec(self, packed, scales, rows, cols, x, y):
        """y [T][rows] = MXFP4 [rows][cols] x [T][cols] (device tensors), the
        reference's mxfp4_matmul FP64 column-order sums."""
        self._check(self.lib.k3xb_mxfp4_matvec(self.h, _p(packed), _p(scales), rows, cols, _p(x), x.shape[0], _p(y)),
                    "mxfp4_matvec")

    def resident_moe_layer_host(self, w: dict, experts, contributions, x, eps, beta, linear_beta=0.0):
        """resident_mxfp4_moe_layer: w holds device f32 projections, experts a
        list of dicts of device MXFP4 arrays (gate_packed, ...), one per slot;
        HOST contributions, x -> HOST y."""
        import numpy as np
        D, H = w["routed_down"].shape
        S = w["shared_gate"].shape[0]
        I = experts[0]["gate_scales"].shape[0]
        names = ("gate_packed", "gate_scales", "up_packed", "up_scales", "down_packed", "down_scales")
        arr = (C.c_void_p * (6 * len(experts)))(*[e[n].data_ptr() for e in experts for n in names])
        con = np.ascontiguousarray(contributions, dtype=np.float32)
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty(H, np.float32)
        self._check(self.lib.k3xb_resident_moe_layer_host(
            self.h, H, D, I, S, *(_p(w[k]) for k in ("routed_down", "routed_norm", "routed_up", "shared_gate",
                                                      "shared_up", "shared_down")),
            arr, len(experts), con.ctypes.data, eps, beta, linear_beta, x.ctypes.data, y.ctypes.data),
            "resident_moe_layer_host")
        return y

    def dense_matvec_host(self, W, x):
        """W device [rows][cols]; HOST x [cols] -> HOST y [rows]."""
        import numpy as np
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty(W.shape[0], np.float32)
        self._check(self.lib.k3xb_dense_matvec_host(self.h, _p(W), W.shape[0], W.shape[1], x.ctypes.data,
                                                    y.ctypes.data), "dense_matvec_host")
        return y

    def dense_situ_mlp_host(self, gate, up, down, x, beta, linear_beta=0.0):
        """Device gate/up [inter][cols], down [out][inter]; HOST x -> HOST y."""
        import numpy as np
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty(down.shape[0], np.float32)
        self._check(self.lib.k3xb_dense_situ_mlp_host(self.h, _p(gate), _p(up), _p(down), gate.shape[0],
                                                      gate.shape[1], down.shape[0], x.ctypes.data, beta,
                                                      linear_beta, y.ctypes.data), "dense_situ_mlp_host")
        return y

    def kda_block_held(self, w: KdaLayer, hidden, x, slot, mode, conv=None, recurrent=None):
        """k3xb_kda_block_held: x [T][H] float32 (HOST) -> out [T][H] from the
        state held in `slot`. mode KDA_SEED takes conv/recurrent as the
        starting state; KDA_PUBLISH writes the new state into them."""
        import numpy as np
        x = np.ascontiguousarray(x, dtype=np.float32)
        for a, dt in ((conv, np.uint16), (recurrent, np.float32)):
            if a is not None and (a.dtype != dt or not a.flags.c_contiguous):
                raise K3xbError(INVALID_EXTENT, "conv must be contiguous uint16 and recurrent float32")
        out = np.empty((x.shape[0], hidden), np.float32)
        self._check(self.lib.k3xb_kda_block_held(self.h, C.byref(w), hidden, x.ctypes.data, x.shape[0], slot, mode,
                                                 None if conv is None else conv.ctypes.data,
                                                 None if recurrent is None else recurrent.ctypes.data,
                                                 out.ctypes.data), "kda_block_held")
        return out

    def release_resident(self):
        self._check(self.lib.k3xb_release_resident(self.h), "release_resident")

    def official_moe_ffn_host(self, tail: MoeLayer, slots, contributions, hidden, prefix):
        """official_mxfp4_moe_ffn for one position (k3xb_official_moe_ffn_host):
        `slots` is a list of one-expert MoeLayer descriptors in route order;
        HOST contributions [K], hidden [H], prefix [H] -> HOST out [H]."""
        import numpy as np
        K = len(slots)
        arr = (MoeLayer * K)(*slots)
        con = np.ascontiguousarray(contributions, dtype=np.float32)
        x = np.ascontiguousarray(hidden, dtype=np.float32)
        p = np.ascontiguousarray(prefix, dtype=np.float32)
        out = np.empty_like(x)
        self._check(self.lib.k3xb_official_moe_ffn_host(self.h, C.byref(tail), arr, K, con.ctypes.data,
                                                        x.ctypes.data, p.ctypes.data, out.ctypes.data),
                    "official_moe_ffn_host")
        return out

    def prepare_layer_scales(self, w: dict):
        """Adds tcgen05-layout copies of the three expert scale arrays to a
        layer dict (one-time, for resident weights)."""
        import torch
        E, H, I = w["experts"], w.get("latent") or w["hidden"], w["inter"]   # H: the experts' width
        for name, rows, cols in (("gate", E * I, H), ("up", E * I, H), ("down", E * H, I)):
            out = torch.empty_like(w[f"{name}_scales"])
            self.prepare_mxfp4_scales(w[f"{name}_scales"], rows, cols, out)
            w[f"{name}_scales_tc"] = out
        return w

    def fill_normal_mxfp4(self, packed, scales, rows, cols, seed, stream, sigma):
        self._check(self.lib.k3xb_fill_normal_mxfp4(self.h, _p(packed), _p(scales), rows, cols, seed, stream,
                                                    sigma), "fill_normal_mxfp4")


def moe_layer_desc(w: dict, engine=ENGINE_SIMT, act_terms=0) -> MoeLayer:
    """Builds the C descriptor from a dict of torch CUDA tensors + dims. The
    descriptor holds a reference to the dict, so the tensors it points at
    stay allocated as long as the descriptor object lives (a struct copied
    by value into another descriptor does not carry it: layer_desc and
    verify_model_desc keep their parts themselves)."""
    L = MoeLayer()
    L._keep = w
    L.hidden, L.inter, L.experts, L.top_k = w["hidden"], w["inter"], w["experts"], w["top_k"]
    L.shared_inter = w.get("shared_inter", 0)
    for name in ("router", "correction", "gate_packed", "gate_scales", "up_packed", "up_scales",
                 "down_packed", "down_scales", "shared_gate", "shared_up", "shared_down",
                 "gate_scales_tc", "up_scales_tc", "down_scales_tc"):
        t = w.get(name)
        setattr(L, name, None if t is None else t.data_ptr())
    L.activation = w.get("activation", ACT_SWIGLU)
    L.situ_beta = w.get("situ_beta", 4.0)
    L.situ_linear_beta = w.get("situ_linear_beta", 0.0)
    L.engine = engine
    L.act_terms = act_terms
    L.latent = w.get("latent", 0)   # LatentMoE width (0: plain MoE)
    for name in ("routed_down", "routed_norm", "routed_up"):
        t = w.get(name)
        setattr(L, name, None if t is None else t.data_ptr())
    L.latent_eps = w.get("latent_eps", 1e-6)
    t = w.get("ep_owner")   # expert placement (device uint32 [experts_total]) for expert parallelism
    L.ep_owner = None if t is None else t.data_ptr()
    return L


def default_act_terms(assignments: int, experts: int) -> int:
    """The MXF4 engine's E2M1 term count for act_terms 0 (k3xb_default_act_terms)."""
    return int(library().k3xb_default_act_terms(assignments, experts))


def phase_name(i: int) -> str:
    n = library().k3xb_phase_name(i)
    return n.decode() if n else None


def stack_layer_desc(stack: ResidentStack, w: dict, engine=ENGINE_MXF4, act_terms=0) -> MoeLayer:
    """moe_layer_desc with the expert arrays taken from a resident stack
    (k3xb_acquire_expert_stack); router, correction and the shared expert
    still come from the dict."""
    if stack.disposition == RESIDENT_BYPASS:
        raise K3xbError(INVALID_STATE, "expert stack was not admitted (resident capacity)")
    L = moe_layer_desc(w, engine=engine, act_terms=act_terms)
    for name, _ in ResidentStack._fields_:
        if name not in ("disposition", "uploaded_bytes"):
            setattr(L, name, getattr(stack, name))
    return L


def kda_layer_desc(w: dict) -> KdaLayer:
    """C descriptor of a KDA block from a dict of torch CUDA tensors + dims."""
    K = KdaLayer()
    K._keep = w   # the tensors stay allocated while the descriptor lives
    K.heads, K.head_dim, K.conv_width = w["heads"], w["head_dim"], w["conv_width"]
    K.eps, K.gate_lower_bound = w["eps"], w["gate_lower_bound"]
    for name in ("q_proj", "k_proj", "v_proj", "q_conv", "k_conv", "v_conv", "f_a_proj", "f_b_proj", "a_log",
                 "dt_bias", "b_proj", "g_proj", "o_norm", "o_proj"):
        setattr(K, name, w[name].data_ptr())
    return K


def layer_desc(w: dict, engine=ENGINE_MXF4, act_terms=0) -> Layer:
    """C descriptor of a KDA + MoE layer: w["kda"], w["moe"] sub-dicts and
    the six [H] bf16 norm/projection vectors."""
    L = Layer()
    L._keep = w   # the norm vectors and both sub-dicts' tensors
    L.hidden = w["hidden"]
    L.rms_eps = w["rms_eps"]
    for name in ("self_residual_norm", "self_residual_proj", "input_norm", "moe_residual_norm",
                 "moe_residual_proj", "post_norm"):
        setattr(L, name, w[name].data_ptr())
    L.kda = kda_layer_desc(w["kda"])
    L.moe = moe_layer_desc(w["moe"], engine=engine, act_terms=act_terms)
    return L


ACCEPT_GREEDY = 0
ACCEPT_REJECTION = 1


def verify_model_desc(layers, vocab, lm_head, embedding=None, final_norm=None, final_eps=1e-6):
    """C descriptor of a verify stack; `layers` is a list of Layer
    descriptors (kept alive by the returned object)."""
    arr = (Layer * len(layers))(*layers)
    m = VerifyModel()
    m.layers, m.vocab = len(layers), vocab
    m.layer = C.cast(arr, C.POINTER(Layer))
    m.embedding = None if embedding is None else embedding.data_ptr()
    m.final_norm = None if final_norm is None else final_norm.data_ptr()
    m.final_eps = final_eps
    m.lm_head = lm_head.data_ptr()
    m._keep = (arr, list(layers), lm_head, embedding, final_norm)
    return m


def verify_io_desc(sequences, drafts, conv, recurrent, accepted, committed, committed_count, draft_tokens,
                   tokens=None, hidden_in=None, block_source=None, logits=None, mode=ACCEPT_GREEDY,
                   draft_logits=None, temperature=1.0, seed=0, sequence_base=0):
    io = VerifyIO()
    io.sequences, io.drafts = sequences, drafts
    ptr = lambda t: None if t is None else t.data_ptr()
    io.tokens, io.hidden_in, io.block_source = ptr(tokens), ptr(hidden_in), ptr(block_source)
    io.draft_tokens, io.conv, io.recurrent = ptr(draft_tokens), ptr(conv), ptr(recurrent)
    io.mode, io.draft_logits, io.temperature = mode, ptr(draft_logits), temperature
    io.seed, io.sequence_base = seed, sequence_base
    io.logits, io.accepted, io.committed = ptr(logits), ptr(accepted), ptr(committed)
    io.committed_count = ptr(committed_count)
    io._keep = (tokens, hidden_in, block_source, draft_tokens, conv, recurrent, draft_logits, logits, accepted,
                committed, committed_count)
    return io


def ep_unique_id() -> bytes:
    """A fresh NCCL unique id (128 bytes) for k3xb_ep_init on every rank."""
    buf = (C.c_uint8 * 128)()
    st = library().k3xb_ep_unique_id(buf)
    if st != OK:
        raise K3xbError(st, "ep_unique_id")
    return bytes(buf)


def ep_balance(load, world: int):
    """k3xb_ep_balance: an expert placement (numpy uint32 [E], entry
    rank << 16 | local index) dealing experts in descending `load` over the
    ranks in a snake."""
    import numpy as np
    load = np.ascontiguousarray(load, np.float32)
    owner = np.empty(load.size, np.uint32)
    st = library().k3xb_ep_balance(load.ctypes.data, load.size, world, owner.ctypes.data)
    if st:
        raise K3xbError(st, "ep_balance")
    return owner


def ep_local_layer(w: dict, rank: int, world: int, owner=None) -> dict:
    """The expert shard of rank `rank`, router/correction/shared kept whole.
    Without `owner`: experts [rank*E/world, ...) of the stacked MXFP4 arrays
    (views, no copies). With `owner` (numpy uint32 [E], as ep_balance makes):
    the experts it gives this rank, in their local order (copies), and the
    table itself on the device as the layer's ep_owner."""
    E = w["experts"]
    if E % world:
        raise K3xbError(INVALID_EXTENT, "experts must divide evenly over the world")
    n = E // world
    if owner is not None:
        import numpy as np
        import torch
        owner = np.ascontiguousarray(owner, np.uint32)
        mine = [(int(o) & 0xffff, e) for e, o in enumerate(owner) if int(o) >> 16 == rank]
        mine.sort()
        if len(owner) != E or [loc for loc, _ in mine] != list(range(n)):
            raise K3xbError(INVALID_EXTENT, "ep_local_layer: owner must give every rank E/world experts")
        idx = torch.tensor([e for _, e in mine], dtype=torch.long, device=w["gate_packed"].device)
        out = dict(w, experts=n)
        for k in ("gate_packed", "gate_scales", "up_packed", "up_scales", "down_packed", "down_scales"):
            out[k] = w[k].index_select(0, idx)
        I, H = w["inter"], w["hidden"]
        for k in ("gate_scales_tc", "up_scales_tc", "down_scales_tc"):
            if w.get(k) is not None:   # whole experts are contiguous in the atom layout
                out[k] = w[k].view(E, -1).index_select(0, idx).view(-1)
        out["ep_owner"] = torch.from_numpy(owner.view(np.int32)).to(w["gate_packed"].device)
        return out
    lo, hi = rank * n, (rank + 1) * n
    out = dict(w, experts=n)
    for k in ("gate_packed", "gate_scales", "up_packed", "up_scales", "down_packed", "down_scales"):
        out[k] = w[k][lo:hi]
    I, H = w["inter"], w["hidden"]
    for k, rows in (("gate_scales_tc", I), ("up_scales_tc", I), ("down_scales_tc", H)):
        if w.get(k) is not None:   # atoms [E*rows/128][K/128][512]: whole experts are contiguous
            per = w[k].numel() // E
            out[k] = w[k].view(-1)[lo * per:hi * per]
    return out
