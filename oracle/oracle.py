"""ctypes bindings for the two CPU checkers (TEST INFRASTRUCTURE ONLY).

`Restatement` wraps libk3x_oracle.so (k3x_oracle.c, the C restatement of the
reference algorithms). `Reference` wraps _ref/libk3x_ref.so (the reference's
own CPU sources compiled by oracle/Makefile). Only tests/, __graft_entry__.smoke()
and bench.py's CPU legs may import this module; the product never does.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
RESTATEMENT_SO = os.path.join(HERE, "libk3x_oracle.so")
REFERENCE_SO = os.path.join(HERE, "_ref", "libk3x_ref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_sz = C.c_size_t
_szp = C.POINTER(C.c_size_t)

ACT_SWIGLU = 0
ACT_SITU = 1

ROUTING_NATURAL, ROUTING_FIXED, ROUTING_ADAPTIVE = 0, 1, 2
_SELECT_ROUTING_ARGS = [_f32p, _f32p, _sz, _sz, C.c_int, _sz, C.c_float, C.c_float, _sz, C.c_void_p,
                        _u32p, _f32p, _szp, _f32p, C.POINTER(C.c_int)]


def _select_routing(fn, scores, bias, natural_k, mode=ROUTING_NATURAL, fixed_k=0, mass_target=0.9,
                    minimum_gap=0.0, quality_floor_k=0):
    """Shared wrapper of k3xo_/k3xr_select_routing: (status, dict)."""
    scores = _c(scores, np.float32)
    bias = _c(bias, np.float32)
    E = scores.size
    order = np.zeros(E, np.uint32)
    ids = np.zeros(max(natural_k, 1), np.uint32)
    w = np.zeros(max(natural_k, 1), np.float32)
    k = C.c_size_t()
    stats = np.zeros(4, np.float32)
    esc = C.c_int()
    st = fn(scores, bias, E, natural_k, mode, fixed_k, mass_target, minimum_gap, quality_floor_k,
            order.ctypes.data_as(C.c_void_p), ids, w, C.byref(k), stats, C.byref(esc))
    if st:
        return st, None
    n = k.value
    return 0, dict(full_order=order, expert_ids=ids[:n], weights=w[:n], selected_k=n,
                   normalized_entropy=stats[0], support=stats[1], mass=stats[2], boundary=stats[3],
                   escalated=bool(esc.value))


class OracleError(RuntimeError):
    def __init__(self, status: int, where: str):
        super().__init__(f"{where} failed with status {status}")
        self.status = status


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class _MoeLayer(C.Structure):
    _fields_ = [
        ("hidden", _sz), ("inter", _sz), ("experts", _sz), ("top_k", _sz),
        ("shared_inter", _sz),
        ("router", C.c_void_p), ("correction", C.c_void_p),
        ("gate_packed", C.c_void_p), ("gate_scales", C.c_void_p),
        ("up_packed", C.c_void_p), ("up_scales", C.c_void_p),
        ("down_packed", C.c_void_p), ("down_scales", C.c_void_p),
        ("shared_gate", C.c_void_p), ("shared_up", C.c_void_p), ("shared_down", C.c_void_p),
        ("activation", C.c_int), ("situ_beta", C.c_float), ("situ_linear_beta", C.c_float),
        ("latent", _sz), ("routed_down", C.c_void_p), ("routed_norm", C.c_void_p), ("routed_up", C.c_void_p),
        ("latent_eps", C.c_float),
    ]


class _KdaWeights(C.Structure):
    _fields_ = [
        ("hidden", _sz), ("heads", _sz), ("head_dim", _sz), ("conv_width", _sz),
        ("eps", C.c_float), ("gate_lower_bound", C.c_float),
        ("q_proj", C.c_void_p), ("k_proj", C.c_void_p), ("v_proj", C.c_void_p),
        ("q_conv", C.c_void_p), ("k_conv", C.c_void_p), ("v_conv", C.c_void_p),
        ("f_a_proj", C.c_void_p), ("f_b_proj", C.c_void_p),
        ("a_log", C.c_void_p), ("dt_bias", C.c_void_p),
        ("b_proj", C.c_void_p), ("g_proj", C.c_void_p),
        ("o_norm", C.c_void_p), ("o_proj", C.c_void_p),
    ]


class _MlaWeights(C.Structure):
    _fields_ = [
        ("hidden", _sz), ("heads", _sz), ("q_rank", _sz), ("kv_rank", _sz), ("q_main", _sz), ("q_extra", _sz),
        ("value_dim", _sz), ("eps", C.c_float),
        ("q_a_proj", C.c_void_p), ("q_a_norm", C.c_void_p), ("q_b_proj", C.c_void_p),
        ("kv_a_proj", C.c_void_p), ("kv_a_norm", C.c_void_p), ("kv_b_proj", C.c_void_p),
        ("g_proj", C.c_void_p), ("o_proj", C.c_void_p),
    ]


MLA_TENSORS = ("q_a_proj", "q_a_norm", "q_b_proj", "kv_a_proj", "kv_a_norm", "kv_b_proj", "g_proj", "o_proj")


def moe_struct(layer: dict):
    """Builds the C layer descriptor from a dict of numpy arrays; returns
    (struct, keepalive)."""
    keep = {k: (_c(v, v.dtype) if isinstance(v, np.ndarray) else v) for k, v in layer.items()}
    s = _MoeLayer()
    s.hidden, s.inter = keep["hidden"], keep["inter"]
    s.experts, s.top_k = keep["experts"], keep["top_k"]
    s.shared_inter = keep.get("shared_inter", 0)
    for name in ("router", "correction", "gate_packed", "gate_scales", "up_packed",
                 "up_scales", "down_packed", "down_scales"):
        setattr(s, name, _ptr(keep[name]))
    for name in ("shared_gate", "shared_up", "shared_down"):
        setattr(s, name, _ptr(keep.get(name)))
    s.activation = keep.get("activation", ACT_SWIGLU)
    s.situ_beta = keep.get("situ_beta", 4.0)
    s.situ_linear_beta = keep.get("situ_linear_beta", 0.0)
    s.latent = keep.get("latent", 0)
    for name in ("routed_down", "routed_norm", "routed_up"):
        setattr(s, name, _ptr(keep.get(name)))
    s.latent_eps = keep.get("latent_eps", 1e-6)
    return s, keep


def kda_struct(w: dict):
    keep = {k: (_c(v, v.dtype) if isinstance(v, np.ndarray) else v) for k, v in w.items()}
    s = _KdaWeights()
    for name in ("hidden", "heads", "head_dim", "conv_width", "eps", "gate_lower_bound"):
        setattr(s, name, keep[name])
    for name in ("q_proj", "k_proj", "v_proj", "q_conv", "k_conv", "v_conv", "f_a_proj",
                 "f_b_proj", "a_log", "dt_bias", "b_proj", "g_proj", "o_norm", "o_proj"):
        setattr(s, name, _ptr(keep[name]))
    return s, keep


class Restatement:
    """The C restatement (k3x_oracle.c)."""

    def __init__(self, path: str = RESTATEMENT_SO):
        L = C.CDLL(path)
        self.lib = L
        L.k3xo_round_bf16.restype = C.c_float
        L.k3xo_round_bf16.argtypes = [C.c_float]
        L.k3xo_decode_mxfp4.argtypes = [_u8p, _u8p, _sz, _sz, _sz, _f32p]
        L.k3xo_mxfp4_matmul.argtypes = [_f32p, _u8p, _u8p, _sz, _sz, _sz, _f32p]
        L.k3xo_quantize_mxfp4.argtypes = [_f32p, _sz, _sz, _u8p, _u8p]
        L.k3xo_quantize_mxfp4.restype = None
        L.k3xo_e2m1_terms.argtypes = [_f32p, C.c_int, _u8p, _u8p]
        L.k3xo_e2m1_terms.restype = C.c_float
        L.k3xo_situ_glu.argtypes = [_f32p, _f32p, _f32p, _sz, C.c_float, C.c_float]
        L.k3xo_situ_glu.restype = None
        L.k3xo_swiglu.argtypes = [_f32p, _f32p, _f32p, _sz]
        L.k3xo_swiglu.restype = None
        L.k3xo_bf16_matvec.argtypes = [_f32p, _u16p, _sz, _sz, _f32p]
        L.k3xo_dense_matvec.argtypes = [_f32p, _f32p, _sz, _sz, _f32p]
        L.k3xo_router_logits.argtypes = [_f32p, _u16p, _sz, _sz, _f32p]
        L.k3xo_route_logits.argtypes = [_f32p, _f32p, _sz, _sz, _u32p, _f32p, C.c_void_p]
        L.k3xo_expert_major_plan.argtypes = [_u32p, _f32p, _sz, _sz, _u32p, _u32p, _u32p,
                                             _u32p, _f32p, _szp]
        L.k3xo_routed_combine.argtypes = [_f32p, _f32p, _sz, _sz, _f32p]
        L.k3xo_routed_combine.restype = None
        L.k3xo_moe_layer_forward.argtypes = [C.c_void_p, _f32p, _sz, _f32p, _u32p, _f32p]
        L.k3xo_kda_step.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _sz, _sz, _f32p]
        L.k3xo_kda_tree.argtypes = [_f32p, _i32p, _sz, _f32p, _f32p, _f32p, _f32p, _f32p,
                                    _sz, _sz, _f32p, C.c_void_p]
        L.k3xo_kda_block.argtypes = [C.c_void_p, _f32p, _sz, _u16p, _u16p, _u16p, _f32p, _f32p]
        L.k3xo_rms_norm_bf16.argtypes = [_f32p, _u16p, _sz, C.c_float, _f32p]
        L.k3xo_select_routing.argtypes = _SELECT_ROUTING_ARGS
        L.k3xo_attention_residual.argtypes = [_f32p, _f32p, _u16p, _u16p, _sz, C.c_float, _f32p]
        L.k3xo_rms_norm_f32.argtypes = [_f32p, _f32p, _sz, C.c_float, _f32p]
        L.k3xo_rms_norm_f32.restype = None
        L.k3xo_block_attention_residual.argtypes = [_f32p, _f32p, _sz, _sz, _sz, _f32p, _f32p, C.c_float, _f32p]
        L.k3xo_mla_step.argtypes = [C.c_void_p, _f32p, _f32p, _f32p, _f32p, _sz, _szp, _f32p]
        L.k3xo_mla_crop.argtypes = [_szp, _sz]
        L.k3xo_mla_tree.argtypes = [C.c_void_p, _f32p, _f32p, _f32p, _sz, _i32p, _sz, _f32p, _f32p, _f32p,
                                    _f32p, _f32p]
        L.k3xo_argmax.restype = C.c_uint32
        L.k3xo_argmax.argtypes = [_f32p, _sz]
        L.k3xo_verify_greedy_block.argtypes = [C.c_uint32, _u32p, _sz, _sz, _sz, _u32p,
                                               _szp, _u32p, _szp, C.POINTER(C.c_int)]
        L.k3xo_uniform.restype = C.c_double
        L.k3xo_uniform.argtypes = [C.c_uint64] * 4
        L.k3xo_verify_rejection.argtypes = [_f32p, _f32p, _u32p, _sz, _sz, C.c_float,
                                            C.c_uint64, C.c_uint64, _szp, _u32p, _szp]
        u64 = C.c_uint64
        L.k3xo_fill_normal_f32.argtypes = [_f32p, _sz, u64, u64, u64, C.c_float, C.c_float]
        L.k3xo_fill_normal_f32.restype = None
        L.k3xo_fill_normal_bf16.argtypes = [_u16p, _sz, u64, u64, u64, C.c_float]
        L.k3xo_fill_normal_bf16.restype = None
        L.k3xo_fill_normal_mxfp4.argtypes = [_u8p, _u8p, _sz, u64, u64, u64, C.c_float]
        L.k3xo_fill_normal_mxfp4.restype = None

    # -- the library's seeded generator (csrc/synth.cu), any slice ---------------
    def fill_normal_f32(self, n, seed, stream, first=0, mean=0.0, sigma=1.0):
        out = np.empty(n, np.float32)
        self.lib.k3xo_fill_normal_f32(out, n, first, seed, stream, mean, sigma)
        return out

    def fill_normal_bf16(self, n, seed, stream, first=0, sigma=1.0):
        """bf16 words."""
        out = np.empty(n, np.uint16)
        self.lib.k3xo_fill_normal_bf16(out, n, first, seed, stream, sigma)
        return out

    def fill_normal_mxfp4(self, blocks, seed, stream, first=0, sigma=0.02):
        """(packed [blocks*16] bytes, scales [blocks]) of 32-blocks first..first+blocks-1."""
        packed = np.empty(blocks * 16, np.uint8)
        scales = np.empty(blocks, np.uint8)
        self.lib.k3xo_fill_normal_mxfp4(packed, scales, blocks, first, seed, stream, sigma)
        return packed, scales

    # -- helpers ---------------------------------------------------------------
    @staticmethod
    def _check(st, where):
        if st != 0:
            raise OracleError(st, where)

    def round_bf16(self, x):
        x = _c(x, np.float32)
        u = x.view(np.uint32).astype(np.uint64)
        special = (u & 0x7F800000) == 0x7F800000
        r = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
        s = np.where((u & 0x7FFFFF) != 0, (u | 0x400000) & 0xFFFF0000, u & 0xFFFF0000)
        return np.where(special, s, r).astype(np.uint32).view(np.float32).reshape(x.shape)

    def decode_mxfp4(self, packed, scales, rows, cols, group=32):
        out = np.empty(rows * cols, np.float32)
        self._check(self.lib.k3xo_decode_mxfp4(_c(packed, np.uint8), _c(scales, np.uint8),
                                               rows, cols, group, out), "decode_mxfp4")
        return out.reshape(rows, cols)

    def mxfp4_matmul(self, x, packed, scales, rows, cols, group=32):
        out = np.empty(rows, np.float32)
        self._check(self.lib.k3xo_mxfp4_matmul(_c(x, np.float32), _c(packed, np.uint8),
                                               _c(scales, np.uint8), rows, cols, group, out),
                    "mxfp4_matmul")
        return out

    def quantize_mxfp4(self, x):
        x = _c(x, np.float32)
        rows, cols = x.shape
        packed = np.empty((rows, cols // 2), np.uint8)
        scales = np.empty((rows, cols // 32), np.uint8)
        self.lib.k3xo_quantize_mxfp4(x, rows, cols, packed, scales)
        return packed, scales

    def e2m1_terms(self, x32, nterms):
        packed = np.empty(nterms * 16, np.uint8)
        scales = np.empty(nterms, np.uint8)
        res = self.lib.k3xo_e2m1_terms(_c(x32, np.float32), nterms, packed, scales)
        return packed.reshape(nterms, 16), scales, res

    def situ_glu(self, gate, up, beta, linear_beta=0.0):
        g, u = _c(gate, np.float32), _c(up, np.float32)
        out = np.empty_like(g)
        self.lib.k3xo_situ_glu(out, g, u, g.size, beta, linear_beta)
        return out

    def swiglu(self, gate, up):
        g, u = _c(gate, np.float32), _c(up, np.float32)
        out = np.empty_like(g)
        self.lib.k3xo_swiglu(out, g, u, g.size)
        return out

    def bf16_matvec(self, x, w):
        w = _c(w, np.uint16)
        out = np.empty(w.shape[0], np.float32)
        self._check(self.lib.k3xo_bf16_matvec(_c(x, np.float32), w, w.shape[0], w.shape[1], out),
                    "bf16_matvec")
        return out

    def dense_matvec(self, x, w):
        """The CPU backend's f32 dense product (backend_cpu.cpp:23-47)."""
        w = _c(w, np.float32)
        out = np.empty(w.shape[0], np.float32)
        self._check(self.lib.k3xo_dense_matvec(_c(x, np.float32), w, w.shape[0], w.shape[1], out), "dense_matvec")
        return out

    def dense_situ_mlp(self, x, gate, up, down, beta, linear_beta=0.0):
        """dense_situ_mlp (backend_cpu.cpp:107-122)."""
        a = self.situ_glu(self.dense_matvec(x, gate), self.dense_matvec(x, up), beta, linear_beta)
        return self.dense_matvec(a, down)

    def resident_moe_layer(self, w: dict, experts: dict, contributions, x, eps, beta, linear_beta=0.0):
        """resident_mxfp4_moe_layer (backend_cpu.cpp:305-339) composed of the
        restated pieces: f32 products, unrounded expert outputs, a float mix
        in slot order, rms_norm (ops.cpp:10-18) in float with FP64 squares."""
        D, H = w["routed_down"].shape
        K, I = experts["gate_packed"].shape[:2]
        latent = self.dense_matvec(x, w["routed_down"])
        ys = []
        for k in range(K):
            g = self.mxfp4_matmul(latent, experts["gate_packed"][k], experts["gate_scales"][k], I, D)
            u = self.mxfp4_matmul(latent, experts["up_packed"][k], experts["up_scales"][k], I, D)
            a = self.situ_glu(g, u, beta, linear_beta)
            ys.append(self.mxfp4_matmul(a, experts["down_packed"][k], experts["down_scales"][k], D, I))
        c = np.asarray(contributions, np.float32)
        mixed = np.zeros(D, np.float32)
        for k in range(K):
            mixed = (mixed + c[k] * ys[k]).astype(np.float32)   # float32 ops, slot order
        squares = 0.0
        for v in mixed.tolist():   # FP64, index order; a float square is exact in FP64
            squares += v * v
        inverse = np.float32(1.0) / np.sqrt(np.float32(np.float32(squares / D) + np.float32(eps)))
        normed = (mixed * inverse).astype(np.float32) * np.asarray(w["routed_norm"], np.float32)
        routed = self.dense_matvec(normed.astype(np.float32), w["routed_up"])
        shared = self.dense_situ_mlp(x, w["shared_gate"], w["shared_up"], w["shared_down"], beta, linear_beta)
        return (routed + shared).astype(np.float32)

    def router_logits(self, hidden, router):
        router = _c(router, np.uint16)
        out = np.empty(router.shape[0], np.float32)
        self._check(self.lib.k3xo_router_logits(_c(hidden, np.float32), router,
                                                router.shape[0], router.shape[1], out),
                    "router_logits")
        return out

    def route_logits(self, logits, correction, top_k, want_scores=False):
        logits = _c(logits, np.float32)
        E = logits.size
        ids = np.empty(top_k, np.uint32)
        contrib = np.empty(top_k, np.float32)
        scores = np.empty(E, np.float32) if want_scores else None
        self._check(self.lib.k3xo_route_logits(logits, _c(correction, np.float32), E, top_k, ids,
                                               contrib, _ptr(scores)), "route_logits")
        return (ids, contrib, scores) if want_scores else (ids, contrib)

    def route(self, hidden, router, correction, top_k):
        return self.route_logits(self.router_logits(hidden, router), correction, top_k)

    def expert_major_plan(self, ids, contrib):
        ids = _c(ids, np.uint32)
        T, K = ids.shape
        n = T * K
        ge = np.zeros(n, np.uint32)
        go = np.zeros(n + 1, np.uint32)
        at = np.zeros(n, np.uint32)
        asl = np.zeros(n, np.uint32)
        ac = np.zeros(n, np.float32)
        ng = C.c_size_t(0)
        self._check(self.lib.k3xo_expert_major_plan(ids, _c(contrib, np.float32), T, K, ge, go, at,
                                                    asl, ac, C.byref(ng)), "expert_major_plan")
        g = ng.value
        return dict(group_expert=ge[:g], group_offset=go[:g + 1], assign_token=at[:n],
                    assign_slot=asl[:n], assign_contrib=ac[:n])

    def routed_combine(self, y, contrib):
        y = _c(y, np.float32)
        K, H = y.shape
        out = np.empty(H, np.float32)
        self.lib.k3xo_routed_combine(y, _c(contrib, np.float32), K, H, out)
        return out

    def moe_layer(self, layer: dict, hidden):
        hidden = _c(hidden, np.float32)
        T = hidden.shape[0]
        s, keep = moe_struct(layer)
        out = np.empty((T, layer["hidden"]), np.float32)
        ids = np.empty((T, layer["top_k"]), np.uint32)
        contrib = np.empty((T, layer["top_k"]), np.float32)
        self._check(self.lib.k3xo_moe_layer_forward(C.byref(s), hidden, T, out, ids, contrib),
                    "moe_layer_forward")
        del keep
        return out, ids, contrib

    def kda_step(self, state, q, k, v, log_decay, beta, heads, head_dim):
        state = np.array(state, np.float32, copy=True, order="C")
        out = np.empty(heads * head_dim, np.float32)
        self._check(self.lib.k3xo_kda_step(state, _c(q, np.float32), _c(k, np.float32),
                                           _c(v, np.float32), _c(log_decay, np.float32),
                                           _c(beta, np.float32), heads, head_dim, out),
                    "kda_step")
        return state, out

    def kda_tree(self, prefix_state, parent, q, k, v, log_decay, beta, heads, head_dim,
                 want_states=False):
        parent = _c(parent, np.int32)
        n = parent.size
        out = np.empty((n, heads * head_dim), np.float32)
        states = np.empty((n, heads, head_dim, head_dim), np.float32) if want_states else None
        self._check(self.lib.k3xo_kda_tree(_c(prefix_state, np.float32), parent, n,
                                           _c(q, np.float32), _c(k, np.float32), _c(v, np.float32),
                                           _c(log_decay, np.float32), _c(beta, np.float32),
                                           heads, head_dim, out, _ptr(states)), "kda_tree")
        return (out, states) if want_states else out

    def kda_block(self, weights: dict, hidden, conv_q, conv_k, conv_v, recurrent):
        s, keep = kda_struct(weights)
        hidden = _c(hidden, np.float32)
        T = hidden.size // weights["hidden"]
        cq, ck, cv = (np.array(a, np.uint16, copy=True) for a in (conv_q, conv_k, conv_v))
        rec = np.array(recurrent, np.float32, copy=True)
        out = np.empty(T * weights["hidden"], np.float32)
        self._check(self.lib.k3xo_kda_block(C.byref(s), hidden, T, cq, ck, cv, rec, out),
                    "kda_block")
        del keep
        return out.reshape(T, weights["hidden"]), (cq, ck, cv, rec)

    def select_routing(self, scores, bias, natural_k, **policy):
        return _select_routing(self.lib.k3xo_select_routing, scores, bias, natural_k, **policy)

    # -- layer composition ------------------------------------------------------
    def rms_norm(self, x, weight, eps):
        x = _c(x, np.float32)
        out = np.empty_like(x)
        self._check(self.lib.k3xo_rms_norm_bf16(x, _c(weight, np.uint16), x.size, eps, out), "rms_norm")
        return out

    def attention_residual(self, prefix, block, norm, proj, eps):
        prefix = _c(prefix, np.float32)
        out = np.empty_like(prefix)
        self._check(self.lib.k3xo_attention_residual(prefix, _c(block, np.float32), _c(norm, np.uint16),
                                                     _c(proj, np.uint16), prefix.size, eps, out),
                    "attention_residual")
        return out

    def rms_norm_f32(self, x, weight, eps):
        """rms_norm (ops.cpp:10-18) with float weights, one row."""
        x = _c(x, np.float32)
        out = np.empty_like(x)
        self.lib.k3xo_rms_norm_f32(x, _c(weight, np.float32), x.size, eps, out)
        return out

    def block_attention_residual(self, prefix, sources, norm, proj, eps):
        """model.cpp:645-666 over T rows: prefix [T][H], sources [S][T][H]."""
        prefix = _c(np.atleast_2d(prefix), np.float32)
        T, H = prefix.shape
        sources = _c(np.asarray(sources, np.float32).reshape(-1, T, H), np.float32)
        out = np.empty_like(prefix)
        self._check(self.lib.k3xo_block_attention_residual(prefix, sources, sources.shape[0], T, H,
                                                           _c(norm, np.float32), _c(proj, np.float32), eps, out),
                    "block_attention_residual")
        return out

    def mla_state(self, w: dict, capacity):
        """An empty MLA state (model.cpp:70): position-major keys, values and
        shared keys with room for `capacity` positions."""
        return {"keys": np.zeros((capacity, w["heads"], w["q_main"]), np.float32),
                "values": np.zeros((capacity, w["heads"], w["value_dim"]), np.float32),
                "shared": np.zeros((capacity, w["q_extra"]), np.float32), "length": 0}

    def mla_prefill(self, w: dict, x, state=None, capacity=64):
        """Gated MLA (model.cpp:755-811) over the rows of x, one position at a
        time, appending to `state` (made empty when None). w holds the dims
        (hidden, heads, q_rank, kv_rank, q_main, q_extra, value_dim, eps) and
        the f32 weights of MLA_TENSORS."""
        x = _c(np.atleast_2d(x), np.float32)
        st = state if state is not None else self.mla_state(w, capacity)
        keep = [_c(w[k], np.float32) for k in MLA_TENSORS]
        ws = _MlaWeights(w["hidden"], w["heads"], w["q_rank"], w["kv_rank"], w["q_main"], w["q_extra"],
                         w["value_dim"], w["eps"], *(a.ctypes.data for a in keep))
        out = np.empty((x.shape[0], w["hidden"]), np.float32)
        length = C.c_size_t(st["length"])
        for i in range(x.shape[0]):
            row = np.empty(w["hidden"], np.float32)
            self._check(self.lib.k3xo_mla_step(C.byref(ws), x[i], st["keys"], st["values"], st["shared"],
                                               st["keys"].shape[0], C.byref(length), row), "mla_step")
            out[i] = row
        st["length"] = length.value
        del keep
        return out, st

    def mla_tree(self, w: dict, state, parent, x):
        """A draft tree over the committed `state` (new: the reference
        verifies chains only): node i attends to the committed positions, its
        ancestors root first, and itself. Returns the outputs [nodes][H] and
        each node's key, value and shared key; the state is not changed."""
        x = _c(np.atleast_2d(x), np.float32)
        n = x.shape[0]
        par = np.ascontiguousarray(parent, np.int32)
        keep = [_c(w[k], np.float32) for k in MLA_TENSORS]
        ws = _MlaWeights(w["hidden"], w["heads"], w["q_rank"], w["kv_rank"], w["q_main"], w["q_extra"],
                         w["value_dim"], w["eps"], *(a.ctypes.data for a in keep))
        nk = np.empty((n, w["heads"], w["q_main"]), np.float32)
        nv = np.empty((n, w["heads"], w["value_dim"]), np.float32)
        ns = np.empty((n, w["q_extra"]), np.float32)
        out = np.empty((n, w["hidden"]), np.float32)
        self._check(self.lib.k3xo_mla_tree(C.byref(ws), state["keys"], state["values"], state["shared"],
                                           state["length"], par, n, x, nk, nv, ns, out), "mla_tree")
        del keep
        return out, nk, nv, ns

    def mla_crop(self, state, keep):
        """The rollback of rejected drafts (model.cpp:1235-1251)."""
        length = C.c_size_t(state["length"])
        self._check(self.lib.k3xo_mla_crop(C.byref(length), keep), "mla_crop")
        state["length"] = length.value
        return state

    def prepare_input(self, prefix, block, norm, proj, post, eps):
        """prepare_official_moe_input (official_moe.cpp:156-209) for one row:
        attention residual then RMSNorm."""
        return self.rms_norm(self.attention_residual(prefix, block, norm, proj, eps), post, eps)

    def kda_block_path(self, weights: dict, x, path, conv, recurrent):
        """The official block over the nodes of one root-to-node path (a
        linear sequence): outputs for those nodes and the state after the
        last. conv = (q, k, v) histories [(w-1)*P] bf16 words."""
        if len(path) == 0:
            return np.zeros((0, weights["hidden"]), np.float32), (*conv, recurrent)
        return self.kda_block(weights, x[list(path)], *conv, recurrent)

    @staticmethod
    def _path(parent, node):
        p = []
        while node >= 0:
            p.append(int(node))
            node = int(parent[node])
        return p[::-1]

    def kda_block_tree(self, weights: dict, x, parent, conv, recurrent):
        """Draft-tree semantics of the block (new; official_kda.cpp:198-426
        per path): node n's output is the block's output for n over the path
        root..n from the prefix state. Runs one path per leaf."""
        n = len(parent)
        has_child = np.zeros(n, bool)
        for i in range(n):
            if parent[i] >= 0:
                has_child[parent[i]] = True
        out = np.full((n, weights["hidden"]), np.nan, np.float32)
        for leaf in np.nonzero(~has_child)[0]:
            path = self._path(parent, leaf)
            o, _ = self.kda_block_path(weights, x, path, conv, recurrent)
            out[path] = o
        return out

    def kda_block_commit(self, weights: dict, x, parent, node, conv, recurrent):
        _, st = self.kda_block_path(weights, x, self._path(parent, node), conv, recurrent)
        return st

    def layer_forward(self, layer: dict, hidden_in, block, parent, conv, recurrent, want_xin=False):
        """official_layer_cpu (official_layer.cpp:134-244) with the plain MoE
        (official_moe.cpp:271-344 minus :296, :323-331) for one sequence's
        draft nodes [N][H]. Returns (out, expert ids, moe input)."""
        eps = layer["rms_eps"]
        N = hidden_in.shape[0]
        xin = np.stack([self.prepare_input(hidden_in[i], block[i], layer["self_residual_norm"],
                                           layer["self_residual_proj"], layer["input_norm"], eps)
                        for i in range(N)])
        kda_out = self.kda_block_tree(layer["kda"], xin, parent, conv, recurrent)
        prefix = self.round_bf16(self.round_bf16(hidden_in) + kda_out)
        moe_in = np.stack([self.prepare_input(prefix[i], block[i], layer["moe_residual_norm"],
                                              layer["moe_residual_proj"], layer["post_norm"], eps)
                           for i in range(N)])
        combined, ids, _ = self.moe_layer(layer["moe"], moe_in)
        out = self.round_bf16(self.round_bf16(prefix) + combined)
        return (out, ids, moe_in, xin) if want_xin else (out, ids, moe_in)

    def verify_greedy_stack(self, layers, lm_head, final_norm, final_eps, hidden_in, block, drafts, conv, rec):
        """One sequence's verify step (model.cpp:133-420 layer-major over the
        anchor + p linear drafts, LM head as bf16_matvec, targets by
        first-max argmax, speculative.cpp:74-112, then each layer's KDA state
        committed at node `accepted`). conv/rec: per-layer lists. Returns
        (logits [p+1][V], targets, accepted, committed, states)."""
        N = hidden_in.shape[0]
        parent = np.arange(-1, N - 1)
        x, xins = hidden_in, []
        for l, layer in enumerate(layers):
            x, _, _, xin = self.layer_forward(layer, x, block, parent, conv[l], rec[l], want_xin=True)
            xins.append(xin)
        if final_norm is not None:
            x = np.stack([self.rms_norm(x[i], final_norm, final_eps) for i in range(N)])
        logits = np.stack([self.bf16_matvec(x[i], lm_head) for i in range(N)])
        targets = np.array([self.argmax(logits[i]) for i in range(N)], np.uint32)
        V = lm_head.shape[0]
        accepted, committed = self.verify_greedy_block(0, drafts, len(drafts), V, targets)[:2]
        states = [self.kda_block_commit(layer["kda"], xins[l], parent, accepted, conv[l], rec[l])
                  for l, layer in enumerate(layers)]
        return logits, targets, accepted, committed, states

    def argmax(self, logits):
        logits = _c(logits, np.float32)
        return int(self.lib.k3xo_argmax(logits, logits.size))

    def verify_greedy_block(self, anchor, drafts, max_draft, vocab, targets):
        drafts = _c(drafts, np.uint32)
        acc, ncom, allacc = C.c_size_t(), C.c_size_t(), C.c_int()
        com = np.zeros(drafts.size + 1, np.uint32)
        self._check(self.lib.k3xo_verify_greedy_block(anchor, drafts, drafts.size, max_draft, vocab,
                                                      _c(targets, np.uint32), C.byref(acc), com,
                                                      C.byref(ncom), C.byref(allacc)),
                    "verify_greedy_block")
        return acc.value, com[:ncom.value].tolist(), bool(allacc.value)

    def uniform(self, seed, seq, pos, purpose):
        return self.lib.k3xo_uniform(seed, seq, pos, purpose)

    def verify_rejection(self, target_logits, draft_logits, drafts, temperature, seed, sequence):
        tl = _c(target_logits, np.float32)
        dl = _c(draft_logits, np.float32)
        drafts = _c(drafts, np.uint32)
        p = drafts.size
        V = tl.shape[-1]
        acc, ncom = C.c_size_t(), C.c_size_t()
        com = np.zeros(p + 1, np.uint32)
        self._check(self.lib.k3xo_verify_rejection(tl, dl if p else np.zeros(1, np.float32),
                                                   drafts if p else np.zeros(1, np.uint32), p, V,
                                                   temperature, seed, sequence, C.byref(acc), com,
                                                   C.byref(ncom)), "verify_rejection")
        return acc.value, com[:ncom.value].tolist()


_STEP_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_uint32, C.POINTER(C.c_uint32))


class Reference:
    """The reference's own CPU code (oracle/_ref/libk3x_ref.so)."""

    def __init__(self, path: str = REFERENCE_SO):
        L = C.CDLL(path)
        self.lib = L
        L.k3xr_decode_mxfp4.argtypes = [_u8p, _u8p, _sz, _sz, _sz, _f32p]
        L.k3xr_mxfp4_matmul.argtypes = [_f32p, _u8p, _u8p, _sz, _sz, _sz, _f32p]
        L.k3xr_situ_glu.argtypes = [_f32p, _f32p, _f32p, _sz, C.c_float, C.c_float]
        L.k3xr_rms_norm.argtypes = [_f32p, _f32p, _f32p, _sz, C.c_float]
        L.k3xr_rms_norm.restype = None
        L.k3xr_situ_glu.restype = None
        L.k3xr_route_official_moe.argtypes = [_f32p, _u16p, _sz, _sz, _f32p, _sz, _u32p, _f32p,
                                              C.c_void_p]
        L.k3xr_route_official_moe_logits.argtypes = [_f32p, _f32p, _sz, _sz, _u32p, _f32p,
                                                     C.c_void_p]
        L.k3xr_expert_major_plan.argtypes = [_u32p, _f32p, _u32p, _sz, _u32p, _u32p, _u32p, _u32p,
                                             _f32p, _szp]
        L.k3xr_verify_greedy_target_block.argtypes = [C.c_uint32, _u32p, _sz, _sz, _sz, _u32p,
                                                      _szp, _u32p, _szp, C.POINTER(C.c_int)]
        L.k3xr_verify_greedy_draft.argtypes = [C.c_uint32, _u32p, _sz, _sz, _sz, _STEP_FN,
                                               C.c_void_p, _szp, _u32p, _szp, C.POINTER(C.c_int)]
        L.k3xr_moe_layer_forward.argtypes = [C.c_void_p, _f32p, _sz, _sz, _f32p, _u32p, _f32p,
                                             C.c_int]
        L.k3xr_official_kda_cpu.argtypes = [C.c_void_p, _f32p, _sz, _u16p, _u16p, _u16p, _f32p,
                                            _f32p]
        L.k3xr_prepare_moe_input.argtypes = [_f32p, _f32p, _u16p, _u16p, _u16p, _sz, C.c_float, _f32p]
        L.k3xr_select_routing.argtypes = _SELECT_ROUTING_ARGS
        L.k3xr_official_moe.argtypes = [C.c_void_p, _f32p, _f32p, _u16p, _u16p, _u16p, C.c_float, _sz, _f32p,
                                        _u32p, _f32p]
        L.k3xr_official_two_layer.argtypes = [C.c_void_p] * 2 + [C.c_void_p, C.c_float, _f32p, _f32p] + \
            [C.c_void_p] * 4 + [_f32p]
        L.k3xr_dense_matvec.argtypes = [_f32p, _sz, _sz, _f32p, _f32p]
        L.k3xr_resident_moe_layer.argtypes = [_sz] * 4 + [_f32p] * 6 + [_u8p] * 6 + [_sz, _f32p, C.c_float, C.c_float,
                                                                                  C.c_float, _f32p, _f32p]
        L.k3xr_dense_situ_mlp.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _sz, _f32p, C.c_float, C.c_float, _f32p]
        L.k3xr_plain_layer.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, _sz, _sz, _f32p, _f32p,
                                       _u16p, _f32p, _f32p, _u32p, C.c_int, C.c_int]
        L.k3xr_official_layer.argtypes = [C.c_void_p, C.c_void_p, _u16p, _u16p, _u16p, _u16p, _u16p, _u16p,
                                          C.c_float, _f32p, _f32p, _sz, _u16p, _u16p, _u16p, _f32p, _f32p, _u32p]

    def decode_mxfp4(self, packed, scales, rows, cols, group=32):
        out = np.empty(rows * cols, np.float32)
        st = self.lib.k3xr_decode_mxfp4(_c(packed, np.uint8), _c(scales, np.uint8), rows, cols,
                                        group, out)
        if st:
            raise OracleError(st, "ref decode_mxfp4")
        return out.reshape(rows, cols)

    def mxfp4_matmul(self, x, packed, scales, rows, cols, group=32):
        out = np.empty(rows, np.float32)
        st = self.lib.k3xr_mxfp4_matmul(_c(x, np.float32), _c(packed, np.uint8),
                                        _c(scales, np.uint8), rows, cols, group, out)
        if st:
            raise OracleError(st, "ref mxfp4_matmul")
        return out

    def situ_glu(self, gate, up, beta, linear_beta=0.0):
        g, u = _c(gate, np.float32), _c(up, np.float32)
        out = np.empty_like(g)
        self.lib.k3xr_situ_glu(out, g, u, g.size, beta, linear_beta)
        return out

    def rms_norm_f32(self, x, weight, eps):
        """The reference's rms_norm (ops.cpp:10-18), float weights, one row."""
        x = _c(x, np.float32)
        out = np.empty_like(x)
        self.lib.k3xr_rms_norm(out, x, _c(weight, np.float32), x.size, eps)
        return out

    def dense_matvec(self, x, w):
        """The reference CPU backend's dense_matvec (make_cpu_backend)."""
        w = _c(w, np.float32)
        out = np.empty(w.shape[0], np.float32)
        st = self.lib.k3xr_dense_matvec(w, w.shape[0], w.shape[1], _c(x, np.float32), out)
        if st:
            raise OracleError(st, "ref dense_matvec")
        return out

    def resident_moe_layer(self, w: dict, experts: dict, contributions, x, eps, beta, linear_beta=0.0):
        """The CPU backend's resident_mxfp4_moe_layer (backend_cpu.cpp:305-339):
        w holds the f32 projections, experts the stacked MXFP4 arrays of the
        slots in route order (gate_packed [K][I][D/2], ...)."""
        D, H = w["routed_down"].shape
        S = w["shared_gate"].shape[0]
        K, I = experts["gate_packed"].shape[:2]
        out = np.empty(H, np.float32)
        st = self.lib.k3xr_resident_moe_layer(
            H, D, I, S, *(_c(w[k], np.float32) for k in ("routed_down", "routed_norm", "routed_up", "shared_gate",
                                                         "shared_up", "shared_down")),
            *(_c(experts[k], np.uint8) for k in ("gate_packed", "gate_scales", "up_packed", "up_scales",
                                                 "down_packed", "down_scales")),
            K, _c(contributions, np.float32), eps, beta, linear_beta, _c(x, np.float32), out)
        if st:
            raise OracleError(st, "ref resident_mxfp4_moe_layer")
        return out

    def dense_situ_mlp(self, x, gate, up, down, beta, linear_beta=0.0):
        gate, up, down = _c(gate, np.float32), _c(up, np.float32), _c(down, np.float32)
        out = np.empty(down.shape[0], np.float32)
        st = self.lib.k3xr_dense_situ_mlp(gate, up, down, gate.shape[0], gate.shape[1], down.shape[0],
                                          _c(x, np.float32), beta, linear_beta, out)
        if st:
            raise OracleError(st, "ref dense_situ_mlp")
        return out

    def route(self, hidden, router, correction, top_k, want_scores=False):
        router = _c(router, np.uint16)
        E, H = router.shape
        ids = np.empty(top_k, np.uint32)
        contrib = np.empty(top_k, np.float32)
        scores = np.empty(E, np.float32) if want_scores else None
        st = self.lib.k3xr_route_official_moe(_c(hidden, np.float32), router, E, H,
                                              _c(correction, np.float32), top_k, ids, contrib,
                                              _ptr(scores))
        if st:
            raise OracleError(st, "ref route_official_moe")
        return (ids, contrib, scores) if want_scores else (ids, contrib)

    def route_logits(self, logits, correction, top_k):
        logits = _c(logits, np.float32)
        ids = np.empty(top_k, np.uint32)
        contrib = np.empty(top_k, np.float32)
        st = self.lib.k3xr_route_official_moe_logits(logits, _c(correction, np.float32),
                                                     logits.size, top_k, ids, contrib, None)
        if st:
            raise OracleError(st, "ref route_official_moe_logits")
        return ids, contrib

    def expert_major_plan(self, ids_list, contrib_list):
        counts = np.array([len(x) for x in ids_list], np.uint32)
        ids = np.array([i for x in ids_list for i in x], np.uint32)
        con = np.array([c for x in contrib_list for c in x], np.float32)
        n = max(int(counts.sum()), 1)
        ge = np.zeros(n, np.uint32)
        go = np.zeros(n + 1, np.uint32)
        at = np.zeros(n, np.uint32)
        asl = np.zeros(n, np.uint32)
        ac = np.zeros(n, np.float32)
        ng = C.c_size_t(0)
        st = self.lib.k3xr_expert_major_plan(ids if ids.size else np.zeros(1, np.uint32),
                                             con if con.size else np.zeros(1, np.float32),
                                             counts if counts.size else np.zeros(1, np.uint32),
                                             len(ids_list), ge, go, at, asl, ac, C.byref(ng))
        if st:
            raise OracleError(st, "ref build_expert_major_plan")
        g = ng.value
        m = int(counts.sum())
        return dict(group_expert=ge[:g], group_offset=go[:g + 1], assign_token=at[:m],
                    assign_slot=asl[:m], assign_contrib=ac[:m])

    def verify_greedy_block(self, anchor, drafts, max_draft, vocab, targets):
        drafts = _c(drafts, np.uint32)
        acc, ncom, allacc = C.c_size_t(), C.c_size_t(), C.c_int()
        com = np.zeros(drafts.size + 1, np.uint32)
        st = self.lib.k3xr_verify_greedy_target_block(anchor,
                                                      drafts if drafts.size else np.zeros(1, np.uint32),
                                                      drafts.size, max_draft, vocab,
                                                      _c(targets, np.uint32), C.byref(acc), com,
                                                      C.byref(ncom), C.byref(allacc))
        if st:
            raise OracleError(st, "ref verify_greedy_target_block")
        return acc.value, com[:ncom.value].tolist(), bool(allacc.value)

    def verify_greedy_draft(self, anchor, drafts, max_draft, vocab, step):
        """step(input_token) -> (status, output_token)"""
        drafts = _c(drafts, np.uint32)

        def cb(_user, inp, outp):
            st, tok = step(int(inp))
            outp[0] = tok
            return st

        fn = _STEP_FN(cb)
        acc, ncom, allacc = C.c_size_t(), C.c_size_t(), C.c_int()
        com = np.zeros(drafts.size + 1, np.uint32)
        st = self.lib.k3xr_verify_greedy_draft(anchor,
                                               drafts if drafts.size else np.zeros(1, np.uint32),
                                               drafts.size, max_draft, vocab, fn, None,
                                               C.byref(acc), com, C.byref(ncom), C.byref(allacc))
        if st:
            raise OracleError(st, "ref verify_greedy_draft")
        return acc.value, com[:ncom.value].tolist(), bool(allacc.value)

    def moe_layer(self, layer: dict, hidden, token_begin=0, token_end=None, threads=1):
        hidden = _c(hidden, np.float32)
        T = hidden.shape[0]
        token_end = T if token_end is None else token_end
        s, keep = moe_struct(layer)
        out = np.zeros((T, layer["hidden"]), np.float32)
        ids = np.zeros((T, layer["top_k"]), np.uint32)
        contrib = np.zeros((T, layer["top_k"]), np.float32)
        st = self.lib.k3xr_moe_layer_forward(C.byref(s), hidden, token_begin, token_end, out, ids,
                                             contrib, threads)
        del keep
        if st:
            raise OracleError(st, "ref moe layer")
        return out, ids, contrib

    def select_routing(self, scores, bias, natural_k, **policy):
        return _select_routing(self.lib.k3xr_select_routing, scores, bias, natural_k, **policy)

    def official_moe(self, layer: dict, prefix, block, residual_norm, residual_proj, post_norm, eps):
        """official_moe_cpu (LatentMoE) for T positions with its own input
        preparation and routing: (out with the prefix residual, ids, contributions)."""
        prefix, block = _c(prefix, np.float32), _c(block, np.float32)
        T, H = prefix.shape
        s, keep = moe_struct(layer)
        out = np.zeros((T, H), np.float32)
        ids = np.zeros((T, layer["top_k"]), np.uint32)
        con = np.zeros((T, layer["top_k"]), np.float32)
        st = self.lib.k3xr_official_moe(C.byref(s), prefix, block, _c(residual_norm, np.uint16),
                                        _c(residual_proj, np.uint16), _c(post_norm, np.uint16), eps, T, out, ids,
                                        con)
        del keep
        if st:
            raise OracleError(st, "ref official_moe_cpu")
        return out, ids, con

    def official_layer(self, layer: dict, hidden_in, block, conv, recurrent):
        """official_layer_cpu (LatentMoE) over T positions of one sequence:
        (out [T][H], ids [T][k], (conv_q, conv_k, conv_v, recurrent) after)."""
        ks, keep_k = kda_struct(layer["kda"])
        ms, keep_m = moe_struct(layer["moe"])
        hidden_in, block = _c(hidden_in, np.float32), _c(block, np.float32)
        T, H = hidden_in.shape
        cq, ck, cv = (np.array(a, np.uint16, copy=True) for a in conv)
        rec = np.array(recurrent, np.float32, copy=True)
        out = np.zeros((T, H), np.float32)
        ids = np.zeros((T, layer["moe"]["top_k"]), np.uint32)
        st = self.lib.k3xr_official_layer(C.byref(ks), C.byref(ms), *(_c(layer[k], np.uint16) for k in (
            "self_residual_norm", "self_residual_proj", "input_norm", "moe_residual_norm", "moe_residual_proj",
            "post_norm")), layer["rms_eps"], hidden_in, block, T, cq, ck, cv, rec, out, ids)
        del keep_k, keep_m
        if st:
            raise OracleError(st, "ref official_layer_cpu")
        return out, ids, (cq, ck, cv, rec)

    def plain_layer(self, layer: dict, hidden_in, block, conv, recurrent, route_only=False, threads=1):
        """One KDA + plain-MoE layer through the reference's own functions
        (ref_shim.cpp:k3xr_plain_layer) for S sequences of T positions:
        hidden_in, block [S][T][H]; conv [S][3][(w-1)*P] bf16 words,
        recurrent [S][h][d][d] (copied, not changed). Returns (out [S][T][H],
        ids [S][T][k], conv after, recurrent after)."""
        ks, keep_k = kda_struct(layer["kda"])
        ms, keep_m = moe_struct(layer["moe"])
        hidden_in, block = _c(hidden_in, np.float32), _c(block, np.float32)
        S, T, H = hidden_in.shape
        conv = np.array(conv, np.uint16, copy=True)
        rec = np.array(recurrent, np.float32, copy=True)
        out = np.zeros((S, T, H), np.float32)
        ids = np.zeros((S, T, layer["moe"]["top_k"]), np.uint32)
        names = ("self_residual_norm", "self_residual_proj", "input_norm", "moe_residual_norm", "moe_residual_proj",
                 "post_norm")
        arrays = [_c(layer[k], np.uint16) for k in names]
        norms = (C.c_void_p * 6)(*[a.ctypes.data for a in arrays])
        st = self.lib.k3xr_plain_layer(C.byref(ks), C.byref(ms), norms, layer["rms_eps"], S, T, hidden_in, block,
                                       conv, rec, out, ids, 1 if route_only else 0, threads)
        del keep_k, keep_m, arrays
        if st:
            raise OracleError(st, "ref plain layer")
        return out, ids, conv, rec

    def official_two_layer(self, layers, hidden_in, block, convs, recs):
        """official_two_layer_cpu over its two positions: (out [2][H], final
        states per layer as (conv_q, conv_k, conv_v, recurrent))."""
        structs = [(kda_struct(L["kda"]), moe_struct(L["moe"])) for L in layers]
        kws = (C.c_void_p * 2)(*[C.cast(C.pointer(k[0]), C.c_void_p) for k, _ in structs])
        mws = (C.c_void_p * 2)(*[C.cast(C.pointer(m[0]), C.c_void_p) for _, m in structs])
        names = ("self_residual_norm", "self_residual_proj", "input_norm", "moe_residual_norm",
                 "moe_residual_proj", "post_norm")
        norm_arrays = [[_c(L[k], np.uint16) for k in names] for L in layers]
        norms = ((C.c_void_p * 6) * 2)(*[(C.c_void_p * 6)(*[a.ctypes.data for a in row]) for row in norm_arrays])
        states = [[np.array(a, np.uint16, copy=True) for a in conv] + [np.array(r, np.float32, copy=True)]
                  for conv, r in zip(convs, recs)]
        ptrs = [(C.c_void_p * 2)(*[states[l][i].ctypes.data for l in range(2)]) for i in range(4)]
        hidden_in, block = _c(hidden_in, np.float32), _c(block, np.float32)
        out = np.zeros_like(hidden_in)
        st = self.lib.k3xr_official_two_layer(kws, mws, norms, layers[0]["rms_eps"], hidden_in, block, *ptrs, out)
        del structs, norm_arrays
        if st:
            raise OracleError(st, "ref official_two_layer_cpu")
        return out, [tuple(s) for s in states]

    def prepare_input(self, prefix, block, norm, proj, post, eps):
        out = np.empty(len(prefix), np.float32)
        st = self.lib.k3xr_prepare_moe_input(_c(prefix, np.float32), _c(block, np.float32), _c(norm, np.uint16),
                                             _c(proj, np.uint16), _c(post, np.uint16), len(prefix), eps, out)
        if st:
            raise OracleError(st, "prepare_official_moe_input")
        return out

    def kda_block(self, weights: dict, hidden, conv_q, conv_k, conv_v, recurrent):
        s, keep = kda_struct(weights)
        hidden = _c(hidden, np.float32)
        T = hidden.size // weights["hidden"]
        cq, ck, cv = (np.array(a, np.uint16, copy=True) for a in (conv_q, conv_k, conv_v))
        rec = np.array(recurrent, np.float32, copy=True)
        out = np.empty(T * weights["hidden"], np.float32)
        st = self.lib.k3xr_official_kda_cpu(C.byref(s), hidden, T, cq, ck, cv, rec, out)
        del keep
        if st:
            raise OracleError(st, "ref official_kda_cpu")
        return out.reshape(T, weights["hidden"]), (cq, ck, cv, rec)


def have_reference() -> bool:
    return os.path.exists(REFERENCE_SO)


REFERENCE_B200_SO = os.path.join(HERE, "_ref", "libk3x_ref_b200.so")


class ReferenceOnB200:
    """The reference's own official_layer_cuda driving this library's
    ComputeBackend (oracle/_ref/libk3x_ref_b200.so, ref_b200.cpp): test
    infrastructure for the drop-in check, needs a B200."""

    def __init__(self, path: str = REFERENCE_B200_SO):
        L = C.CDLL(path)
        self.lib = L
        L.k3xr_official_layer_b200.argtypes = [C.c_int, C.c_int, _sz, C.c_void_p, C.c_void_p] + [_u16p] * 6 + [
            C.c_float, _f32p, _f32p, _sz, _u16p, _u16p, _u16p, _f32p, _f32p, _u32p, C.c_char_p, _sz]
        L.k3xr_official_two_layer_b200.argtypes = [C.c_int, C.c_int] + [C.c_void_p] * 2 + [C.c_void_p, C.c_float, _f32p,
                                                                                 _f32p] + [C.c_void_p] * 4 + [
            _f32p, _u32p, C.c_char_p, _sz]

    def official_layer(self, layer: dict, hidden_in, block, conv, recurrent, device=0, device_route=False,
                       kda_split=0):
        """official_layer_cuda(B200Backend) with host (or, device_route,
        device) route preparation; kda_split > 0 runs two calls, the KDA
        state kept on the device between them: the arguments and results of
        Reference.official_layer."""
        ks, keep_k = kda_struct(layer["kda"])
        ms, keep_m = moe_struct(layer["moe"])
        hidden_in, block = _c(hidden_in, np.float32), _c(block, np.float32)
        T, H = hidden_in.shape
        cq, ck, cv = (np.array(a, np.uint16, copy=True) for a in conv)
        rec = np.array(recurrent, np.float32, copy=True)
        out = np.zeros((T, H), np.float32)
        ids = np.zeros((T, layer["moe"]["top_k"]), np.uint32)
        err = C.create_string_buffer(512)
        st = self.lib.k3xr_official_layer_b200(device, 1 if device_route else 0, kda_split, C.byref(ks), C.byref(ms), *(_c(layer[k], np.uint16) for k in (
            "self_residual_norm", "self_residual_proj", "input_norm", "moe_residual_norm", "moe_residual_proj",
            "post_norm")), layer["rms_eps"], hidden_in, block, T, cq, ck, cv, rec, out, ids, err, len(err))
        del keep_k, keep_m
        if st:
            raise OracleError(st, "official_layer_cuda on B200Backend: " + err.value.decode(errors="replace"))
        return out, ids, (cq, ck, cv, rec)


    def official_two_layer(self, layers, hidden_in, block, convs, recs, device=0, device_closure=False):
        """official_two_layer_cuda(B200Backend) in its host_round_trip (or,
        device_closure, its front/tail) mode: the arguments and results of
        Reference.official_two_layer."""
        structs = [(kda_struct(L["kda"]), moe_struct(L["moe"])) for L in layers]
        kws = (C.c_void_p * 2)(*[C.cast(C.pointer(k[0]), C.c_void_p) for k, _ in structs])
        mws = (C.c_void_p * 2)(*[C.cast(C.pointer(m[0]), C.c_void_p) for _, m in structs])
        names = ("self_residual_norm", "self_residual_proj", "input_norm", "moe_residual_norm",
                 "moe_residual_proj", "post_norm")
        norm_arrays = [[_c(L[k], np.uint16) for k in names] for L in layers]
        norms = ((C.c_void_p * 6) * 2)(*[(C.c_void_p * 6)(*[a.ctypes.data for a in row]) for row in norm_arrays])
        states = [[np.array(a, np.uint16, copy=True) for a in conv] + [np.array(r, np.float32, copy=True)]
                  for conv, r in zip(convs, recs)]
        ptrs = [(C.c_void_p * 2)(*[states[l][i].ctypes.data for l in range(2)]) for i in range(4)]
        hidden_in, block = _c(hidden_in, np.float32), _c(block, np.float32)
        out = np.zeros_like(hidden_in)
        ids = np.zeros((2, 2, layers[0]["moe"]["top_k"]), np.uint32)
        err = C.create_string_buffer(512)
        st = self.lib.k3xr_official_two_layer_b200(device, 1 if device_closure else 0, kws, mws, norms,
                                                   layers[0]["rms_eps"], hidden_in, block, *ptrs, out, ids, err,
                                                   len(err))
        del structs, norm_arrays
        if st:
            raise OracleError(st, "official_two_layer_cuda on B200Backend: " + err.value.decode(errors="replace"))
        return out, [tuple(s) for s in states], ids


def have_reference_on_b200() -> bool:
    return os.path.exists(REFERENCE_B200_SO)


# ---------------------------------------------------------------------------
# seeded synthetic inputs shared by tests and bench (numpy; small sizes)
# ---------------------------------------------------------------------------

def bf16_words(x):
    """float32 -> bf16 words with the reference's round-to-nearest-even."""
    x = np.ascontiguousarray(x, np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)


def bf16_values(words):
    return (np.asarray(words, np.uint16).astype(np.uint32) << 16).view(np.float32)


def make_moe_layer(rs: Restatement, seed, hidden, inter, experts, top_k, shared_inter=0,
                   sigma=0.02, activation=ACT_SWIGLU, latent=0):
    """Synthetic MoE layer: N(0, sigma) weights, experts quantised to MXFP4
    with the restated quantiser, router/shared in bf16. latent > 0 makes a
    LatentMoE layer: routed_down [L][H], routed_norm [L] (1 + N(0, 0.1)),
    routed_up [H][L] in bf16, experts of width L."""
    g = np.random.default_rng(seed)
    D = latent or hidden

    def mx(rows, cols):
        w = g.normal(0.0, sigma, size=(rows, cols)).astype(np.float32)
        return rs.quantize_mxfp4(w)

    gp, gs, up_, us, dp, ds = [], [], [], [], [], []
    for _ in range(experts):
        a, b = mx(inter, D); gp.append(a); gs.append(b)
        a, b = mx(inter, D); up_.append(a); us.append(b)
        a, b = mx(D, inter); dp.append(a); ds.append(b)
    layer = dict(
        hidden=hidden, inter=inter, experts=experts, top_k=top_k, shared_inter=shared_inter,
        router=bf16_words(g.normal(0.0, sigma, size=(experts, hidden))),
        correction=g.normal(0.0, sigma, size=experts).astype(np.float32),
        gate_packed=np.stack(gp), gate_scales=np.stack(gs),
        up_packed=np.stack(up_), up_scales=np.stack(us),
        down_packed=np.stack(dp), down_scales=np.stack(ds),
        activation=activation, situ_beta=4.0, situ_linear_beta=25.0 if activation else 0.0,
    )
    if shared_inter:
        layer["shared_gate"] = bf16_words(g.normal(0.0, sigma, size=(shared_inter, hidden)))
        layer["shared_up"] = bf16_words(g.normal(0.0, sigma, size=(shared_inter, hidden)))
        layer["shared_down"] = bf16_words(g.normal(0.0, sigma, size=(hidden, shared_inter)))
    if latent:
        layer["latent"] = latent
        layer["latent_eps"] = 1e-6
        layer["routed_down"] = bf16_words(g.normal(0.0, 1.0 / np.sqrt(hidden), size=(latent, hidden)))
        layer["routed_norm"] = bf16_words(1.0 + g.normal(0.0, 0.1, size=latent))
        layer["routed_up"] = bf16_words(g.normal(0.0, sigma, size=(hidden, latent)))
    return layer


def make_resident_moe_case(rs: Restatement, seed, H=128, D=64, I=96, S=64, K=3):
    """Synthetic inputs of resident_mxfp4_moe_layer (backend_cpu.cpp:305-339):
    (f32 projections, stacked MXFP4 experts of K slots, contributions summing
    to 1, x [H])."""
    g = np.random.default_rng(seed)
    f32 = lambda *shape, s=0.05: g.normal(0, s, size=shape).astype(np.float32)
    w = dict(routed_down=f32(D, H), routed_norm=(1 + f32(D, s=0.1)).astype(np.float32), routed_up=f32(H, D),
             shared_gate=f32(S, H), shared_up=f32(S, H), shared_down=f32(H, S))
    ex = {}
    for name, rows, cols in (("gate", I, D), ("up", I, D), ("down", D, I)):
        pk, sc = zip(*[rs.quantize_mxfp4(f32(rows, cols, s=0.1)) for _ in range(K)])
        ex[f"{name}_packed"], ex[f"{name}_scales"] = np.stack(pk), np.stack(sc)
    con = g.random(K).astype(np.float32)
    con /= con.sum()
    return w, ex, con, g.normal(0, 1, size=H).astype(np.float32)


def bf16_normal(g, shape, sigma=1.0):
    return bf16_values(bf16_words(g.normal(0.0, sigma, size=shape).astype(np.float32)))


def make_kda_weights(g, hidden, heads, head_dim, conv_width=4, sigma=0.02):
    """Synthetic official KDA block weights (the dict kda_struct reads):
    projections N(0, sigma) in bf16, conv taps and gate parameters float."""
    P = heads * head_dim
    n = lambda *s: bf16_words(g.normal(0.0, sigma, size=s))
    return dict(hidden=hidden, heads=heads, head_dim=head_dim, conv_width=conv_width, eps=1e-5,
                gate_lower_bound=-5.0,
                q_proj=n(P, hidden), k_proj=n(P, hidden), v_proj=n(P, hidden),
                q_conv=g.normal(0.0, 0.5, size=(P, conv_width)).astype(np.float32),
                k_conv=g.normal(0.0, 0.5, size=(P, conv_width)).astype(np.float32),
                v_conv=g.normal(0.0, 0.5, size=(P, conv_width)).astype(np.float32),
                f_a_proj=n(head_dim, hidden), f_b_proj=bf16_words(g.normal(0.0, 0.1, size=(P, head_dim))),
                a_log=g.normal(0.0, 0.3, size=head_dim).astype(np.float32),
                dt_bias=g.normal(0.0, 0.3, size=P).astype(np.float32),
                b_proj=n(heads, hidden), g_proj=n(P, hidden),
                o_norm=np.ones(head_dim, np.float32), o_proj=n(hidden, P))


def make_layer(rs: Restatement, seed, hidden, heads, head_dim, experts, top_k, inter, shared_inter,
               conv_width=4, sigma=0.02, latent=0):
    """Synthetic KDA + MoE layer (BASELINE configs[0] recipe: N(0, sigma)
    weights, norms = 1, residual projections N(0, sigma), MXFP4 experts)."""
    g = np.random.default_rng(seed)
    ones = bf16_words(np.ones(hidden, np.float32))
    return dict(hidden=hidden, rms_eps=1e-6,
                self_residual_norm=ones, self_residual_proj=bf16_words(g.normal(0.0, sigma, size=hidden)),
                input_norm=ones, moe_residual_norm=ones,
                moe_residual_proj=bf16_words(g.normal(0.0, sigma, size=hidden)), post_norm=ones,
                kda=make_kda_weights(g, hidden, heads, head_dim, conv_width, sigma),
                moe=dict(make_moe_layer(rs, seed + 1000, hidden, inter, experts, top_k, shared_inter, sigma,
                                        latent=latent), latent_eps=1e-6))
