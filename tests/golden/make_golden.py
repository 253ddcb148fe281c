"""Generates the golden fixtures in this folder from the reference's own CPU
code: oracle/_ref/libk3x_ref.so, compiled by `make -C oracle` from the
reference's unmodified runtime sources (ops.cpp, official_moe.cpp,
official_kda.cpp, expert_major.cpp, speculative.cpp, routing_policy.cpp)
where they lie. Inputs are seeded synthetic data at the c1 dimensions; each
fixture stores inputs and the reference's outputs, so the oracle pin
(tests/test_golden.py) and the GPU parity tests (tests/test_gpu_golden.py)
run where neither the reference tree nor its build exists.

Run from the repository root: python tests/golden/make_golden.py [fixture function ...]
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "oracle")]

from oracle import (ROUTING_ADAPTIVE, ROUTING_FIXED, ROUTING_NATURAL, Reference, Restatement,  # noqa: E402
                    bf16_normal, bf16_words, make_kda_weights, make_layer, make_moe_layer)

MOE = dict(hidden=256, inter=128, experts=8, top_k=2, shared_inter=128)
KDA = dict(hidden=256, heads=2, head_dim=64, conv_width=4, tokens=5)


def save(name, **arrays):
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **{k: np.asarray(v) for k, v in arrays.items()})
    print(f"{name}: {os.path.getsize(path)} bytes")


def route(ref):
    """route_official_moe (official_moe.cpp:247-269) for 6 tokens."""
    g = np.random.default_rng(1001)
    T, E, H, K = 6, 16, 256, 4
    hidden = bf16_normal(g, (T, H))
    router = bf16_words(g.normal(0, 0.02, size=(E, H)))
    correction = g.normal(0, 0.02, size=E).astype(np.float32)
    ids, con, sco = zip(*(ref.route(hidden[t], router, correction, K, want_scores=True) for t in range(T)))
    save("route.npz", hidden=hidden, router=router, correction=correction, top_k=K,
         ids=np.stack(ids), contributions=np.stack(con), scores=np.stack(sco))


def expert_major(ref):
    """build_expert_major_plan (expert_major.cpp:10-54) for 12 tokens x 3 slots."""
    g = np.random.default_rng(1002)
    T, K, E = 12, 3, 10
    ids = np.stack([g.choice(E, size=K, replace=False) for _ in range(T)]).astype(np.uint32)
    con = g.random((T, K)).astype(np.float32)
    p = ref.expert_major_plan(ids.tolist(), con.tolist())
    save("expert_major.npz", ids=ids, contributions=con, experts=E, **p)


def mxfp4(ref, rs):
    """decode_mxfp4 / mxfp4_matmul (ops.cpp:32-76) of a 64 x 256 matrix."""
    g = np.random.default_rng(1003)
    rows, cols = 64, 256
    packed, scales = rs.quantize_mxfp4(g.normal(0, 0.02, size=(rows, cols)).astype(np.float32))
    x = bf16_normal(g, (cols,))
    save("mxfp4.npz", packed=packed, scales=scales, x=x,
         decoded=ref.decode_mxfp4(packed, scales, rows, cols), y=ref.mxfp4_matmul(x, packed, scales, rows, cols))


def moe_layer(ref, rs):
    """The plain hidden-space MoE layer (official_moe.cpp:271-344 without the
    latent steps) composed from the reference's exported functions."""
    d = MOE
    layer = make_moe_layer(rs, 1004, d["hidden"], d["inter"], d["experts"], d["top_k"], d["shared_inter"])
    hidden = bf16_normal(np.random.default_rng(1005), (5, d["hidden"]))
    out, ids, con = ref.moe_layer(layer, hidden)
    arrays = {k: v for k, v in layer.items() if isinstance(v, np.ndarray)}
    dims = {k: v for k, v in layer.items() if not isinstance(v, np.ndarray)}
    save("moe_layer.npz", hidden=hidden, out=out, ids=ids, contributions=con,
         **arrays, **{f"dim_{k}": v for k, v in dims.items()})


def latent_moe(ref, rs):
    """official_moe_cpu (official_moe.cpp:271-344, LatentMoE) with its own
    input preparation and routing, for 4 positions."""
    d = dict(MOE, experts=8, top_k=2, latent=128)
    layer = make_moe_layer(rs, 1011, d["hidden"], d["inter"], d["experts"], d["top_k"], d["shared_inter"],
                           latent=d["latent"])
    g = np.random.default_rng(1012)
    T, H, eps = 4, d["hidden"], 1e-6
    prefix, block = bf16_normal(g, (T, H)), bf16_normal(g, (T, H))
    norm = bf16_words(1.0 + g.normal(0, 0.1, size=H))
    proj = bf16_words(g.normal(0, 0.05, size=H))
    post = bf16_words(1.0 + g.normal(0, 0.1, size=H))
    out, ids, con = ref.official_moe(layer, prefix, block, norm, proj, post, eps)
    arrays = {k: v for k, v in layer.items() if isinstance(v, np.ndarray)}
    dims = {k: v for k, v in layer.items() if not isinstance(v, np.ndarray)}
    save("latent_moe.npz", prefix=prefix, block=block, residual_norm=norm, residual_proj=proj, post_norm=post,
         eps=eps, out=out, ids=ids, contributions=con, **arrays, **{f"dim_{k}": v for k, v in dims.items()})


def kda_block(ref):
    """official_kda_cpu (official_kda.cpp:198-426) over 5 positions from a
    non-zero state."""
    d = KDA
    g = np.random.default_rng(1006)
    P = d["heads"] * d["head_dim"]
    w = make_kda_weights(g, d["hidden"], d["heads"], d["head_dim"], d["conv_width"])
    conv = [bf16_words(g.normal(0, 0.5, size=(d["conv_width"] - 1) * P)) for _ in range(3)]
    rec = g.normal(0, 0.05, size=(d["heads"], d["head_dim"], d["head_dim"])).astype(np.float32)
    x = bf16_normal(g, (d["tokens"], d["hidden"]))
    out, (cq, ck, cv, r) = ref.kda_block(w, x, conv[0], conv[1], conv[2], rec.ravel())
    arrays = {f"w_{k}": v for k, v in w.items() if isinstance(v, np.ndarray)}
    dims = {f"dim_{k}": v for k, v in w.items() if not isinstance(v, np.ndarray)}
    save("kda_block.npz", x=x, conv_q=conv[0], conv_k=conv[1], conv_v=conv[2], recurrent=rec, out=out,
         next_conv_q=cq, next_conv_k=ck, next_conv_v=cv, next_recurrent=r.reshape(rec.shape), **arrays, **dims)


def official_layer(ref, rs):
    """official_layer_cpu (official_layer.cpp:134-244) with LatentMoE over
    5 positions from a non-zero KDA state (one epsilon for every norm, as
    the reference's OfficialKdaConfig has)."""
    g = np.random.default_rng(1013)
    H, h, d, T, W = 256, 2, 64, 5, 4
    layer = make_layer(rs, 1014, H, h, d, 8, 2, 128, 128, latent=128)
    layer["moe"]["latent_eps"] = layer["kda"]["eps"] = layer["rms_eps"]
    hidden, block = bf16_normal(g, (T, H)), bf16_normal(g, (T, H))
    conv = [bf16_words(g.normal(0, 0.5, size=(W - 1) * h * d)) for _ in range(3)]
    rec = g.normal(0, 0.05, size=h * d * d).astype(np.float32)
    out, ids, (cq, ck, cv, r) = ref.official_layer(layer, hidden, block, conv, rec)
    arrays = {f"norm_{k}": layer[k] for k in ("self_residual_norm", "self_residual_proj", "input_norm",
                                              "moe_residual_norm", "moe_residual_proj", "post_norm")}
    arrays.update({f"kda_{k}": v for k, v in layer["kda"].items()})
    arrays.update({f"moe_{k}": v for k, v in layer["moe"].items()})
    save("official_layer.npz", rms_eps=layer["rms_eps"], hidden=hidden, block=block, conv_q=conv[0], conv_k=conv[1],
         conv_v=conv[2], recurrent=rec, out=out, ids=ids, next_conv_q=cq, next_conv_k=ck, next_conv_v=cv,
         next_recurrent=r, **arrays)


def kda_kat_inputs():
    """The known-answer case of the reference's tests/cpp/test_official_kda.cpp
    (and tests/python/test_cpp_parity.py): H 4, 2 heads of 2, conv width 3,
    eps 1e-5, gate lower bound -5, zero state, two positions."""
    eye = np.eye(4, dtype=np.float32)
    conv = np.array([[0.25, -0.5, 1.0], [-0.25, 0.5, 0.75], [0.5, 0.25, -0.5], [-0.5, 0.25, 1.25]], np.float32)
    w = dict(hidden=4, heads=2, head_dim=2, conv_width=3, eps=1e-5, gate_lower_bound=-5.0,
             q_proj=bf16_words(eye),
             k_proj=bf16_words(np.array([[0.5, 0, 0.25, 0], [0, 0.75, 0, -0.25], [0.25, 0, 1, 0], [0, -0.5, 0, 0.5]])),
             v_proj=bf16_words(eye), q_conv=conv, k_conv=(conv * 0.75).astype(np.float32),
             v_conv=(conv * -0.5).astype(np.float32),
             f_a_proj=bf16_words(np.array([[0.5, -0.25, 0, 0.25], [0, 0.5, -0.5, 0.25]])),
             f_b_proj=bf16_words(np.array([[1, 0], [0.5, -0.5], [0, 1], [-0.25, 0.75]])),
             a_log=np.array([0.0, 0.5], np.float32), dt_bias=np.array([0.25, -0.5, 0.75, -0.25], np.float32),
             b_proj=bf16_words(np.array([[0.5, -0.25, 0.25, 0], [0, 0.5, -0.5, 0.25]])),
             g_proj=bf16_words(np.array([[0.5, 0, 0, -0.25], [0, 0.5, 0.25, 0], [-0.25, 0, 0.5, 0], [0, 0.25, 0, 0.75]])),
             o_norm=np.array([1.0, 1.5], np.float32), o_proj=bf16_words(eye))
    hidden = np.array([[0.5, -1.0, 0.25, 0.75], [-0.25, 0.5, 1.0, -0.5]], np.float32)
    return w, hidden


def kda_kat(ref):
    """The reference's KDA known-answer case through its C++ official_kda_cpu
    and, where the reference tree is importable, its independent torch
    implementation (reference/k3x_ref/official_kda.py)."""
    w, hidden = kda_kat_inputs()
    z16 = np.zeros(2 * 4, np.uint16)
    out, (cq, ck, cv, r) = ref.kda_block(w, hidden, z16, z16, z16, np.zeros(8, np.float32))
    arrays = dict(out=out, conv_q=cq, conv_k=ck, conv_v=cv, recurrent=r)
    torch_ref = _torch_kda(w, hidden)
    if torch_ref is not None:
        arrays.update({f"torch_{k}": v for k, v in torch_ref.items()})
    save("kda_kat.npz", **arrays)


def _torch_kda(w, hidden):
    # the reference tree: K3X_REFERENCE, else a checkout beside this repository (oracle/Makefile's rule)
    ref_root = os.environ.get("K3X_REFERENCE") or os.path.abspath(os.path.join(ROOT, "..", "reference"))
    pkg = os.path.join(ref_root, "reference")
    if not os.path.isdir(os.path.join(pkg, "k3x_ref")):
        return None
    sys.path.insert(0, pkg)
    import torch
    from k3x_ref.official_kda import (OfficialKdaConfig, OfficialKdaWeights, official_kda,
                                      zero_official_kda_state)
    bf = lambda a: torch.from_numpy((np.asarray(a, np.uint32) << 16).view(np.float32).copy()).to(torch.bfloat16)
    f32 = lambda a: torch.from_numpy(np.asarray(a, np.float32).copy())
    cfg = OfficialKdaConfig(4, 2, 2, 3, 1.0e-5, -5.0)
    weights = OfficialKdaWeights(
        q_proj=bf(w["q_proj"]), k_proj=bf(w["k_proj"]), v_proj=bf(w["v_proj"]),
        q_conv=f32(w["q_conv"]), k_conv=f32(w["k_conv"]), v_conv=f32(w["v_conv"]),
        f_a_proj=bf(w["f_a_proj"]), f_b_proj=bf(w["f_b_proj"]), a_log=f32(w["a_log"]), dt_bias=f32(w["dt_bias"]),
        b_proj=bf(w["b_proj"]), g_proj=bf(w["g_proj"]), o_norm=f32(w["o_norm"]), o_proj=bf(w["o_proj"]))
    x = torch.from_numpy(hidden).to(torch.bfloat16).reshape(1, 2, 4)
    res = official_kda(x, weights, zero_official_kda_state(cfg, 1, x.device), cfg)
    words = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16).reshape(-1)
    return dict(out=res.output.float().numpy().reshape(2, 4), conv_q=words(res.state.conv_q),
                conv_k=words(res.state.conv_k), conv_v=words(res.state.conv_v))


def prepare_input(ref):
    """prepare_official_moe_input (official_moe.cpp:156-209) for 4 rows."""
    g = np.random.default_rng(1007)
    T, H, eps = 4, 256, 1e-6
    prefix, block = bf16_normal(g, (T, H)), bf16_normal(g, (T, H))
    norm = bf16_words(1.0 + g.normal(0, 0.1, size=H))
    proj = bf16_words(g.normal(0, 0.02, size=H))
    post = bf16_words(1.0 + g.normal(0, 0.1, size=H))
    out = np.stack([ref.prepare_input(prefix[t], block[t], norm, proj, post, eps) for t in range(T)])
    save("prepare_input.npz", prefix=prefix, block=block, norm=norm, proj=proj, post=post, eps=eps, out=out)


POLICIES = [
    dict(mode=ROUTING_NATURAL),
    dict(mode=ROUTING_FIXED, fixed_k=8),
    dict(mode=ROUTING_FIXED, fixed_k=4, quality_floor_k=6),
    dict(mode=ROUTING_ADAPTIVE, mass_target=0.5, minimum_gap=0.0),
    dict(mode=ROUTING_ADAPTIVE, mass_target=0.9, minimum_gap=0.02, quality_floor_k=8),
]


def select_routing(ref):
    """select_routing (routing_policy.cpp:31-159): 8 tokens x 64 experts,
    natural Top-16, each policy of POLICIES."""
    g = np.random.default_rng(1008)
    T, E, K = 8, 64, 16
    scores = (1.0 / (1.0 + np.exp(-g.normal(0, 1.5, size=(T, E))))).astype(np.float32)
    bias = g.normal(0, 0.05, size=E).astype(np.float32)
    arrays = dict(scores=scores, bias=bias, natural_k=K)
    for i, pol in enumerate(POLICIES):
        ids = np.full((T, K), 0xFFFFFFFF, np.uint32)
        wts = np.zeros((T, K), np.float32)
        sel = np.zeros(T, np.uint32)
        esc = np.zeros(T, np.uint32)
        stats = np.zeros((T, 4), np.float32)
        for t in range(T):
            st, r = ref.select_routing(scores[t], bias, K, **pol)
            assert st == 0, st
            n = r["selected_k"]
            ids[t, :n], wts[t, :n], sel[t], esc[t] = r["expert_ids"], r["weights"], n, r["escalated"]
            stats[t] = (r["normalized_entropy"], r["support"], r["mass"], r["boundary"])
        arrays.update({f"p{i}_ids": ids, f"p{i}_weights": wts, f"p{i}_selected": sel, f"p{i}_escalated": esc,
                       f"p{i}_stats": stats})
    save("select_routing.npz", **arrays)


def verify_greedy(ref):
    """verify_greedy_target_block (speculative.cpp:74-112): 6 sequences of
    anchor + 5 drafts over vocab 1000, accepting 0..5 drafts."""
    g = np.random.default_rng(1009)
    S, p, V = 6, 5, 1000
    drafts = g.integers(0, V, size=(S, p)).astype(np.uint32)
    targets = g.integers(0, V, size=(S, p + 1)).astype(np.uint32)
    accepted = np.zeros(S, np.uint32)
    committed = np.zeros((S, p + 1), np.uint32)
    count = np.zeros(S, np.uint32)
    for s in range(S):
        targets[s, :s] = drafts[s, :s]            # sequence s accepts exactly s drafts
        if s < p:
            targets[s, s] = (drafts[s, s] + 1) % V
        a, com, _ = ref.verify_greedy_block(0, drafts[s], p, V, targets[s])
        accepted[s], count[s] = a, len(com)
        committed[s, :len(com)] = com
    save("verify_greedy.npz", drafts=drafts, targets=targets, vocab=V, accepted=accepted, committed=committed,
         count=count)


def block_attn_res(ref, rs):
    """The block attention residual with many sources (model.cpp:645-666):
    the reference's torch form (reference/k3x_ref/attn_res.py:9-23) on 5 rows
    x 3 sources, and the reference's own known-answer case
    (tests/python/test_attn_res.py). The torch form sums in its own order,
    so it is a float-tolerance pin for the restatement. Skipped when the
    reference tree is not importable."""
    ref_root = os.environ.get("K3X_REFERENCE") or os.path.abspath(os.path.join(ROOT, "..", "reference"))
    pkg = os.path.join(ref_root, "reference")
    if not os.path.isdir(os.path.join(pkg, "k3x_ref")):
        print("block_attn_res: reference tree not found, skipped")
        return
    sys.path.insert(0, pkg)
    import torch
    from k3x_ref.attn_res import apply_attn_res
    g = np.random.default_rng(1013)
    T, S, H, eps = 5, 3, 256, 1e-6
    scale = np.array([0.5, 1.0, 2.0, 4.0], np.float32)[:, None, None]
    values = (g.normal(size=(S + 1, T, H)) * scale).astype(np.float32)
    sources, prefix = values[:S], values[S]
    norm = (1.0 + 0.1 * g.normal(size=H)).astype(np.float32)
    proj = (g.normal(size=H) / np.sqrt(H)).astype(np.float32)
    got = apply_attn_res(torch.from_numpy(prefix), torch.from_numpy(np.ascontiguousarray(sources.transpose(1, 0, 2))),
                         torch.from_numpy(norm), torch.from_numpy(proj), eps).numpy()
    kat = apply_attn_res(torch.tensor([[1.0, 1.0]]), torch.tensor([[[3.0, 0.0], [0.0, 4.0]]]), torch.ones(2),
                         torch.tensor([1.0, 0.0]), 0.0).numpy()
    save("block_attn_res.npz", prefix=prefix, sources=sources, norm=norm, proj=proj, eps=np.float32(eps),
         torch_out=got, kat_out=kat)


def mla(ref, rs):
    """The gated MLA (model.cpp:755-811) through the reference's torch form
    (reference/k3x_ref/mla.py: mla_prefill, NoPE with a shared extra key) at
    the reference's default synthetic config, 5 positions from an empty
    state: outputs and the final keys, values and shared keys (position-major
    here). The torch form sums in its own order, so it is a float-tolerance
    pin. Skipped when the reference tree is not importable."""
    ref_root = os.environ.get("K3X_REFERENCE") or os.path.abspath(os.path.join(ROOT, "..", "reference"))
    pkg = os.path.join(ref_root, "reference")
    if not os.path.isdir(os.path.join(pkg, "k3x_ref")):
        print("mla: reference tree not found, skipped")
        return
    sys.path.insert(0, pkg)
    import torch
    from k3x_ref.config import SyntheticK3Config
    from k3x_ref.mla import MLAWeights, mla_prefill
    cfg = SyntheticK3Config.default()
    H, nh, qr, kr = cfg.hidden_size, cfg.mla_heads, cfg.q_lora_rank, cfg.kv_lora_rank
    qm, qe, vd = cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim
    g = np.random.default_rng(1019)
    f = lambda *shape, sd=0.15: (g.normal(0, sd, size=shape)).astype(np.float32)
    w = dict(q_a_proj=f(qr, H), q_a_norm=(1 + f(qr, sd=0.1)), q_b_proj=f(nh * (qm + qe), qr),
             kv_a_proj=f(kr + qe, H), kv_a_norm=(1 + f(kr, sd=0.1)), kv_b_proj=f(nh * (qm + vd), kr),
             g_proj=f(nh * vd, H), o_proj=f(H, nh * vd))
    x = g.normal(size=(5, H)).astype(np.float32)
    t = {k: torch.from_numpy(v) for k, v in w.items()}
    out, st = mla_prefill(torch.from_numpy(x).reshape(1, 5, H), MLAWeights(**t), None, cfg)
    save("mla.npz", x=x, eps=np.float32(cfg.rms_norm_eps),
         dims=np.array([H, nh, qr, kr, qm, qe, vd], np.int64), torch_out=out.reshape(5, H).numpy(),
         torch_keys=st.keys[0].transpose(0, 1).numpy(), torch_values=st.values[0].transpose(0, 1).numpy(),
         torch_shared=st.shared_keys[0, 0].numpy(), **w)


def main():
    ref, rs = Reference(), Restatement()
    if len(sys.argv) > 1:   # named fixtures only
        for name in sys.argv[1:]:
            fn = globals()[name]
            fn(*[a for a, p in ((ref, "ref"), (rs, "rs")) if p in fn.__code__.co_varnames[:fn.__code__.co_argcount]])
        return
    route(ref)
    expert_major(ref)
    mxfp4(ref, rs)
    moe_layer(ref, rs)
    latent_moe(ref, rs)
    kda_block(ref)
    kda_kat(ref)
    official_layer(ref, rs)
    prepare_input(ref)
    select_routing(ref)
    verify_greedy(ref)
    block_attn_res(ref, rs)
    mla(ref, rs)


if __name__ == "__main__":
    main()
