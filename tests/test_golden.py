"""The oracle restatement (oracle/k3x_oracle.c) against the golden fixtures
that the reference's own CPU code produced (tests/golden/make_golden.py):
bit for bit, with no reference tree or build needed. This is the pin that
travels: tests/test_oracle_pin.py checks the same functions against the
live reference build where it exists."""
import numpy as np

import golden_util as gu
from golden.make_golden import POLICIES


def test_route(rs):
    f = gu.load("route.npz")
    K = int(f["top_k"])
    for t in range(f["hidden"].shape[0]):
        ids, con, sco = rs.route_logits(rs.router_logits(f["hidden"][t], f["router"]), f["correction"], K,
                                        want_scores=True)
        np.testing.assert_array_equal(ids, f["ids"][t])
        np.testing.assert_array_equal(con, f["contributions"][t])
        np.testing.assert_array_equal(sco, f["scores"][t])


def test_expert_major_plan(rs):
    f = gu.load("expert_major.npz")
    p = rs.expert_major_plan(f["ids"], f["contributions"])
    for k in ("group_expert", "group_offset", "assign_token", "assign_slot", "assign_contrib"):
        np.testing.assert_array_equal(p[k], f[k], err_msg=k)


def test_mxfp4(rs):
    f = gu.load("mxfp4.npz")
    rows, cols = f["decoded"].shape
    np.testing.assert_array_equal(rs.decode_mxfp4(f["packed"], f["scales"], rows, cols), f["decoded"])
    np.testing.assert_array_equal(rs.mxfp4_matmul(f["x"], f["packed"], f["scales"], rows, cols), f["y"])


def test_moe_layer(rs):
    layer, hidden, out, ids, con = gu.moe_layer()
    got_out, got_ids, got_con = rs.moe_layer(layer, hidden)
    np.testing.assert_array_equal(got_ids, ids)
    np.testing.assert_array_equal(got_con, con)
    np.testing.assert_array_equal(got_out, out)


def test_kda_block(rs):
    w, f = gu.kda_block()
    out, (cq, ck, cv, r) = rs.kda_block(w, f["x"], f["conv_q"], f["conv_k"], f["conv_v"], f["recurrent"].ravel())
    np.testing.assert_array_equal(out, f["out"])
    np.testing.assert_array_equal(cq, f["next_conv_q"])
    np.testing.assert_array_equal(ck, f["next_conv_k"])
    np.testing.assert_array_equal(cv, f["next_conv_v"])
    np.testing.assert_array_equal(r.reshape(f["next_recurrent"].shape), f["next_recurrent"])


def test_kda_block_tree_restatement_on_the_chain(rs):
    """The draft-tree composition the GPU path is checked against, on a
    chain, reproduces the reference block's outputs."""
    w, f = gu.kda_block()
    T = f["x"].shape[0]
    got = rs.kda_block_tree(w, f["x"], np.arange(-1, T - 1), (f["conv_q"], f["conv_k"], f["conv_v"]),
                            f["recurrent"].ravel())
    np.testing.assert_array_equal(got, f["out"])


def test_prepare_input(rs):
    f = gu.load("prepare_input.npz")
    for t in range(f["prefix"].shape[0]):
        got = rs.prepare_input(f["prefix"][t], f["block"][t], f["norm"], f["proj"], f["post"], float(f["eps"]))
        np.testing.assert_array_equal(got, f["out"][t])


def test_select_routing(rs):
    f = gu.load("select_routing.npz")
    K = int(f["natural_k"])
    for i, pol in enumerate(POLICIES):
        for t in range(f["scores"].shape[0]):
            st, r = rs.select_routing(f["scores"][t], f["bias"], K, **pol)
            assert st == 0
            n = int(f[f"p{i}_selected"][t])
            assert r["selected_k"] == n, (i, t)
            np.testing.assert_array_equal(r["expert_ids"], f[f"p{i}_ids"][t, :n])
            np.testing.assert_array_equal(r["weights"], f[f"p{i}_weights"][t, :n])
            assert r["escalated"] == bool(f[f"p{i}_escalated"][t])
            stats = (r["normalized_entropy"], r["support"], r["mass"], r["boundary"])
            np.testing.assert_array_equal(np.array(stats, np.float32), f[f"p{i}_stats"][t])


def test_verify_greedy(rs):
    f = gu.load("verify_greedy.npz")
    p = f["drafts"].shape[1]
    for s in range(f["drafts"].shape[0]):
        a, com, _ = rs.verify_greedy_block(0, f["drafts"][s], p, int(f["vocab"]), f["targets"][s])
        assert a == f["accepted"][s]
        assert com == f["committed"][s, :f["count"][s]].tolist()


def test_latent_moe(rs):
    """LatentMoE: input preparation, routing, the latent layer and the
    prefix residual, restated, against official_moe_cpu's output."""
    layer, f = gu.latent_moe()
    eps = float(f["eps"])
    layer["latent_eps"] = eps
    T = f["prefix"].shape[0]
    hidden = np.stack([rs.prepare_input(f["prefix"][t], f["block"][t], f["residual_norm"], f["residual_proj"],
                                        f["post_norm"], eps) for t in range(T)])
    moe, ids, con = rs.moe_layer(layer, hidden)
    np.testing.assert_array_equal(ids, f["ids"])
    np.testing.assert_array_equal(con, f["contributions"])
    np.testing.assert_array_equal(rs.round_bf16(rs.round_bf16(f["prefix"]) + moe), f["out"])


def test_kda_known_answer(rs):
    """The reference's own KDA known-answer case (tests/cpp/test_official_kda.cpp,
    tests/python/test_cpp_parity.py): the restatement equals the reference's
    C++ official_kda_cpu bit for bit, equals its independent torch
    implementation to 1e-6 with identical conv-state words, and running the
    two positions one call at a time (the second from the first's state)
    gives the same outputs and state as one call over both."""
    from golden.make_golden import kda_kat_inputs
    f = gu.load("kda_kat.npz")
    w, hidden = kda_kat_inputs()
    z16, z32 = np.zeros(8, np.uint16), np.zeros(8, np.float32)
    out, (cq, ck, cv, r) = rs.kda_block(w, hidden, z16, z16, z16, z32)
    np.testing.assert_array_equal(out, f["out"])
    for got, key in ((cq, "conv_q"), (ck, "conv_k"), (cv, "conv_v"), (r, "recurrent")):
        np.testing.assert_array_equal(got, f[key])
    if "torch_out" in f:
        np.testing.assert_allclose(out, f["torch_out"], atol=1e-6, rtol=0)
        for got, key in ((cq, "conv_q"), (ck, "conv_k"), (cv, "conv_v")):
            np.testing.assert_array_equal(got, f["torch_" + key])
    o1, s1 = rs.kda_block(w, hidden[:1], z16, z16, z16, z32)
    o2, s2 = rs.kda_block(w, hidden[1:], *s1)
    np.testing.assert_array_equal(np.concatenate([o1, o2]), out)
    for a, b in zip(s2, (cq, ck, cv, r)):
        np.testing.assert_array_equal(a, b)


def test_official_layer_latent(rs):
    """The restated layer composition with LatentMoE against the reference's
    official_layer_cpu output, routes and final KDA state."""
    layer, f = gu.official_layer()
    T = f["hidden"].shape[0]
    parent = np.arange(-1, T - 1)
    conv = (f["conv_q"], f["conv_k"], f["conv_v"])
    out, ids, _, xin = rs.layer_forward(layer, f["hidden"], f["block"], parent, conv, f["recurrent"], want_xin=True)
    np.testing.assert_array_equal(ids, f["ids"])
    np.testing.assert_array_equal(out, f["out"])
    state = rs.kda_block_commit(layer["kda"], xin, parent, T - 1, conv, f["recurrent"])
    for a, key in zip(state, ("next_conv_q", "next_conv_k", "next_conv_v", "next_recurrent")):
        np.testing.assert_array_equal(a, f[key])
