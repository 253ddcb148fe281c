"""The full KDA block and the KDA + MoE layer on the GPU (through the C ABI)
against the oracle's composition of pinned pieces.

The block's projections run on tensor cores with FP32 accumulation where
the reference accumulates in FP64 and rounds to bf16, so a projection
output occasionally lands on the other side of a bf16 rounding midpoint;
the recurrence carries that forward. Outputs and states are therefore held
to the north-star hidden-state tolerance (rel 2e-2 / abs 1e-3) with a small
fraction of elements allowed a few bf16 steps (assert_mostly_close).
The commit replay is bit-identical to the verify pass (checked exactly).
"""
import numpy as np
import pytest

from gpu_util import layer_to_dev, to_dev, torch_cuda
from oracle import bf16_normal, bf16_words, make_kda_weights, make_layer

pytestmark = pytest.mark.gpu

C1 = dict(hidden=256, heads=4, head_dim=64, experts=16, top_k=4, inter=128, shared_inter=128)


@pytest.fixture(scope="module")
def torch():
    return torch_cuda()


@pytest.fixture(scope="module")
def ctx(torch):
    import k3xb
    c = k3xb.Context(0)
    c.use_stream()
    yield c
    c.close()


def assert_mostly_close(got, want, rtol=2e-2, atol=1e-3, max_frac=0.01, loose=8.0, what=""):
    err = np.abs(got - want)
    tol = atol + rtol * np.abs(want)
    frac = float((err > tol).mean())
    worst = float((err / tol).max())
    assert frac <= max_frac and worst <= loose, (
        f"{what}: {frac:.4f} of elements beyond rel {rtol}/abs {atol}; worst {worst:.2f}x tolerance; "
        f"max|err| {err.max():.3e}")


def _kda_dev(torch, w):
    d = {k: (to_dev(torch, v) if isinstance(v, np.ndarray) else v) for k, v in w.items()}
    return d


def _states(g, S, h, d, W, P):
    conv = np.stack([np.stack([bf16_words(g.normal(0, 0.5, size=(W - 1) * P)) for _ in range(3)])
                     for _ in range(S)])                          # [S][3][(w-1)*P]
    rec = g.normal(0, 0.05, size=(S, h, d, d)).astype(np.float32)
    return conv, rec


def test_attention_residual_norm(torch, ctx, rs):
    g = np.random.default_rng(5)
    for T, H in ((9, 256), (3, 7168)):
        a = bf16_normal(g, (T, H))
        delta = bf16_normal(g, (T, H), 0.3)
        block = bf16_normal(g, (T, H))
        norm = bf16_words(1 + g.normal(0, 0.1, size=H))
        proj = bf16_words(g.normal(0, 0.05, size=H))
        post = bf16_words(1 + g.normal(0, 0.1, size=H))
        out = torch.empty((T, H), dtype=torch.float32, device="cuda")
        pre = torch.empty((T, H), dtype=torch.float32, device="cuda")
        dv = lambda x: to_dev(torch, x)
        ctx.attention_residual_norm(dv(a), dv(block), dv(norm), dv(proj), dv(post), 1e-6, out)
        ctx.sync()
        got = out.cpu().numpy()
        want = np.stack([rs.prepare_input(a[t], block[t], norm, proj, post, 1e-6) for t in range(T)])
        # tree vs sequential FP64 sums: the float score/inverse may differ in the last bit
        assert (got != want).mean() < 0.01
        assert_mostly_close(got, want, what="attention residual")
        ctx.attention_residual_norm(dv(a), dv(block), dv(norm), dv(proj), dv(post), 1e-6, out, delta=dv(delta),
                                    prefix_out=pre)
        ctx.sync()
        prefix = rs.round_bf16(rs.round_bf16(a) + delta)
        np.testing.assert_array_equal(pre.cpu().numpy(), prefix)
        want = np.stack([rs.prepare_input(prefix[t], block[t], norm, proj, post, 1e-6) for t in range(T)])
        assert_mostly_close(out.cpu().numpy(), want, what="attention residual with delta")


@pytest.mark.parametrize("parent", [
    [-1, 0, 1, 2, 3],                 # anchor + 4 linear drafts
    [-1, 0, 0, 1, 1, 2, 5],           # a tree, depth 4
    [-1, 0, -1, 2],                   # two roots (a forest)
])
def test_kda_block_vs_oracle(torch, ctx, rs, parent):
    import k3xb
    g = np.random.default_rng(len(parent))
    H, h, d, W, S = C1["hidden"], C1["heads"], C1["head_dim"], 4, 2
    P, N = h * d, len(parent)
    w = make_kda_weights(g, H, h, d, W)
    conv, rec = _states(g, S, h, d, W, P)
    x = bf16_normal(g, (S, N, H))
    wd = _kda_dev(torch, w)
    desc = k3xb.kda_layer_desc(wd)
    out = torch.empty((S, N, H), dtype=torch.float32, device="cuda")
    trace = torch.empty(ctx.kda_trace_bytes(desc, N, S), dtype=torch.uint8, device="cuda")
    conv_d, rec_d = to_dev(torch, conv), to_dev(torch, rec)
    ctx.kda_block(desc, to_dev(torch, x), parent, conv_d, rec_d, out, trace)
    # commit: sequence 0 at the deepest node, sequence 1 keeps the prefix
    commit = [N - 1, -1]
    conv_out = torch.empty_like(conv_d)
    rec_out = torch.empty_like(rec_d)
    ctx.kda_block_commit(desc, trace, parent, S, commit, conv_d, rec_d, conv_out, rec_out)
    ctx.sync()
    got = out.cpu().numpy()
    par = np.array(parent)
    for s in range(S):
        cs = tuple(conv[s, i] for i in range(3))
        want = rs.kda_block_tree(w, x[s], par, cs, rec[s].ravel())
        assert_mostly_close(got[s], want, what=f"KDA block, sequence {s}")
    co, ro = conv_out.cpu().numpy().view(np.uint16), rec_out.cpu().numpy()
    np.testing.assert_array_equal(co[1], conv[1])
    np.testing.assert_array_equal(ro[1], rec[1])
    cq, ck, cv, r = rs.kda_block_commit(w, x[0], par, commit[0], tuple(conv[0, i] for i in range(3)),
                                        rec[0].ravel())
    for i, want_rows in enumerate((cq, ck, cv)):
        assert_mostly_close(bf16_to_f32(co[0, i]), bf16_to_f32(want_rows), what=f"conv history {i}")
    assert_mostly_close(ro[0].ravel(), r, what="recurrent state")


def bf16_to_f32(words):
    return (np.asarray(words, np.uint16).astype(np.uint32) << 16).view(np.float32)


def test_kda_block_commit_is_the_verify_state(torch, ctx, rs):
    """Committing a node twice (from the same trace) is bit-identical, and
    committing on top of a committed state continues the chain."""
    import k3xb
    g = np.random.default_rng(77)
    H, h, d, W, S, N = 256, 2, 64, 4, 3, 4
    P = h * d
    w = make_kda_weights(g, H, h, d, W)
    conv, rec = _states(g, S, h, d, W, P)
    x = bf16_normal(g, (S, N, H))
    desc = k3xb.kda_layer_desc(_kda_dev(torch, w))
    parent = [-1, 0, 1, 2]
    out = torch.empty((S, N, H), dtype=torch.float32, device="cuda")
    trace = torch.empty(ctx.kda_trace_bytes(desc, N, S), dtype=torch.uint8, device="cuda")
    conv_d, rec_d = to_dev(torch, conv), to_dev(torch, rec)
    ctx.kda_block(desc, to_dev(torch, x), parent, conv_d, rec_d, out, trace)
    outs = []
    for _ in range(2):
        co, ro = torch.empty_like(conv_d), torch.empty_like(rec_d)
        ctx.kda_block_commit(desc, trace, parent, S, [1, 3, 0], conv_d, rec_d, co, ro)
        outs.append((co.cpu().numpy(), ro.cpu().numpy()))
    np.testing.assert_array_equal(outs[0][0], outs[1][0])
    np.testing.assert_array_equal(outs[0][1], outs[1][1])
    # in-place conv commit equals the out-of-place one
    ro = torch.empty_like(rec_d)
    ctx.kda_block_commit(desc, trace, parent, S, [1, 3, 0], conv_d, rec_d, conv_d, ro)
    ctx.sync()
    np.testing.assert_array_equal(conv_d.cpu().numpy(), outs[0][0])


def test_layer_forward_c1_vs_oracle(torch, ctx, rs):
    """BASELINE configs[0] layer dims (H 256, 4 heads x 64, 16 experts Top-4,
    I 128, shared 128, SwiGLU): two sequences of anchor + 4 drafts."""
    import k3xb
    c = C1
    layer = make_layer(rs, 0, c["hidden"], c["heads"], c["head_dim"], c["experts"], c["top_k"], c["inter"],
                       c["shared_inter"])
    g = np.random.default_rng(1)
    S, N, H = 2, 5, c["hidden"]
    P = c["heads"] * c["head_dim"]
    conv, rec = _states(g, S, c["heads"], c["head_dim"], 4, P)
    hidden = bf16_normal(g, (S, N, H))
    block = bf16_normal(g, (S, N, H))
    parent = [-1, 0, 1, 2, 3]
    dl = dict(layer)
    dl["kda"] = _kda_dev(torch, layer["kda"])
    dl["moe"] = layer_to_dev(torch, layer["moe"])
    for k in ("self_residual_norm", "self_residual_proj", "input_norm", "moe_residual_norm", "moe_residual_proj",
              "post_norm"):
        dl[k] = to_dev(torch, layer[k])
    desc = k3xb.layer_desc(dl)
    out = torch.empty((S, N, H), dtype=torch.float32, device="cuda")
    ids = torch.empty((S * N, c["top_k"]), dtype=torch.int32, device="cuda")
    ctx.layer_forward(desc, to_dev(torch, hidden), to_dev(torch, block), parent, to_dev(torch, conv),
                      to_dev(torch, rec), out, ids)
    ctx.sync()
    got, gids = out.cpu().numpy(), ids.cpu().numpy().view(np.uint32).reshape(S, N, -1)
    agree = 0
    for s in range(S):
        want, wids, _ = rs.layer_forward(layer, hidden[s], block[s], np.array(parent),
                                         tuple(conv[s, i] for i in range(3)), rec[s].ravel())
        same = np.all(gids[s] == wids, axis=1)
        agree += same.sum()
        assert_mostly_close(got[s][same], want[same], what=f"layer output, sequence {s}")
    assert agree >= 0.9 * S * N, f"expert ids agree on {agree}/{S * N} tokens"


def _layer_dev(torch, layer):
    dl = dict(layer)
    dl["kda"] = _kda_dev(torch, layer["kda"])
    dl["moe"] = layer_to_dev(torch, layer["moe"])
    for k in ("self_residual_norm", "self_residual_proj", "input_norm", "moe_residual_norm", "moe_residual_proj",
              "post_norm"):
        dl[k] = to_dev(torch, layer[k])
    return dl


def test_verify_step_c1_vs_oracle(torch, ctx, rs):
    """BASELINE configs[0] shapes end to end: embedding, 2 KDA+MoE layers,
    final norm, V 1024 LM head, greedy acceptance, device-side commit.
    Sequence 0's first two drafts are the oracle's own greedy continuation,
    so acceptance is exercised past the first draft."""
    import k3xb
    c = C1
    L, S, p, V, H = 2, 2, 4, 1024, c["hidden"]
    N, P = p + 1, c["heads"] * c["head_dim"]
    layers = [make_layer(rs, 10 + l, H, c["heads"], c["head_dim"], c["experts"], c["top_k"], c["inter"],
                         c["shared_inter"]) for l in range(L)]
    g = np.random.default_rng(3)
    emb = bf16_words(g.normal(0, 1.0, size=(V, H)))
    lm = bf16_words(g.normal(0, 0.02, size=(V, H)))
    fnorm = bf16_words(np.ones(H, np.float32))
    states = [_states(g, S, c["heads"], c["head_dim"], 4, P) for _ in range(L)]
    conv = np.stack([st[0] for st in states])     # [L][S][3][(w-1)P]
    rec = np.stack([st[1] for st in states])      # [L][S][h][d][d]
    embf = (emb.astype(np.uint32) << 16).view(np.float32)
    tokens = g.integers(0, V, size=(S, N)).astype(np.uint32)

    def oracle(s, toks):
        x = embf[toks]
        return rs.verify_greedy_stack(layers, lm, fnorm, 1e-6, x, x, toks[1:],
                                      [tuple(conv[l, s, i] for i in range(3)) for l in range(L)],
                                      [rec[l, s].ravel() for l in range(L)])

    for i in range(1, 3):   # sequence 0: drafts 1, 2 follow the oracle's targets
        tokens[0, i] = oracle(0, tokens[0, :i + 1])[1][i - 1]
    want = [oracle(s, tokens[s]) for s in range(S)]

    dls = [_layer_dev(torch, layer) for layer in layers]
    emb_d, lm_d, fnorm_d = to_dev(torch, emb), to_dev(torch, lm), to_dev(torch, fnorm)   # kept alive
    model = k3xb.verify_model_desc([k3xb.layer_desc(d) for d in dls], V, lm_d, embedding=emb_d,
                                   final_norm=fnorm_d)
    u32 = lambda *shape: torch.zeros(shape, dtype=torch.int32, device="cuda")
    conv_d, rec_d = to_dev(torch, conv), to_dev(torch, rec)
    tok_d = to_dev(torch, tokens.view(np.int32))
    drafts_d = to_dev(torch, np.ascontiguousarray(tokens[:, 1:]).view(np.int32))
    logits = torch.empty((S, N, V), dtype=torch.float32, device="cuda")
    acc, com, cnt = u32(S), u32(S, N), u32(S)
    io = k3xb.verify_io_desc(S, p, conv_d, rec_d, acc, com, cnt, drafts_d, tokens=tok_d, logits=logits)
    ctx.verify_step(model, io)
    ctx.sync()
    gl = logits.cpu().numpy()
    ga, gc, gn = acc.cpu().numpy(), com.cpu().numpy().view(np.uint32), cnt.cpu().numpy()
    gconv, grec = conv_d.cpu().numpy().view(np.uint16), rec_d.cpu().numpy()
    for s in range(S):
        wl, wt, wa, wc, wst = want[s]
        assert_mostly_close(gl[s], wl, what=f"logits, sequence {s}")
        # acceptance on the GPU's own logits is bit-exact (speculative.cpp:74-112)
        targets = np.array([rs.argmax(gl[s, i]) for i in range(N)], np.uint32)
        a, cm, _ = rs.verify_greedy_block(0, tokens[s, 1:], p, V, targets)
        assert ga[s] == a and gn[s] == len(cm) and gc[s, :len(cm)].tolist() == cm
        if s == 0:
            assert ga[s] >= 2 or not np.array_equal(targets[:2], wt[:2])
        # committed state at the GPU's accepted node vs the oracle's commit there
        x = embf[tokens[s]]
        xl, parent = x, np.arange(-1, N - 1)
        for l in range(L):
            out, _, _, xin = rs.layer_forward(layers[l], xl, x, parent,
                                              tuple(conv[l, s, i] for i in range(3)), rec[l, s].ravel(),
                                              want_xin=True)
            cq, ck, cv, r = rs.kda_block_commit(layers[l]["kda"], xin, parent, int(ga[s]),
                                                tuple(conv[l, s, i] for i in range(3)), rec[l, s].ravel())
            for i, rows in enumerate((cq, ck, cv)):
                assert_mostly_close(bf16_to_f32(gconv[l, s, i]), bf16_to_f32(rows), what=f"layer {l} conv {i}")
            assert_mostly_close(grec[l, s].ravel(), r, what=f"layer {l} recurrent state")
            xl = out
