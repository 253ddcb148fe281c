"""The device AURORA drafter (k3xb_draft_greedy): reduced-Top-K greedy
self-drafting from the committed KDA state.

- With draft_top_k equal to the target's top_k the drafter is the target
  model decoding one position at a time, so the verify step must accept
  every draft (its batched pass computes each position exactly as the
  single-position steps did) and commit the drafts plus its bonus token.
- With a reduced K, draft 0 is the argmax of the reduced model's logits at
  the anchor, and those logits match the oracle's reduced stack within the
  north-star tolerance.
- The target's state arrays are left as they were."""
import numpy as np
import pytest

from gpu_util import to_dev, torch_cuda
from oracle import bf16_words, make_layer

pytestmark = pytest.mark.gpu

C1 = dict(hidden=256, heads=4, head_dim=64, experts=16, top_k=4, inter=128, shared_inter=128)


def _states(g, S, h, d, W, P):
    conv = np.stack([np.stack([bf16_words(g.normal(0, 0.5, size=(W - 1) * P)) for _ in range(3)])
                     for _ in range(S)])
    rec = g.normal(0, 0.05, size=(S, h, d, d)).astype(np.float32)
    return conv, rec


def _layer_dev(torch, layer):
    from gpu_util import layer_to_dev
    dl = dict(layer)
    dl["kda"] = {k: (to_dev(torch, v) if isinstance(v, np.ndarray) else v) for k, v in layer["kda"].items()}
    dl["moe"] = layer_to_dev(torch, layer["moe"])
    for k in ("self_residual_norm", "self_residual_proj", "input_norm", "moe_residual_norm", "moe_residual_proj",
              "post_norm"):
        dl[k] = to_dev(torch, layer[k])
    return dl


def _setup(rs, torch, S):
    c = C1
    L, V, H = 2, 1024, c["hidden"]
    P = c["heads"] * c["head_dim"]
    layers = [make_layer(rs, 40 + l, H, c["heads"], c["head_dim"], c["experts"], c["top_k"], c["inter"],
                         c["shared_inter"]) for l in range(L)]
    g = np.random.default_rng(41)
    emb = bf16_words(g.normal(0, 1.0, size=(V, H)))
    lm = bf16_words(g.normal(0, 0.02, size=(V, H)))
    fnorm = bf16_words(np.ones(H, np.float32))
    states = [_states(g, S, c["heads"], c["head_dim"], 4, P) for _ in range(L)]
    conv = np.stack([st[0] for st in states])
    rec = np.stack([st[1] for st in states])
    anchors = g.integers(0, V, size=S).astype(np.uint32)
    return layers, emb, lm, fnorm, conv, rec, anchors, V


def _model(torch, layers, emb, lm, fnorm, V, top_k=None):
    import k3xb
    dls = [_layer_dev(torch, layer) for layer in layers]
    descs = [k3xb.layer_desc(d) for d in dls]
    if top_k:
        for d in descs:
            d.moe.top_k = top_k
    keep = (dls, to_dev(torch, emb), to_dev(torch, lm), to_dev(torch, fnorm))
    return k3xb.verify_model_desc(descs, V, keep[2], embedding=keep[1], final_norm=keep[3]), keep


def test_full_k_drafts_are_all_accepted(rs):
    import k3xb
    torch = torch_cuda()
    S, p = 3, 4
    layers, emb, lm, fnorm, conv, rec, anchors, V = _setup(rs, torch, S)
    ctx = k3xb.Context(0)
    ctx.use_stream()
    try:
        model, keep = _model(torch, layers, emb, lm, fnorm, V)
        conv_d, rec_d = to_dev(torch, conv), to_dev(torch, rec)
        drafts = torch.zeros((S, p), dtype=torch.int32, device="cuda")
        ctx.draft_greedy(model, to_dev(torch, anchors.view(np.int32)), conv_d, rec_d, drafts, C1["top_k"])
        ctx.sync()
        np.testing.assert_array_equal(conv_d.cpu().numpy().view(np.uint16), conv)   # target state untouched
        np.testing.assert_array_equal(rec_d.cpu().numpy(), rec)
        d = drafts.cpu().numpy().view(np.uint32)
        assert d.max() < V
        tokens = np.concatenate([anchors[:, None], d], axis=1)
        u32 = lambda *shape: torch.zeros(shape, dtype=torch.int32, device="cuda")
        acc, com, cnt = u32(S), u32(S, p + 1), u32(S)
        io = k3xb.verify_io_desc(S, p, conv_d, rec_d, acc, com, cnt, drafts,
                                 tokens=to_dev(torch, np.ascontiguousarray(tokens).view(np.int32)))
        ctx.verify_step(model, io)
        ctx.sync()
        assert acc.cpu().numpy().tolist() == [p] * S
        assert cnt.cpu().numpy().tolist() == [p + 1] * S
        np.testing.assert_array_equal(com.cpu().numpy().view(np.uint32)[:, :p], d)
    finally:
        ctx.close()


def test_reduced_k_first_draft_is_the_reduced_argmax(rs):
    import k3xb
    torch = torch_cuda()
    S, p, k = 2, 3, 2
    layers, emb, lm, fnorm, conv, rec, anchors, V = _setup(rs, torch, S)
    ctx = k3xb.Context(0)
    ctx.use_stream()
    try:
        model, keep = _model(torch, layers, emb, lm, fnorm, V)
        drafts = torch.zeros((S, p), dtype=torch.int32, device="cuda")
        ctx.draft_greedy(model, to_dev(torch, anchors.view(np.int32)), to_dev(torch, conv), to_dev(torch, rec),
                         drafts, k)
        # the reduced model's own single-position step at the anchor
        reduced, keep2 = _model(torch, layers, emb, lm, fnorm, V, top_k=k)
        u32 = lambda *shape: torch.zeros(shape, dtype=torch.int32, device="cuda")
        acc, com, cnt = u32(S), u32(S, 1), u32(S)
        logits = torch.empty((S, 1, V), dtype=torch.float32, device="cuda")
        io = k3xb.verify_io_desc(S, 0, to_dev(torch, conv), to_dev(torch, rec), acc, com, cnt, None,
                                 tokens=to_dev(torch, anchors.view(np.int32)), logits=logits)
        ctx.verify_step(reduced, io)
        ctx.sync()
        gl = logits.cpu().numpy()
        d = drafts.cpu().numpy().view(np.uint32)
        for s in range(S):
            assert d[s, 0] == rs.argmax(gl[s, 0])
        # and those logits are the oracle's reduced stack at the anchor
        embf = (emb.astype(np.uint32) << 16).view(np.float32)
        small = [dict(layer, moe=dict(layer["moe"], top_k=k)) for layer in layers]
        for s in range(S):
            x = embf[anchors[s:s + 1]]
            want = rs.verify_greedy_stack(small, lm, fnorm, 1e-6, x, x, anchors[s:s + 1][1:],
                                          [tuple(conv[l, s, i] for i in range(3)) for l in range(len(layers))],
                                          [rec[l, s].ravel() for l in range(len(layers))])[0]
            err = np.abs(gl[s] - want)
            tol = 1e-3 + 2e-2 * np.abs(want)
            assert (err > tol).mean() <= 0.01 and (err / tol).max() <= 8.0
    finally:
        ctx.close()


def test_on_device_steps_follow_the_greedy_decode(rs):
    """Two on-device speculative steps (draft with the full K, verify,
    advance, next anchor) commit exactly the target's greedy decode: every
    draft is accepted, and the committed tokens of the first step then the
    second are the 2(p+1) tokens a plain greedy decode from the same state
    produces."""
    import k3xb
    torch = torch_cuda()
    S, p = 2, 3
    layers, emb, lm, fnorm, conv, rec, anchors, V = _setup(rs, torch, S)
    ctx = k3xb.Context(0)
    ctx.use_stream()
    try:
        model, keep = _model(torch, layers, emb, lm, fnorm, V)
        ref = torch.zeros((S, 2 * (p + 1)), dtype=torch.int32, device="cuda")
        ctx.draft_greedy(model, to_dev(torch, anchors.view(np.int32)), to_dev(torch, conv), to_dev(torch, rec),
                         ref, C1["top_k"])
        a_d, conv_d, rec_d = to_dev(torch, anchors.view(np.int32)), to_dev(torch, conv), to_dev(torch, rec)
        i32 = lambda *shape: torch.zeros(shape, dtype=torch.int32, device="cuda")
        drafts, acc, com, cnt = i32(S, p), i32(S), i32(S, p + 1), i32(S)
        committed = []
        for _ in range(2):
            ctx.speculative_step(model, a_d, conv_d, rec_d, drafts, acc, com, cnt, C1["top_k"])
            ctx.sync()
            assert acc.cpu().numpy().tolist() == [p] * S and cnt.cpu().numpy().tolist() == [p + 1] * S
            committed.append(com.cpu().numpy().view(np.uint32).copy())
        want = ref.cpu().numpy().view(np.uint32)
        np.testing.assert_array_equal(np.concatenate(committed, axis=1), want)
        np.testing.assert_array_equal(a_d.cpu().numpy().view(np.uint32), want[:, -1])
    finally:
        ctx.close()
