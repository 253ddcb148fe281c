"""Host-I/O entry points a ComputeBackend adapter calls with the reference's
host views (backend.hpp:326-462): k3xb_expert_grid_host
(mxfp4_situ_mlp_grid / _group / _batch / mxfp4_situ_moe) and
k3xb_kda_block_host (official_kda, host-roundtrip state). Each must equal
the device entry points it is made of, bit for bit, also when its weights
come from the resident table (k3xb_acquire_*), and the grid must equal the
oracle's expert FFN within the north-star tolerance."""
import numpy as np
import pytest

from gpu_util import assert_close_bf16, layer_to_dev, to_dev, torch_cuda
from oracle import bf16_normal, bf16_words, make_kda_weights, make_moe_layer

pytestmark = pytest.mark.gpu

DIMS = dict(hidden=256, inter=128, experts=8, top_k=2, shared_inter=0)


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


def _expert(rs, L, e, x):
    H, I = L["hidden"], L["inter"]
    g = rs.mxfp4_matmul(x, L["gate_packed"][e], L["gate_scales"][e], I, H)
    u = rs.mxfp4_matmul(x, L["up_packed"][e], L["up_scales"][e], I, H)
    return rs.round_bf16(rs.mxfp4_matmul(rs.swiglu(g, u), L["down_packed"][e], L["down_scales"][e], H, I))


def test_expert_grid_host_vs_oracle_and_single_expert_stacks(torch, ctx, rs):
    import k3xb
    d = DIMS
    L = make_moe_layer(rs, 81, d["hidden"], d["inter"], d["experts"], d["top_k"])
    x = bf16_normal(np.random.default_rng(82), (5, d["hidden"]))
    d_dev = layer_to_dev(torch, L)
    desc = k3xb.moe_layer_desc(d_dev, engine=k3xb.ENGINE_MXF4)
    ids = [3, 0, 7]
    got = ctx.expert_grid_host(desc, ids, x)
    assert got.shape == (3, 5, d["hidden"])
    for j, e in enumerate(ids):
        want = np.stack([_expert(rs, L, e, x[t]) for t in range(x.shape[0])])
        assert_close_bf16(got[j], want)
    # the adapter's layout: every expert its own resident stack of one
    names = ("gate_packed", "gate_scales", "up_packed", "up_scales", "down_packed", "down_scales")
    for j, e in enumerate(ids):
        stack = ctx.acquire_expert_stack(1000 + e, d["hidden"], d["inter"], [{n: L[n][e] for n in names}])
        one = dict(hidden=d["hidden"], inter=d["inter"], experts=1, top_k=1)
        single = ctx.expert_grid_host(k3xb.stack_layer_desc(stack, one), [0], x)
        np.testing.assert_array_equal(single[0], got[j])
    with pytest.raises(k3xb.K3xbError, match="INVALID_MXFP4"):
        ctx.expert_grid_host(desc, [1, 1], x)


def test_kda_block_host_equals_device_chain_and_resident_weights(torch, ctx, rs):
    import k3xb
    g = np.random.default_rng(83)
    H, h, dh, W, T = 256, 2, 64, 4, 5
    P = h * dh
    w = make_kda_weights(g, H, h, dh, W)
    conv = np.stack([bf16_words(g.normal(0, 0.5, size=(W - 1) * P)) for _ in range(3)])   # [3][(w-1)*P]
    rec = g.normal(0, 0.05, size=(h, dh, dh)).astype(np.float32)
    x = bf16_normal(g, (T, H))

    wd = {k: (to_dev(torch, v) if isinstance(v, np.ndarray) else v) for k, v in w.items()}
    desc = k3xb.kda_layer_desc(wd)
    parent = list(range(-1, T - 1))
    out_d = torch.empty((1, T, H), dtype=torch.float32, device="cuda")
    trace = torch.empty(ctx.kda_trace_bytes(desc, T, 1), dtype=torch.uint8, device="cuda")
    conv_d, rec_d = to_dev(torch, conv[None]), to_dev(torch, rec[None])
    ctx.kda_block(desc, to_dev(torch, x[None]), parent, conv_d, rec_d, out_d, trace)
    conv_o, rec_o = torch.empty_like(conv_d), torch.empty_like(rec_d)
    ctx.kda_block_commit(desc, trace, parent, 1, [T - 1], conv_d, rec_d, conv_o, rec_o)
    ctx.sync()
    want_out = out_d.cpu().numpy()[0]
    want_conv = conv_o.cpu().numpy().view(np.uint16)[0]
    want_rec = rec_o.cpu().numpy()[0]

    c1, r1 = conv.copy(), rec.copy()
    got = ctx.kda_block_host(desc, H, x, c1, r1)
    np.testing.assert_array_equal(got, want_out)
    np.testing.assert_array_equal(c1, want_conv)
    np.testing.assert_array_equal(r1, want_rec)

    # the same block with every weight uploaded through the resident table
    res = dict(w)
    keep = []
    for tensor_id, (name, v) in enumerate(w.items(), start=5000):
        if not isinstance(v, np.ndarray):
            continue
        rows, cols = (v.shape if v.ndim == 2 else (1, v.shape[0]))
        kind = k3xb.WEIGHT_BF16 if v.dtype == np.uint16 else k3xb.WEIGHT_F32
        r = ctx.acquire_weight(tensor_id, kind, rows, cols, 0, v)
        assert r.disposition == k3xb.RESIDENT_ADMITTED
        keep.append(r)
        res[name] = r.primary
    K = k3xb.KdaLayer()
    K.heads, K.head_dim, K.conv_width, K.eps, K.gate_lower_bound = h, dh, W, w["eps"], w["gate_lower_bound"]
    for name in ("q_proj", "k_proj", "v_proj", "q_conv", "k_conv", "v_conv", "f_a_proj", "f_b_proj", "a_log",
                 "dt_bias", "b_proj", "g_proj", "o_norm", "o_proj"):
        setattr(K, name, res[name])
    c2, r2 = conv.copy(), rec.copy()
    got2 = ctx.kda_block_host(K, H, x, c2, r2)
    np.testing.assert_array_equal(got2, want_out)
    np.testing.assert_array_equal(c2, want_conv)
    np.testing.assert_array_equal(r2, want_rec)
    ctx.release_resident()


def test_kda_block_held_split_equals_one_call(torch, ctx, rs):
    """k3xb_kda_block_held (official_kda's device_seed / device_continue /
    device_publish): the five positions of the test above as seed (2),
    continue (1) and publish (2) from the state the device keeps give the
    one-call outputs and final state (a chain split at any position is the
    same recurrence; the restatement's incremental run equals its full run
    bit for bit, tests/test_golden.py). The bar is 1e-6 relative: the
    kernels run the same operations per row and per state element, so any
    difference would be a last-bit one. A continuation
    on an empty slot, or on a slot holding a state of another shape, is
    INVALID_STATE."""
    import k3xb
    g = np.random.default_rng(84)
    H, h, dh, W, T = 256, 2, 64, 4, 5
    P = h * dh
    w = make_kda_weights(g, H, h, dh, W)
    conv = np.stack([bf16_words(g.normal(0, 0.5, size=(W - 1) * P)) for _ in range(3)])
    rec = g.normal(0, 0.05, size=(h, dh, dh)).astype(np.float32)
    x = bf16_normal(g, (T, H))
    wd = {k: (to_dev(torch, v) if isinstance(v, np.ndarray) else v) for k, v in w.items()}
    desc = k3xb.kda_layer_desc(wd)
    c1, r1 = conv.copy(), rec.copy()
    want = ctx.kda_block_host(desc, H, x, c1, r1)

    with pytest.raises(k3xb.K3xbError) as e:
        ctx.kda_block_held(desc, H, x[:1], 5, k3xb.KDA_CONTINUE)
    assert e.value.status == k3xb.INVALID_STATE
    c2, r2 = conv.copy(), rec.copy()
    parts = [ctx.kda_block_held(desc, H, x[:2], 3, k3xb.KDA_SEED, c2, r2),
             ctx.kda_block_held(desc, H, x[2:3], 3, k3xb.KDA_CONTINUE)]
    c3, r3 = np.zeros_like(conv), np.zeros_like(rec)
    parts.append(ctx.kda_block_held(desc, H, x[3:], 3, k3xb.KDA_PUBLISH, c3, r3))
    np.testing.assert_allclose(np.concatenate(parts), want, rtol=1e-6, atol=1e-7)
    np.testing.assert_array_equal(c3, c1)
    np.testing.assert_allclose(r3, r1, rtol=1e-6, atol=1e-7)
    np.testing.assert_array_equal(c2, conv)   # a seed reads its arrays and leaves them
    # another block shape on the same slot
    w2 = make_kda_weights(g, H, 1, dh, W)
    wd2 = {k: (to_dev(torch, v) if isinstance(v, np.ndarray) else v) for k, v in w2.items()}
    with pytest.raises(k3xb.K3xbError) as e:
        ctx.kda_block_held(k3xb.kda_layer_desc(wd2), H, x[:1], 3, k3xb.KDA_CONTINUE)
    assert e.value.status == k3xb.INVALID_STATE


def test_dense_matvec_bit_identical_to_the_cpu_backend(torch, ctx, rs):
    """k3xb_dense_matvec / _host (dense_matvec, backend_cpu.cpp:23-47): one
    FP64 chain per row in column order, so bit-identical to the reference
    CPU backend's (the restatement is pinned to it in test_oracle_pin.py),
    over odd shapes, unaligned rows, several tokens and a released-size
    matrix; dense_situ_mlp within 1e-5 (the activation's tanhf/expf are the
    device's)."""
    g = np.random.default_rng(172)
    for rows, cols, T in ((1, 1, 1), (7, 33, 2), (130, 257, 3), (7168, 2048, 1)):
        w = (g.normal(0, 1, size=(rows, cols)) * np.exp(g.normal(0, 2, size=(rows, cols)))).astype(np.float32)
        x = g.normal(0, 1, size=(T, cols)).astype(np.float32)
        wd = to_dev(torch, w)
        y = torch.empty((T, rows), dtype=torch.float32, device="cuda")
        ctx.dense_matvec(wd, to_dev(torch, x), y)
        ctx.sync()
        got = y.cpu().numpy()
        for t in range(T):
            want = rs.dense_matvec(x[t], w)
            np.testing.assert_array_equal(got[t], want, err_msg=f"{rows}x{cols} token {t}")
        np.testing.assert_array_equal(ctx.dense_matvec_host(wd, x[0]), rs.dense_matvec(x[0], w))
    inter, cols, out_rows = 256, 512, 384
    gate, up = (g.normal(0, 0.05, size=(inter, cols)).astype(np.float32) for _ in range(2))
    down = g.normal(0, 0.05, size=(out_rows, inter)).astype(np.float32)
    x = g.normal(0, 1, size=cols).astype(np.float32)
    for beta, lin in ((4.0, 0.0), (2.0, 25.0)):
        got = ctx.dense_situ_mlp_host(to_dev(torch, gate), to_dev(torch, up), to_dev(torch, down), x, beta, lin)
        want = rs.dense_situ_mlp(x, gate, up, down, beta, lin)
        # the products are exact; only situ_glu's tanhf/expf (device vs glibc)
        # may differ by an ulp, and the down projection carries that into an
        # output as a few ulps of the output scale (|y| up to ~1)
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=8 * np.finfo(np.float32).eps * np.abs(want).max())


def test_mxfp4_matvec_and_resident_layer_vs_cpu_backend(torch, ctx, rs):
    """k3xb_mxfp4_matvec (mxfp4_matmul, ops.cpp:44-76) bit-identical to the
    restatement (pinned to the reference), including rows and chunks that are
    not multiples of the tile; k3xb_resident_moe_layer_host
    (resident_mxfp4_moe_layer, backend_cpu.cpp:305-339) within 1e-5 of the
    restated composition (pinned in test_oracle_pin.py): its products and
    norm are the reference's bit for bit, its situ_glu uses the device's
    tanhf/expf."""
    from oracle import make_resident_moe_case
    g = np.random.default_rng(191)
    for rows, cols, T in ((1, 32, 1), (130, 96, 2), (257, 1024, 1), (2048, 7168, 1)):
        packed, scales = rs.quantize_mxfp4(g.normal(0, 0.1, size=(rows, cols)).astype(np.float32))
        x = g.normal(0, 1, size=(T, cols)).astype(np.float32)
        y = torch.empty((T, rows), dtype=torch.float32, device="cuda")
        ctx.mxfp4_matvec(to_dev(torch, packed), to_dev(torch, scales), rows, cols, to_dev(torch, x), y)
        ctx.sync()
        got = y.cpu().numpy()
        for t in range(T):
            np.testing.assert_array_equal(got[t], rs.mxfp4_matmul(x[t], packed, scales, rows, cols),
                                          err_msg=f"{rows}x{cols} token {t}")
    for seed, lin in ((181, 0.0), (182, 25.0)):
        w, ex, con, x = make_resident_moe_case(rs, seed)
        wd = {k: to_dev(torch, v) for k, v in w.items()}
        experts = [{k: to_dev(torch, v[e]) for k, v in ex.items()} for e in range(len(con))]
        got = ctx.resident_moe_layer_host(wd, experts, con, x, 1e-6, 4.0, lin)
        np.testing.assert_allclose(got, rs.resident_moe_layer(w, ex, con, x, 1e-6, 4.0, lin), rtol=1e-5, atol=1e-6)


def test_prepare_moe_route_host_vs_restatement(torch, ctx, rs):
    """k3xb_prepare_moe_route_host (prepare_official_moe_route): the prepared
    input within the attention-residual bars of test_gpu_golden.py, its
    router logits bit-identical to the restatement's over that input (the
    router's FP64 chains), and with delta the prefix round_bf16(round_bf16(a)
    + delta) bit for bit; without a router, no logits."""
    import golden_util as gu
    from test_gpu_latent import assert_mostly_close
    f = gu.load("prepare_input.npz")
    g = np.random.default_rng(193)
    H = f["prefix"].shape[1]
    E = 64
    router = bf16_words(g.normal(0, 0.02, size=(E, H)))
    dv = lambda x: to_dev(torch, x)
    norm, proj, post, rd = dv(f["norm"]), dv(f["proj"]), dv(f["post"]), dv(router)
    eps = float(f["eps"])
    for t in range(f["prefix"].shape[0]):
        _, hidden, logits = ctx.prepare_moe_route_host(f["prefix"][t], f["block"][t], norm, proj, post, eps, rd)
        assert_mostly_close(hidden, f["out"][t], what="prepared input")
        np.testing.assert_array_equal(logits, rs.router_logits(hidden, router))
    delta = g.normal(0, 0.5, size=H).astype(np.float32)
    prefix, hidden, logits = ctx.prepare_moe_route_host(f["prefix"][0], f["block"][0], norm, proj, post, eps,
                                                        None, delta)
    np.testing.assert_array_equal(prefix, rs.round_bf16(rs.round_bf16(f["prefix"][0]) + delta))
    assert logits is None and np.isfinite(hidden).all()
