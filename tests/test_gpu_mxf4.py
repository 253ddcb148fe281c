"""Parity of the tcgen05 expert engines (through the C ABI).

Routed experts run on kind::mxf4, the shared expert on kind::f16. Checked
against the CPU oracle at small shapes and at the released c2 shape (for a
few tokens, with the selected experts fetched per token). Routes bit-exact;
hidden states within the north-star tolerance, with the bf16 rounding-point
allowance of gpu_util.assert_hidden_close.
"""
import numpy as np
import pytest

from gpu_util import assert_hidden_close, layer_to_dev, to_dev, torch_cuda
from oracle import ACT_SITU, ACT_SWIGLU, bf16_normal, make_moe_layer

pytestmark = pytest.mark.gpu


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


def _run(torch, ctx, d, hidden_dev, T, engine, terms=6):
    import k3xb
    desc = k3xb.moe_layer_desc(d, engine=engine, act_terms=terms)
    out = torch.empty((T, d["hidden"]), dtype=torch.float32, device="cuda")
    ids = torch.empty((T, d["top_k"]), dtype=torch.int32, device="cuda")
    ctx.moe_layer_forward(desc, hidden_dev, out, ids)
    ctx.sync()
    return out.cpu().numpy(), ids.cpu().numpy().view(np.uint32)


def _report(got, want):
    err = np.abs(got - want)
    tol = 1e-3 + 2e-2 * np.abs(want)
    return f"max|err| {err.max():.3e}, violations {(err > tol).sum()}/{err.size}"


@pytest.mark.parametrize("act", [ACT_SWIGLU, ACT_SITU])
@pytest.mark.parametrize("dims", [(256, 128, 16, 4, 5), (512, 256, 32, 8, 40), (384, 640, 12, 3, 9),
                                  # ~25 rows per expert x 6 terms: 128-row activation tiles
                                  (256, 384, 8, 2, 100)])
def test_mxf4_matches_oracle(torch, ctx, rs, act, dims):
    import k3xb
    H, I, E, K, T = dims
    layer = make_moe_layer(rs, H + I + act, hidden=H, inter=I, experts=E, top_k=K, shared_inter=128,
                           activation=act)
    hidden = bf16_normal(np.random.default_rng(H), (T, H))
    d = layer_to_dev(torch, layer)
    got, ids = _run(torch, ctx, d, to_dev(torch, hidden), T, k3xb.ENGINE_MXF4)
    want, want_ids, _ = rs.moe_layer(layer, hidden)
    np.testing.assert_array_equal(ids, want_ids)
    np.testing.assert_allclose(got, want, rtol=2e-2, atol=1e-3, err_msg=_report(got, want))


def test_mxf4_prepared_scales_identical(torch, ctx, rs):
    """Scales re-laid once (k3xb_prepare_mxfp4_scales) give bit-identical
    results to the per-call re-layout."""
    import k3xb
    layer = make_moe_layer(rs, 17, hidden=256, inter=256, experts=8, top_k=2, shared_inter=0)
    hidden = bf16_normal(np.random.default_rng(18), (6, 256))
    d = layer_to_dev(torch, layer)
    a, _ = _run(torch, ctx, d, to_dev(torch, hidden), 6, k3xb.ENGINE_MXF4)
    ctx.prepare_layer_scales(d)
    b, _ = _run(torch, ctx, d, to_dev(torch, hidden), 6, k3xb.ENGINE_MXF4)
    np.testing.assert_array_equal(a, b)


def test_mxf4_term_count_converges(torch, ctx, rs):
    """More E2M1 terms -> closer to the FP64 oracle (the split is exact in
    the limit)."""
    import k3xb
    layer = make_moe_layer(rs, 5, hidden=512, inter=256, experts=16, top_k=4, shared_inter=0)
    hidden = bf16_normal(np.random.default_rng(6), (8, 512))
    d = layer_to_dev(torch, layer)
    want, _, _ = rs.moe_layer(layer, hidden)
    errs = []
    for terms in (2, 4, 8):
        got, _ = _run(torch, ctx, d, to_dev(torch, hidden), 8, k3xb.ENGINE_MXF4, terms)
        errs.append(np.abs(got - want).max())
    assert errs[2] <= errs[0], errs


def _c2_layer(torch, ctx):
    import k3xb
    H, I, E, K, T, Is = 7168, 2048, 384, 16, 64, 2048
    u8 = lambda *s: torch.empty(s, dtype=torch.uint8, device="cuda")
    d = dict(hidden=H, inter=I, experts=E, top_k=K, shared_inter=Is, activation=k3xb.ACT_SWIGLU)
    for i, (name, shape) in enumerate((("shared_gate", (Is, H)), ("shared_up", (Is, H)),
                                        ("shared_down", (H, Is)))):
        d[name] = torch.empty(shape, dtype=torch.int16, device="cuda")
        ctx.fill_normal_bf16(d[name], 1, 22 + i, 0.02)
    d["gate_packed"], d["gate_scales"] = u8(E, I, H // 2), u8(E, I, H // 32)
    d["up_packed"], d["up_scales"] = u8(E, I, H // 2), u8(E, I, H // 32)
    d["down_packed"], d["down_scales"] = u8(E, H, I // 2), u8(E, H, I // 32)
    ctx.fill_normal_mxfp4(d["gate_packed"], d["gate_scales"], E * I, H, 1, 10, 0.02)
    ctx.fill_normal_mxfp4(d["up_packed"], d["up_scales"], E * I, H, 1, 11, 0.02)
    ctx.fill_normal_mxfp4(d["down_packed"], d["down_scales"], E * H, I, 1, 12, 0.02)
    d["router"] = torch.empty((E, H), dtype=torch.int16, device="cuda")
    ctx.fill_normal_bf16(d["router"], 1, 20, 0.02)
    d["correction"] = torch.empty(E, dtype=torch.float32, device="cuda")
    ctx.fill_normal_f32(d["correction"], 1, 21, 0.0, 0.02)
    words = torch.empty((T, H), dtype=torch.int16, device="cuda")
    ctx.fill_normal_bf16(words, 1, 30, 1.0)
    hidden = (words.to(torch.int32) << 16).view(torch.float32).contiguous()
    return d, hidden


def _oracle_token(rs, d, x):
    """Plain-MoE oracle for one token (official_moe.cpp:271-344 minus the
    latent steps), fetching only the selected experts from the device."""
    H, I, K = d["hidden"], d["inter"], d["top_k"]
    router = d["router"].cpu().numpy().view(np.uint16)
    ids, con = rs.route(x, router, d["correction"].cpu().numpy(), K)
    ys = []
    for e in ids:
        e = int(e)
        g = rs.mxfp4_matmul(x, d["gate_packed"][e].cpu().numpy(), d["gate_scales"][e].cpu().numpy(), I, H)
        u = rs.mxfp4_matmul(x, d["up_packed"][e].cpu().numpy(), d["up_scales"][e].cpu().numpy(), I, H)
        a = rs.swiglu(g, u)
        ys.append(rs.round_bf16(rs.mxfp4_matmul(a, d["down_packed"][e].cpu().numpy(),
                                                d["down_scales"][e].cpu().numpy(), H, I)))
    mixed = rs.routed_combine(np.stack(ys), con)
    gs = rs.bf16_matvec(x, d["shared_gate"].cpu().numpy().view(np.uint16))
    us = rs.bf16_matvec(x, d["shared_up"].cpu().numpy().view(np.uint16))
    shared = rs.bf16_matvec(rs.swiglu(gs, us), d["shared_down"].cpu().numpy().view(np.uint16))
    return rs.round_bf16(mixed + shared), ids, mixed, shared


def test_mxf4_c2_shape_vs_oracle(torch, ctx, rs):
    """Released c2 shape (H 7168, 384 experts, I 2048, Top-16, shared 2048,
    64 tokens) on device-generated weights: the tensor-core layer against
    the oracle on three tokens, and against the SIMT engine on all 64."""
    import k3xb
    d, hidden = _c2_layer(torch, ctx)
    T = hidden.shape[0]
    a, ia = _run(torch, ctx, d, hidden, T, k3xb.ENGINE_MXF4)
    b, ib = _run(torch, ctx, d, hidden, T, k3xb.ENGINE_SIMT)
    np.testing.assert_array_equal(ia, ib)
    x_all = hidden.cpu().numpy()
    for t in (0, 13, 63):
        want, ids, mixed, shared = _oracle_token(rs, d, x_all[t])
        assert ia[t].tolist() == ids.tolist()
        scale = np.maximum(np.abs(mixed), np.abs(shared))
        assert_hidden_close(a[t], want, scale)
        assert_hidden_close(b[t], want, scale)
    del d
    torch.cuda.empty_cache()


@pytest.mark.parametrize("terms", [4, 5])
@pytest.mark.parametrize("dims", [(256, 384, 8, 2, 100), (512, 256, 16, 8, 96)])
def test_mxf4_fewer_terms_within_tolerance(torch, ctx, rs, terms, dims):
    """Fewer E2M1 terms per activation row (cheaper large-M tiles) against
    the FP64 oracle at ~25-48 rows per expert: within the north-star
    tolerance (rel 2e-2 / abs 1e-3), with the bf16 rounding-point allowance
    of assert_hidden_close."""
    import k3xb
    H, I, E, K, T = dims
    layer = make_moe_layer(rs, H + I + terms, hidden=H, inter=I, experts=E, top_k=K, shared_inter=128)
    hidden = bf16_normal(np.random.default_rng(H + T), (T, H))
    d = layer_to_dev(torch, layer)
    got, ids = _run(torch, ctx, d, to_dev(torch, hidden), T, k3xb.ENGINE_MXF4, terms)
    want, want_ids, _ = rs.moe_layer(layer, hidden)
    np.testing.assert_array_equal(ids, want_ids)
    assert_hidden_close(got, want, np.abs(want))


def test_mxf4_library_default_terms_at_large_m(torch, ctx, rs):
    """act_terms 0 (the library default) at ~25 rows per expert resolves to
    4 terms and stays within the north-star tolerance of the FP64 oracle."""
    import k3xb
    H, I, E, K, T = 256, 384, 8, 2, 100
    assert k3xb.default_act_terms(T * K, E) == 4
    layer = make_moe_layer(rs, 77, hidden=H, inter=I, experts=E, top_k=K, shared_inter=128)
    hidden = bf16_normal(np.random.default_rng(78), (T, H))
    got, ids = _run(torch, ctx, layer_to_dev(torch, layer), to_dev(torch, hidden), T, k3xb.ENGINE_MXF4, 0)
    want, want_ids, _ = rs.moe_layer(layer, hidden)
    np.testing.assert_array_equal(ids, want_ids)
    assert_hidden_close(got, want, np.abs(want))
