"""The block attention residual with many sources on the GPU (through the C
ABI, k3xb_block_attention_residual) against the pinned restatement of
model.cpp:645-666 and the reference's own cases.

The kernel takes each score as an FP64 sum rounded once to float, where
the reference rounds every key element and product to float and chains
float adds; the softmax and the output sum follow the reference's order.
Outputs are held to 3e-5 of the largest |value|: emulating the kernel's
arithmetic on the CPU against the restatement gives at most 5e-6 of it at
H 7168 (the reference's own float-chain error).
"""
import os

import numpy as np
import pytest

from gpu_util import to_dev, torch_cuda

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "block_attn_res.npz")
RTOL_SCALE = 3e-5


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


def _run(torch, ctx, prefix, sources, norm, proj, eps):
    T, H = prefix.shape
    out = torch.empty((T, H), dtype=torch.float32, device="cuda")
    ctx.block_attention_residual(to_dev(torch, prefix), None if sources.shape[0] == 0 else to_dev(torch, sources),
                                 to_dev(torch, norm), to_dev(torch, proj), eps, out)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _case(g, S, T, H):
    scale = g.choice(np.array([0.25, 1.0, 4.0], np.float32), size=(S + 1, 1, 1))
    values = (g.normal(size=(S + 1, T, H)) * scale).astype(np.float32)
    norm = (1.0 + 0.1 * g.normal(size=H)).astype(np.float32)
    proj = (g.normal(size=H) * 3.0 / np.sqrt(H)).astype(np.float32)
    return values[S], values[:S], norm, proj


def _assert_close(got, want, values, what):
    err = np.abs(got - want).max()
    bound = RTOL_SCALE * max(float(np.abs(values).max()), 1e-30)
    assert err <= bound, f"{what}: max|err| {err:.3e} > {bound:.3e}"


def test_known_answer(torch, ctx):
    # tests/python/test_attn_res.py of the reference (H 2: the scalar path)
    out = _run(torch, ctx, np.array([[1.0, 1.0]], np.float32), np.array([[[3.0, 0.0]], [[0.0, 4.0]]], np.float32),
               np.ones(2, np.float32), np.array([1.0, 0.0], np.float32), 0.0)
    np.testing.assert_allclose(out, [[1.9227442, 0.85785025]], atol=1e-6)


def test_torch_reference_fixture(torch, ctx, rs):
    z = np.load(GOLDEN)
    eps = float(z["eps"])
    out = _run(torch, ctx, z["prefix"], z["sources"], z["norm"], z["proj"], eps)
    values = np.concatenate([z["sources"], z["prefix"][None]])
    _assert_close(out, z["torch_out"], values, "vs torch reference")
    _assert_close(out, rs.block_attention_residual(z["prefix"], z["sources"], z["norm"], z["proj"], eps), values,
                  "vs restatement")


# the float4 form (H % 4 == 0): up to the 63-source maximum, H from 4 to
# 7168 and 64 rows; the scalar form: (5, 3, 257)
@pytest.mark.parametrize("S,T,H", [(1, 1, 7168), (12, 6, 7168), (4, 64, 7168), (63, 2, 128), (40, 3, 7168),
                                   (3, 4, 1028), (2, 9, 4), (5, 3, 257)])
def test_matches_restatement(torch, ctx, rs, S, T, H):
    g = np.random.default_rng(7000 + 131 * S + T + H)
    prefix, sources, norm, proj = _case(g, S, T, H)
    out = _run(torch, ctx, prefix, sources, norm, proj, 1e-6)
    want = rs.block_attention_residual(prefix, sources, norm, proj, 1e-6)
    _assert_close(out, want, np.concatenate([sources, prefix[None]]), f"S={S} T={T} H={H}")


def test_no_sources_is_the_prefix(torch, ctx):
    g = np.random.default_rng(7101)
    prefix, _, norm, proj = _case(g, 0, 3, 7168)
    out = _run(torch, ctx, prefix, np.zeros((0, 3, 7168), np.float32), norm, proj, 1e-6)
    assert np.array_equal(out, prefix)


def test_unaligned_rows_take_the_scalar_path(torch, ctx, rs):
    # rows one float past a 16-byte boundary: the kernel must not use float4s
    g = np.random.default_rng(7103)
    S, T, H = 3, 4, 512
    prefix, sources, norm, proj = _case(g, S, T, H)
    buf = torch.zeros(1 + (S + 1) * T * H, dtype=torch.float32, device="cuda")
    src = buf[1:1 + S * T * H].view(S, T, H)
    pre = buf[1 + S * T * H:].view(T, H)
    src.copy_(torch.from_numpy(sources))
    pre.copy_(torch.from_numpy(prefix))
    out_buf = torch.empty(1 + T * H, dtype=torch.float32, device="cuda")
    out = out_buf[1:].view(T, H)
    ctx.block_attention_residual(pre, src, to_dev(torch, norm), to_dev(torch, proj), 1e-6, out)
    torch.cuda.synchronize()
    want = rs.block_attention_residual(prefix, sources, norm, proj, 1e-6)
    _assert_close(out.cpu().numpy(), want, np.concatenate([sources, prefix[None]]), "unaligned")


def test_full_size_properties(torch, ctx, rs):
    # c5's 576 verify positions at H 7168 with 8 sources: against the
    # restatement, a convex combination of the values, and equal values
    # averaging to themselves
    g = np.random.default_rng(7107)
    S, T, H = 8, 576, 7168
    prefix, sources, norm, proj = _case(g, S, T, H)
    values = np.concatenate([sources, prefix[None]])
    out = _run(torch, ctx, prefix, sources, norm, proj, 1e-6)
    _assert_close(out, rs.block_attention_residual(prefix, sources, norm, proj, 1e-6), values, "full size")
    slack = 1e-6 * np.abs(values).max()
    assert np.all(out >= values.min(axis=0) - slack) and np.all(out <= values.max(axis=0) + slack)
    same = np.broadcast_to(prefix, (S, T, H)).copy()
    out = _run(torch, ctx, prefix, same, norm, proj, 1e-6)
    np.testing.assert_allclose(out, prefix, rtol=1e-5, atol=1e-6)


def test_arguments_rejected(torch, ctx):
    import k3xb
    T, H = 2, 64
    prefix = torch.zeros((T, H), dtype=torch.float32, device="cuda")
    w = torch.ones(H, dtype=torch.float32, device="cuda")
    out = torch.empty_like(prefix)
    too_many = torch.zeros((64, T, H), dtype=torch.float32, device="cuda")
    for args in ((prefix, too_many, w, w, 1e-6, out), (prefix, None, w, w, -1.0, out),
                 (prefix, None, w, w, float("nan"), out)):
        with pytest.raises(k3xb.K3xbError) as e:
            ctx.block_attention_residual(*args)
        assert e.value.status == k3xb.INVALID_EXTENT
    ctx.sync()
