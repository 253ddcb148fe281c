"""k3xb_select_routing (routing_policy.cpp:31-159) against the oracle on
the GPU: expert ids, selected K, floor escalation and weights exactly; the
entropy statistics within 1e-6 (log/exp of the entropy are correctly
rounded on the GPU, glibc's logf/expf on the CPU)."""
import numpy as np
import pytest

from gpu_util import to_dev, torch_cuda

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


def _routing_borderline(d, mode, kw, eps=1e-5, margin=2e-6):
    """True when an adaptive decision sits within `margin` of one of its
    thresholds (the GPU's entropy support may differ from glibc's in the
    last bit there)."""
    if mode != 2:
        return False
    probs = d["_probs"]
    cum = np.cumsum(probs, dtype=np.float32)
    for k in (4, 6, 8, 12, 16):
        if abs(cum[k - 1] + eps - kw.get("mass_target", 0.9)) < margin or abs(k + eps - d["support"]) < margin:
            return True
    return False


@pytest.mark.parametrize("mode,kw", [
    (0, {}), (1, dict(fixed_k=8)), (1, dict(fixed_k=4, quality_floor_k=12)),
    (2, dict(mass_target=0.6, minimum_gap=0.0)), (2, dict(mass_target=0.8, minimum_gap=0.05, quality_floor_k=8)),
])
def test_select_routing_matches_oracle(torch, ctx, rs, mode, kw):
    """k3xb_select_routing == select_routing (routing_policy.cpp:31-159):
    expert ids, selected K, floor escalation and weights exactly; the
    entropy statistics within 1e-6 (log/exp of the entropy are correctly
    rounded on the GPU, glibc's logf/expf on the CPU)."""
    g = np.random.default_rng(7 + mode)
    T, E, K = 48, 384, 16
    scores = (1 / (1 + np.exp(-g.normal(0, 1.5, size=(T, E))))).astype(np.float32)
    scores[::5, :40] = scores[::5, :1]          # ties, broken by index
    bias = g.normal(0, 0.02, size=E).astype(np.float32)
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    w = torch.empty((T, K), dtype=torch.float32, device="cuda")
    sel = torch.empty(T, dtype=torch.int32, device="cuda")
    esc = torch.empty(T, dtype=torch.int32, device="cuda")
    stats = torch.empty((T, 4), dtype=torch.float32, device="cuda")
    ctx.select_routing(to_dev(torch, scores), to_dev(torch, bias), K, ids, w, sel, esc, stats, mode=mode, **kw)
    ctx.sync()
    gi, gw, gs = ids.cpu().numpy().view(np.uint32), w.cpu().numpy(), sel.cpu().numpy()
    ge, gst = esc.cpu().numpy(), stats.cpu().numpy()
    checked = 0
    for t in range(T):
        st, d = rs.select_routing(scores[t], bias, K, mode=mode, **kw)
        assert st == 0
        order = d["full_order"][:K]
        d["_probs"] = scores[t][order] / np.float32(np.sum(scores[t][order], dtype=np.float32))
        if _routing_borderline(d, mode, kw):
            continue
        k = d["selected_k"]
        assert gs[t] == k, (t, gs[t], k)
        np.testing.assert_array_equal(gi[t, :k], d["expert_ids"])
        np.testing.assert_array_equal(gw[t, :k], d["weights"])
        assert bool(ge[t]) == d["escalated"]
        np.testing.assert_allclose(gst[t], [d["normalized_entropy"], d["support"], d["mass"], d["boundary"]],
                                   rtol=1e-6, atol=1e-7)
        checked += 1
    assert checked >= T - 2


def test_select_routing_rejects_bad_policy(torch, ctx):
    import k3xb
    s = torch.full((2, 16), 0.5, dtype=torch.float32, device="cuda")
    b = torch.zeros(16, dtype=torch.float32, device="cuda")
    ids = torch.empty((2, 16), dtype=torch.int32, device="cuda")
    w = torch.empty((2, 16), dtype=torch.float32, device="cuda")
    sel = torch.empty(2, dtype=torch.int32, device="cuda")
    for kw in (dict(mode=1, fixed_k=2), dict(mode=2, quality_floor_k=5), dict(mode=2, mass_target=float("nan"))):
        with pytest.raises(k3xb.K3xbError) as e:
            ctx.select_routing(s, b, 16, ids, w, sel, **kw)
        assert e.value.status == k3xb.INVALID_STATE
