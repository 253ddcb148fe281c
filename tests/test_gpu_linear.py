"""bf16 linear layer on tcgen05 kind::f16 vs the oracle's bf16_matvec
(runtime/src/official_moe.cpp:39-59, FP64 accumulation + bf16 rounding)."""
import numpy as np
import pytest

from gpu_util import to_dev, torch_cuda
from oracle import bf16_normal, bf16_words

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


@pytest.mark.parametrize("T,K,rows,xkind", [
    (5, 256, 1024, "bf16"),        # c1 LM head
    (64, 7168, 2048, "bf16"),      # shared gate at c2
    (64, 2048, 7168, "f32"),       # shared down at c2 (fp32 activations)
    (3, 7168, 129280, "bf16"),     # c4 LM head, 3 tokens
    (70, 384, 200, "f32"),         # ragged tokens and rows
])
def test_linear_matches_bf16_matvec(torch, ctx, rs, T, K, rows, xkind):
    g = np.random.default_rng(T + K + rows)
    W = bf16_words(g.normal(0, 0.02, size=(rows, K)))
    x = bf16_normal(g, (T, K)) if xkind == "bf16" else (g.normal(size=(T, K)) * 2).astype(np.float32)
    out = torch.empty((T, rows), dtype=torch.float32, device="cuda")
    raw = torch.empty((T, rows), dtype=torch.float32, device="cuda")
    ctx.linear_bf16(to_dev(torch, x), to_dev(torch, W), out, round_output=True)
    ctx.linear_bf16(to_dev(torch, x), to_dev(torch, W), raw, round_output=False)
    ctx.sync()
    got, got_raw = out.cpu().numpy(), raw.cpu().numpy()
    sample = range(T) if T <= 8 else range(0, T, max(1, T // 8))
    w64 = (W.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    for t in sample:
        want = rs.bf16_matvec(x[t], W)
        ref = w64 @ x[t].astype(np.float64)
        # unrounded: FP32 accumulation vs FP64
        np.testing.assert_allclose(got_raw[t], ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())
        # rounded: FP32-vs-FP64 differences of ~1e-6 flip the bf16 rounding when
        # the value sits next to a rounding midpoint: one bf16 step (of the larger
        # binade), rarely
        mag = np.maximum(np.abs(want), np.abs(got[t])) + 1e-30
        # plus an absolute floor of 1e-5 of the output scale: near cancellation
        # the tensor core's FP32 accumulation is ~1e-6 of the operand scale away
        ulp = np.ldexp(1.0, np.floor(np.log2(mag)).astype(int) - 7) + 1e-5 * np.abs(ref).max()
        err = np.abs(got[t] - want)
        bad = np.nonzero(err > ulp)[0]
        assert bad.size == 0, (f"token {t}: {bad.size} elements beyond one bf16 step, first {bad[:3]}: "
                               f"got {got[t][bad[:3]]} raw {got_raw[t][bad[:3]]} want {want[bad[:3]]} "
                               f"fp64 {ref[bad[:3]]}")
        assert (err > 0).mean() < 0.02
