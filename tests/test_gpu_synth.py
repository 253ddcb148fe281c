"""The library's seeded generator on the GPU (k3xb_fill_normal_f32 / _bf16
/ _mxfp4, csrc/synth.cu) equals its C restatement
(oracle/k3x_oracle.c:k3xo_fill_normal_*) bit for bit, whole arrays and
slices: a CPU can rebuild any part of a workload the GPU generates in place
(bench.py's reference arm builds its weights this way)."""
import numpy as np
import pytest

from gpu_util import torch_cuda

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


def test_f32_and_bf16_bit_identical(torch, ctx, rs):
    for seed, stream, n, mean, sigma in ((1, 21, 1 << 20, 0.0, 0.02), (3, 81, 100003, 0.25, 0.05),
                                         (4, 5, 7, -1.0, 2.0)):
        t = torch.empty(n, dtype=torch.float32, device="cuda")
        ctx.fill_normal_f32(t, seed, stream, mean, sigma)
        np.testing.assert_array_equal(t.cpu().numpy().view(np.uint32),
                                      rs.fill_normal_f32(n, seed, stream, 0, mean, sigma).view(np.uint32))
        w = torch.empty(n, dtype=torch.int16, device="cuda")
        ctx.fill_normal_bf16(w, seed, stream, sigma)
        np.testing.assert_array_equal(w.cpu().numpy().view(np.uint16), rs.fill_normal_bf16(n, seed, stream, 0, sigma))


def test_mxfp4_bit_identical_including_an_expert_slice(torch, ctx, rs):
    E, rows, cols = 6, 256, 512          # a stack of 6 experts of [256][512]
    packed = torch.empty((E * rows, cols // 2), dtype=torch.uint8, device="cuda")
    scales = torch.empty((E * rows, cols // 32), dtype=torch.uint8, device="cuda")
    ctx.fill_normal_mxfp4(packed, scales, E * rows, cols, 1, 10, 0.02)
    gp, gs = packed.cpu().numpy().reshape(-1), scales.cpu().numpy().reshape(-1)
    wp, ws = rs.fill_normal_mxfp4(E * rows * cols // 32, 1, 10, 0, 0.02)
    np.testing.assert_array_equal(gp, wp)
    np.testing.assert_array_equal(gs, ws)
    per = rows * cols // 32                    # 32-blocks per expert
    sp, ss = rs.fill_normal_mxfp4(per, 1, 10, 4 * per, 0.02)   # expert 4 alone
    np.testing.assert_array_equal(sp, gp[4 * per * 16:5 * per * 16])
    np.testing.assert_array_equal(ss, gs[4 * per:5 * per])
