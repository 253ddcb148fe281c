"""Phase timing (k3xb_set_profiling / k3xb_get_profile) on one MoE layer
and one KDA block: every phase the call ran is timed once per call with a
positive device time, nothing is dropped, switching it off clears the
totals, and the outputs do not change when it is on."""
import numpy as np
import pytest

from gpu_util import layer_to_dev, to_dev, torch_cuda
from oracle import bf16_normal, make_moe_layer

pytestmark = pytest.mark.gpu


def test_phase_profile_moe_layer(rs):
    import k3xb
    torch = torch_cuda()
    layer = make_moe_layer(rs, 91, 256, 128, 16, 4, 128)
    x = to_dev(torch, bf16_normal(np.random.default_rng(92), (7, 256)))
    ctx = k3xb.Context(0)
    ctx.use_stream()
    try:
        d = layer_to_dev(torch, layer)
        desc = k3xb.moe_layer_desc(d, engine=k3xb.ENGINE_MXF4)
        plain = torch.empty((7, 256), dtype=torch.float32, device="cuda")
        ctx.moe_layer_forward(desc, x, plain)
        ctx.sync()
        ctx.set_profiling(True)
        timed = torch.empty_like(plain)
        for _ in range(3):
            ctx.moe_layer_forward(desc, x, timed)
        ctx.sync()
        prof = ctx.profile()
        assert prof.pop("dropped") == 0
        for phase in ("route", "plan", "expert_prep", "expert_gateup", "expert_down", "shared", "combine"):
            ms, calls = prof[phase]
            assert calls == 3 and ms > 0.0, (phase, ms, calls)
        assert "kda_recurrence" not in prof
        np.testing.assert_array_equal(timed.cpu().numpy(), plain.cpu().numpy())
        ctx.set_profiling(False)
        assert ctx.profile() == {"dropped": 0}
    finally:
        ctx.close()
