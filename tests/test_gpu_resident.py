"""Resident weights through the C ABI: host arrays uploaded once by tensor
id (k3xb_acquire_weight, k3xb_acquire_expert_stack) and then used by the
kernels. A MoE layer whose experts come from a resident stack must equal
the same layer over caller-owned device copies bit for bit; a resident bf16
weight read back through the tensor-core linear must equal the host words.
The table's hit / bypass / validation rules are the CPU test
test_resident_table.py; here they are checked once through the library."""
import ctypes as C

import numpy as np
import pytest

from gpu_util import layer_to_dev, to_dev, torch_cuda
from oracle import bf16_normal, make_moe_layer

pytestmark = pytest.mark.gpu

DIMS = dict(hidden=256, inter=128, experts=16, top_k=4, shared_inter=128)


def _experts_host(layer):
    return [{name: layer[name][e] for name in ("gate_packed", "gate_scales", "up_packed", "up_scales",
                                               "down_packed", "down_scales")}
            for e in range(layer["experts"])]


def test_resident_stack_layer_equals_device_copies(rs):
    import k3xb
    torch = torch_cuda()
    d = DIMS
    layer = make_moe_layer(rs, 71, d["hidden"], d["inter"], d["experts"], d["top_k"], d["shared_inter"])
    x = to_dev(torch, bf16_normal(np.random.default_rng(72), (9, d["hidden"])))
    dev = layer_to_dev(torch, layer)
    ctx = k3xb.Context(0)
    ctx.use_stream()
    try:
        T, H, K = 9, d["hidden"], d["top_k"]
        want = torch.empty((T, H), dtype=torch.float32, device="cuda")
        want_ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
        ctx.moe_layer_forward(k3xb.moe_layer_desc(dev, engine=k3xb.ENGINE_MXF4), x, want, want_ids)

        stack = ctx.acquire_expert_stack(5, H, d["inter"], _experts_host(layer))
        assert stack.disposition == k3xb.RESIDENT_ADMITTED
        again = ctx.acquire_expert_stack(5, H, d["inter"], _experts_host(layer))
        assert again.disposition == k3xb.RESIDENT_HIT and again.gate_packed == stack.gate_packed
        shared_only = {k: v for k, v in dev.items() if "packed" not in k and "scales" not in k}
        got = torch.empty((T, H), dtype=torch.float32, device="cuda")
        got_ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
        ctx.moe_layer_forward(k3xb.stack_layer_desc(stack, shared_only), x, got, got_ids)
        ctx.sync()
        np.testing.assert_array_equal(got_ids.cpu().numpy(), want_ids.cpu().numpy())
        np.testing.assert_array_equal(got.cpu().numpy(), want.cpu().numpy())
        s = ctx.stats()
        assert s["weight_cache_misses"] == 1 and s["weight_cache_hits"] == 1
        per_expert = 2 * (d["inter"] * H // 2 + d["inter"] * H // 32) + H * d["inter"] // 2 + H * d["inter"] // 32
        assert s["weight_h2d_bytes"] == d["experts"] * per_expert
    finally:
        ctx.close()


def test_resident_bf16_weight_reads_back_through_linear():
    import k3xb
    torch = torch_cuda()
    g = np.random.default_rng(73)
    rows, cols = 128, 64
    words = (g.integers(0, 2, size=(rows, cols)) * 0x8000 + g.integers(0x3c00, 0x4100, size=(rows, cols)))
    words = words.astype(np.uint16)
    ctx = k3xb.Context(0)
    ctx.use_stream()
    try:
        r = ctx.acquire_weight(901, k3xb.WEIGHT_BF16, rows, cols, 0, words)
        assert r.disposition == k3xb.RESIDENT_ADMITTED and r.primary and not r.secondary
        eye = torch.eye(cols, dtype=torch.float32, device="cuda").contiguous()
        out = torch.empty((cols, rows), dtype=torch.float32, device="cuda")
        ctx._check(ctx.lib.k3xb_linear_bf16(ctx.h, k3xb._p(eye), cols, cols, C.c_void_p(r.primary), rows, 0,
                                            k3xb._p(out)), "linear_bf16")
        ctx.sync()
        want = (words.astype(np.uint32) << 16).view(np.float32).T
        np.testing.assert_array_equal(out.cpu().numpy(), want)
        # same key: a hit at the same address; the same id with another shape is refused
        assert ctx.acquire_weight(901, k3xb.WEIGHT_BF16, rows, cols, 0, words).primary == r.primary
        with pytest.raises(k3xb.K3xbError, match="INVALID_EXTENT"):
            ctx.acquire_weight(901, k3xb.WEIGHT_BF16, cols, rows, 0, words)
    finally:
        ctx.close()


def test_resident_mxfp4_admission_and_capacity(rs):
    import k3xb
    torch_cuda()
    w = np.random.default_rng(74).normal(0, 0.02, size=(128, 256)).astype(np.float32)
    packed, scales = rs.quantize_mxfp4(w)
    ctx = k3xb.Context(0)
    ctx.use_stream()
    try:
        r = ctx.acquire_weight(31, k3xb.WEIGHT_MXFP4, 128, 256, 32, packed, scales)
        assert r.disposition == k3xb.RESIDENT_ADMITTED and r.secondary and r.scales_tc
        bad = scales.copy()
        bad[3, 2] = 0xFF
        with pytest.raises(k3xb.K3xbError, match="INVALID_MXFP4"):
            ctx.acquire_weight(32, k3xb.WEIGHT_MXFP4, 128, 256, 32, packed, bad)
        ctx.set_resident_capacity(ctx.stats()["resident_weight_bytes"])
        b = ctx.acquire_weight(33, k3xb.WEIGHT_MXFP4, 128, 256, 32, packed, scales)
        assert b.disposition == k3xb.RESIDENT_BYPASS and not b.primary
        assert ctx.stats()["weight_cache_bypasses"] == 1
        ctx.release_resident()
        assert ctx.stats()["resident_weight_bytes"] == 0
    finally:
        ctx.close()
