"""The drop-in, whole layers: the reference's own layer drivers,
official_layer_cuda (official_layer.cpp:246-500) and official_two_layer_cuda
(official_two_layer.cpp:102-414), unchanged, drive this library's
ComputeBackend (B200Backend) through oracle/_ref/libk3x_ref_b200.so, built
from the reference's sources where they are (oracle/Makefile). Ordered after
the other GPU files: a driver runs most of the adapter's paths at once.
"""
import numpy as np
import pytest

import golden_util as gu
from test_gpu_latent import assert_mostly_close

pytestmark = pytest.mark.gpu

@pytest.mark.parametrize("route,kda_split", [("host", 0), ("device", 0), ("host", 2), ("device", 3)])
def test_reference_layer_driver_on_the_b200_backend(route, kda_split):
    """The drop-in, whole-layer: the reference's own official_layer_cuda
    (official_layer.cpp:246-500), unchanged, drives this library's
    ComputeBackend (B200Backend: official_kda on k3xb_kda_block_host; host
    route preparation: official_mxfp4_moe_ffn on k3xb_official_moe_ffn_host;
    device route preparation: prepare_official_moe_route on
    k3xb_prepare_moe_route_host, then official_mxfp4_moe_ffn_prepared)
    through oracle/_ref/libk3x_ref_b200.so, against the golden
    official_layer_cpu output with the bars of the test above; the final
    KDA state as well. kda_split > 0 runs the positions as two calls, the
    first with device_seed and the second with device_publish from the
    state the device kept (k3xb_kda_block_held), which must equal one call."""
    from oracle import ReferenceOnB200, have_reference_on_b200
    if not have_reference_on_b200():
        pytest.skip("oracle/_ref/libk3x_ref_b200.so is built where the reference tree is (oracle/Makefile); "
                    "this snapshot has none")
    layer, f = gu.official_layer()
    T = f["hidden"].shape[0]
    out, ids, state = ReferenceOnB200().official_layer(layer, f["hidden"], f["block"],
                                                       (f["conv_q"], f["conv_k"], f["conv_v"]), f["recurrent"],
                                                       device_route=route == "device", kda_split=kda_split)
    same = np.all(ids == f["ids"], axis=1)
    assert same.sum() >= T - 1, f"routes agree on {same.sum()}/{T} positions"
    assert_mostly_close(out[same], f["out"][same], what="official_layer_cuda on B200Backend")
    words = lambda a: (np.asarray(a, np.uint16).astype(np.uint32) << 16).view(np.float32)
    for got, key in zip(state[:3], ("next_conv_q", "next_conv_k", "next_conv_v")):
        assert_mostly_close(words(got), words(f[key]), what=key)
    assert_mostly_close(state[3].reshape(f["next_recurrent"].shape), f["next_recurrent"], what="recurrent state")


@pytest.mark.parametrize("mode", ["host_round_trip", "device_closure"])
def test_reference_two_layer_driver_on_the_b200_backend(rs, ref, mode):
    """The reference's own official_two_layer_cuda (official_two_layer.cpp:
    102-414: each layer's KDA state seeded on the device at position 0 and
    published at position 1; host_round_trip: official_layer_cuda with
    device route preparation per layer; device_closure: official_layer_front
    / _tail with layer 1's output held for layer 2), unchanged, over
    B200Backend, against the reference's
    official_two_layer_cpu run here on the same inputs (the case of
    test_oracle_pin.py::test_two_layer_stack_matches_reference): outputs
    and both layers' final states within the bars above."""
    from oracle import ReferenceOnB200, bf16_normal, bf16_words, have_reference_on_b200, make_layer
    if not have_reference_on_b200():
        pytest.skip("oracle/_ref/libk3x_ref_b200.so is built where the reference tree is (oracle/Makefile); "
                    "this snapshot has none")
    g = np.random.default_rng(65)
    H, h, d, W = 256, 2, 64, 4
    layers = [make_layer(rs, 66 + l, H, h, d, 16, 4, 128, 128, latent=128) for l in range(2)]
    for L in layers:
        L["moe"]["latent_eps"] = L["kda"]["eps"] = L["rms_eps"]
    hidden, block = bf16_normal(g, (2, H)), bf16_normal(g, (2, H))
    convs = [tuple(bf16_words(g.normal(0, 0.5, size=(W - 1) * h * d)) for _ in range(3)) for _ in range(2)]
    recs = [g.normal(0, 0.05, size=h * d * d).astype(np.float32) for _ in range(2)]
    want, want_states = ref.official_two_layer(layers, hidden, block, convs, recs)
    got, got_states, got_ids = ReferenceOnB200().official_two_layer(layers, hidden, block, convs, recs,
                                                                    device_closure=mode == "device_closure")
    # the CPU routes, layer-major through the restatement (equal to the
    # reference's, test_oracle_pin.py): a position is compared where its
    # routes agree in both layers (an FP32 projection can move a score by
    # an ulp across a Top-k boundary)
    x, parent = hidden, np.arange(-1, 1)
    want_ids = []
    for l, L in enumerate(layers):
        x, ids, _, _ = rs.layer_forward(L, x, block, parent, convs[l], recs[l], want_xin=True)
        want_ids.append(ids)
    same = np.array([all(np.array_equal(got_ids[t, l], want_ids[l][t]) for l in range(2)) for t in range(2)])
    assert same.any(), "routes differ at both positions"
    assert_mostly_close(got[same], want[same], what="official_two_layer_cuda on B200Backend")
    if not same.all():   # a flipped route changes what the later layer and state see
        return
    words = lambda a: (np.asarray(a, np.uint16).astype(np.uint32) << 16).view(np.float32)
    for l in range(2):
        for i in range(3):
            assert_mostly_close(words(got_states[l][i]), words(want_states[l][i]), what=f"layer {l + 1} conv {i}")
        assert_mostly_close(got_states[l][3], want_states[l][3], what=f"layer {l + 1} recurrent state")
