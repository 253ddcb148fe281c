"""CPU-side checks of the C ABI: the library loads, exports every symbol that
include/k3xb.h declares, and fails loudly (no CPU fallback) without a GPU."""
import ctypes as C
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "k3xb.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*int\s+(k3xb_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_symbols()
    for required in ("k3xb_create", "k3xb_route", "k3xb_expert_major_plan", "k3xb_moe_layer_forward",
                     "k3xb_moe_layer_forward_host", "k3xb_kda_tree", "k3xb_kda_commit",
                     "k3xb_accept_greedy", "k3xb_accept_rejection"):
        assert required in names


def test_library_exports_every_declared_symbol():
    import k3xb
    lib = k3xb.library()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_no_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import k3xb
    with pytest.raises(k3xb.K3xbError) as e:
        k3xb.Context(0)
    assert e.value.status == k3xb.BACKEND_UNAVAILABLE


def test_null_context_rejected():
    import k3xb
    lib = k3xb.library()
    assert lib.k3xb_sync(None) == k3xb.INVALID_EXTENT
    assert lib.k3xb_destroy(None) == k3xb.OK


def test_resident_entry_points_marshal_and_reject_null_context():
    """The ctypes structs of the resident-weight calls marshal (the same
    code the GPU tests use) and a null context is refused before any CUDA
    call."""
    import ctypes as C

    import numpy as np

    import k3xb
    lib = k3xb.library()
    assert C.sizeof(k3xb.Stats) == 16 * 8
    words = np.zeros((4, 8), np.uint16)
    out = k3xb.Resident()
    assert lib.k3xb_acquire_weight(None, 1, k3xb.WEIGHT_BF16, 4, 8, 0, words.ctypes.data, words.nbytes, None, 0,
                                   C.byref(out)) == k3xb.INVALID_EXTENT
    views = (k3xb.ExpertHost * 2)()
    views[1].down_scales = words.ctypes.data
    stack = k3xb.ResidentStack()
    assert lib.k3xb_acquire_expert_stack(None, 1, 2, 128, 128, views, C.byref(stack)) == k3xb.INVALID_EXTENT
    assert lib.k3xb_set_resident_capacity(None, 0) == k3xb.INVALID_EXTENT
    assert lib.k3xb_release_resident(None) == k3xb.INVALID_EXTENT


def test_profiling_entry_points():
    """Phase names cover every K3XB_PHASE_* value of the header; the calls
    refuse a null context before any CUDA call."""
    import re

    import k3xb
    lib = k3xb.library()
    header = open(HEADER).read()
    block = header[header.index("K3XB_PHASE_ROUTE = 0"):header.index("K3XB_PHASE_COUNT")]
    assert len(re.findall(r"K3XB_PHASE_\w+", block)) == k3xb.PHASE_COUNT
    names = [k3xb.phase_name(i) for i in range(k3xb.PHASE_COUNT)]
    assert all(names) and len(set(names)) == k3xb.PHASE_COUNT and names[0] == "route"
    assert k3xb.phase_name(k3xb.PHASE_COUNT) is None and k3xb.phase_name(-1) is None
    arr = (k3xb.PhaseTime * k3xb.PHASE_COUNT)()
    assert lib.k3xb_set_profiling(None, 1) == k3xb.INVALID_EXTENT
    assert lib.k3xb_get_profile(None, arr, None) == k3xb.INVALID_EXTENT


def test_draft_entry_point_rejects_null_context():
    import ctypes as C

    import k3xb
    lib = k3xb.library()
    io = k3xb.DraftIO(1, 1, 1, None, None, None, None)
    assert lib.k3xb_draft_greedy(None, C.byref(k3xb.VerifyModel()), C.byref(io)) == k3xb.INVALID_EXTENT


def test_ep_balance_deals_by_load():
    """k3xb_ep_balance (host function): experts dealt in descending load over
    the ranks in a snake; every rank gets E/world, local indices 0.. in
    dealing order; ties keep the lower id first; bad arguments are
    INVALID_EXTENT."""
    import k3xb
    E, world = 48, 4
    load = np.random.default_rng(3).random(E).astype(np.float32)
    owner = k3xb.ep_balance(load, world)
    rank, local = owner >> 16, owner & 0xFFFF
    order = np.argsort(-load, kind="stable")
    for i, e in enumerate(order):
        r, p = divmod(i, world)
        assert rank[e] == (p if r % 2 == 0 else world - 1 - p) and local[e] == r
    for g in range(world):
        assert sorted(local[rank == g].tolist()) == list(range(E // world))
    hot = order[:world]
    assert len(set(rank[hot].tolist())) == world          # the heaviest experts on different ranks
    tie = k3xb.ep_balance(np.zeros(8, np.float32), 2)   # all equal: ids in order, snake
    assert (tie >> 16).tolist() == [0, 1, 1, 0, 0, 1, 1, 0] and (tie & 0xFFFF).tolist() == [0, 0, 1, 1, 2, 2, 3, 3]
    with pytest.raises(k3xb.K3xbError):
        k3xb.ep_balance(np.ones(10, np.float32), 4)      # does not split evenly
    with pytest.raises(k3xb.K3xbError):
        k3xb.ep_balance(np.array([1.0, np.nan], np.float32), 2)


def test_default_act_terms_rule():
    """The MXF4 engine's default E2M1 term count (k3xb_default_act_terms, a
    host function): exact 6 terms while experts see fewer than 12 tokens on
    average, 4 from there on."""
    import k3xb
    assert k3xb.default_act_terms(64 * 16, 384) == 6       # c2: ~2.7 tokens per expert
    assert k3xb.default_act_terms(144 * 16, 384) == 6      # c4: 6
    assert k3xb.default_act_terms(576 * 16, 384) == 4      # c5: 24
    assert k3xb.default_act_terms(11 * 384, 384) == 6 and k3xb.default_act_terms(12 * 384, 384) == 4
