"""Pins the restatement of the gated MLA layer and its KV crop
(Engine::mla, runtime/src/model.cpp:755-811; restore, :1235-1251) on the
CPU, before any device path is built on it:
  * against the reference's torch form (reference/k3x_ref/mla.py,
    mla_prefill) on tests/golden/mla.npz at the reference's default
    synthetic config: outputs and the final keys, values and shared keys to
    2e-6 of their largest value (torch sums in its own order);
  * the crop: rolling back to k positions and replaying gives the same bits
    as never having gone past k;
  * the draft-tree form the device path will implement (new; the reference
    verifies chains): a node's output is, bit for bit, the sequential
    prefill over the committed rows and its root-to-node path.
CPU only."""
import os

import numpy as np
import pytest

from oracle import MLA_TENSORS, OracleError

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "mla.npz")


def _weights(z):
    H, nh, qr, kr, qm, qe, vd = (int(v) for v in z["dims"])
    return dict(hidden=H, heads=nh, q_rank=qr, kv_rank=kr, q_main=qm, q_extra=qe, value_dim=vd,
                eps=float(z["eps"]), **{k: z[k] for k in MLA_TENSORS})


def _close(got, want, what):
    bound = 2e-6 * float(np.abs(want).max())
    assert np.abs(got - want).max() <= bound, f"{what}: {np.abs(got - want).max():.3e} > {bound:.3e}"


def test_matches_torch_reference_fixture(rs):
    z = np.load(GOLDEN)
    out, st = rs.mla_prefill(_weights(z), z["x"])
    n = st["length"]
    assert n == z["x"].shape[0]
    _close(out, z["torch_out"], "outputs")
    _close(st["keys"][:n], z["torch_keys"], "keys")
    _close(st["values"][:n], z["torch_values"], "values")
    _close(st["shared"][:n], z["torch_shared"], "shared keys")


def test_crop_then_replay_is_bit_identical(rs):
    z = np.load(GOLDEN)
    w = _weights(z)
    x = z["x"]
    full, _ = rs.mla_prefill(w, x)
    out, st = rs.mla_prefill(w, x)
    for keep in (3, 1, 0):
        rs.mla_crop(st, keep)
        again, st = rs.mla_prefill(w, x[keep:], st)
        assert np.array_equal(again, full[keep:]), keep
    # a rolled-back draft replaced by other rows equals a fresh run over them
    g = np.random.default_rng(23)
    other = g.normal(size=(2, w["hidden"])).astype(np.float32)
    rs.mla_crop(st, 3)
    branch, st = rs.mla_prefill(w, other, st)
    fresh, _ = rs.mla_prefill(w, np.concatenate([x[:3], other]))
    assert np.array_equal(branch, fresh[3:])


def test_crop_and_capacity_rejected(rs):
    z = np.load(GOLDEN)
    w = _weights(z)
    _, st = rs.mla_prefill(w, z["x"][:2], capacity=2)
    with pytest.raises(OracleError):
        rs.mla_crop(st, 3)   # the reference's restore refuses to grow the state
    with pytest.raises(OracleError):
        rs.mla_prefill(w, z["x"][2:3], st)   # no room for a third position


def test_single_position_attends_to_itself(rs):
    """With one position the softmax weight is 1, so the merged heads are
    that position's values: the output is o_proj((values) * sigmoid(g x))
    through the same FP64 products."""
    z = np.load(GOLDEN)
    w = _weights(z)
    x = z["x"][:1]
    out, st = rs.mla_prefill(w, x)
    merged = st["values"][0].reshape(-1).astype(np.float32)
    gate = (np.asarray(w["g_proj"], np.float64) @ x[0].astype(np.float64)).astype(np.float32)
    sig = (np.float32(1) / (np.float32(1) + np.exp(-gate))).astype(np.float32)
    want = (np.asarray(w["o_proj"], np.float64) @ (merged * sig).astype(np.float64)).astype(np.float32)
    _close(out[0], want, "single position")


def _copy_state(st):
    return {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in st.items()}


def test_tree_on_a_chain_is_the_prefill(rs):
    z = np.load(GOLDEN)
    w = _weights(z)
    x = z["x"]
    full, full_st = rs.mla_prefill(w, x)
    _, st = rs.mla_prefill(w, x[:2])
    out, nk, nv, ns = rs.mla_tree(w, st, [-1, 0, 1], x[2:])
    assert np.array_equal(out, full[2:])
    assert np.array_equal(nk, full_st["keys"][2:5]) and np.array_equal(nv, full_st["values"][2:5])
    assert np.array_equal(ns, full_st["shared"][2:5])
    assert st["length"] == 2   # the tree leaves the committed state alone


def test_tree_node_is_the_prefill_of_its_path(rs):
    """Every node of a branching tree gives the bits of a sequential prefill
    over the committed rows and its root-to-node path."""
    z = np.load(GOLDEN)
    w = _weights(z)
    g = np.random.default_rng(29)
    parent = [-1, 0, 0, 1, 1, 2, -1, 6]
    nodes = g.normal(size=(len(parent), w["hidden"])).astype(np.float32)
    _, st = rs.mla_prefill(w, z["x"][:3])
    out, _, _, _ = rs.mla_tree(w, st, parent, nodes)
    for i in range(len(parent)):
        path = []
        a = i
        while a >= 0:
            path.append(a)
            a = parent[a]
        rows = nodes[path[::-1]]
        ref_out, _ = rs.mla_prefill(w, rows, _copy_state(st))
        assert np.array_equal(out[i], ref_out[-1]), i


def test_tree_rejects_forward_parents(rs):
    z = np.load(GOLDEN)
    w = _weights(z)
    _, st = rs.mla_prefill(w, z["x"][:1])
    with pytest.raises(OracleError):
        rs.mla_tree(w, st, [-1, 2, 0], z["x"][1:4])
