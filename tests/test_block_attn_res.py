"""Pins the restatement of the block attention residual with many sources
(Engine::attention_residual, runtime/src/model.cpp:645-666) on the CPU:
  * the reference's known-answer case (tests/python/test_attn_res.py),
  * the reference's torch form (reference/k3x_ref/attn_res.py:9-23) on the
    committed fixture tests/golden/block_attn_res.npz, to float tolerance
    (torch sums in its own order),
  * its key, rms_norm (ops.cpp:10-18), bit for bit against the reference's
    compiled rms_norm (oracle/_ref).
"""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "block_attn_res.npz")


def test_known_answer(rs):
    # tests/python/test_attn_res.py: eps 0, unit norm, projection (1, 0)
    out = rs.block_attention_residual(np.array([[1.0, 1.0]]), np.array([[[3.0, 0.0]], [[0.0, 4.0]]]), np.ones(2),
                                      np.array([1.0, 0.0]), 0.0)
    np.testing.assert_allclose(out, [[1.9227442, 0.85785025]], atol=1e-6)
    z = np.load(GOLDEN)
    np.testing.assert_allclose(out, z["kat_out"], atol=1e-6)


def test_matches_torch_reference_fixture(rs):
    z = np.load(GOLDEN)
    out = rs.block_attention_residual(z["prefix"], z["sources"], z["norm"], z["proj"], float(z["eps"]))
    want = z["torch_out"]
    scale = np.abs(np.concatenate([z["sources"], z["prefix"][None]])).max()
    assert np.abs(out - want).max() <= 1e-6 * scale, np.abs(out - want).max()


def test_key_is_the_reference_rms_norm(rs, ref):
    g = np.random.default_rng(1017)
    for n in (1, 2, 255, 7168):
        x = (g.normal(size=n) * 3).astype(np.float32)
        w = g.normal(size=n).astype(np.float32)
        for eps in (0.0, 1e-6, 1e-5):
            assert np.array_equal(rs.rms_norm_f32(x, w, eps), ref.rms_norm_f32(x, w, eps))


def test_no_sources_is_the_prefix(rs):
    # one value: softmax gives 1, and 0 + 1 * v is v
    g = np.random.default_rng(1019)
    prefix = g.normal(size=(3, 64)).astype(np.float32)
    out = rs.block_attention_residual(prefix, np.zeros((0, 3, 64), np.float32), np.ones(64, np.float32),
                                      g.normal(size=64).astype(np.float32), 1e-6)
    assert np.array_equal(out, prefix)


def test_output_is_a_convex_combination(rs):
    g = np.random.default_rng(1021)
    S, T, H = 6, 4, 96
    values = g.normal(size=(S + 1, T, H)).astype(np.float32)
    out = rs.block_attention_residual(values[S], values[:S], np.ones(H, np.float32),
                                      g.normal(size=H).astype(np.float32), 1e-6)
    lo, hi = values.min(axis=0), values.max(axis=0)
    slack = 1e-6 * np.abs(values).max()
    assert np.all(out >= lo - slack) and np.all(out <= hi + slack)


def test_identical_sources_average_to_themselves(rs):
    # equal values give equal scores, p = 1/(S+1) each
    g = np.random.default_rng(1023)
    row = g.normal(size=(2, 128)).astype(np.float32)
    sources = np.stack([row, row, row])
    out = rs.block_attention_residual(row, sources, np.ones(128, np.float32),
                                      g.normal(size=128).astype(np.float32), 1e-6)
    np.testing.assert_allclose(out, row, rtol=1e-6, atol=1e-7)
