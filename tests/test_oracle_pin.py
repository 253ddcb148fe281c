"""Pins the C restatement (oracle/k3x_oracle.c) before anything is checked
against it:
  * against the reference's golden literals and known-answer tests
    (tests/cpp/test_official_moe.cpp, test_expert_major.cpp,
    test_speculative.cpp, reference/k3x_ref/fixtures.py), and
  * bit for bit against the reference's own compiled CPU code
    (oracle/_ref/libk3x_ref.so) on seeded random inputs.
CPU only.
"""
import numpy as np
import pytest

from oracle import (ACT_SITU, ACT_SWIGLU, OracleError, bf16_normal, bf16_values, bf16_words,
                    make_moe_layer)


# ---------------------------------------------------------------- MXFP4 ----

def test_mxfp4_known_answer(rs):
    # reference/k3x_ref/fixtures.py:265 — 0x10 then zeros, scale 127, 1x32
    packed = np.array([0x10] + [0] * 15, np.uint8)
    out = rs.decode_mxfp4(packed, np.array([127], np.uint8), 1, 32)
    assert out[0, 0] == 0.0 and out[0, 1] == 0.5 and not out[0, 2:].any()


def test_mxfp4_reserved_scale_rejected(rs):
    # ops.cpp:46-48: scale byte 0xFF is reserved
    packed = np.zeros(16, np.uint8)
    with pytest.raises(OracleError) as e:
        rs.decode_mxfp4(packed, np.array([0xFF], np.uint8), 1, 32)
    assert e.value.status == 15
    with pytest.raises(OracleError):
        rs.mxfp4_matmul(np.zeros(32, np.float32), packed, np.array([0xFF], np.uint8), 1, 32)


def test_mxfp4_bad_extent_rejected(rs):
    with pytest.raises(OracleError):
        rs.decode_mxfp4(np.zeros(8, np.uint8), np.zeros(1, np.uint8), 1, 17, 17)


def test_mxfp4_decode_and_matmul_match_reference(rs, ref):
    g = np.random.default_rng(11)
    rows, cols = 48, 256
    packed = g.integers(0, 256, size=rows * cols // 2, dtype=np.uint8)
    scales = g.integers(100, 140, size=rows * cols // 32, dtype=np.uint8)
    x = g.normal(size=cols).astype(np.float32)
    np.testing.assert_array_equal(rs.decode_mxfp4(packed, scales, rows, cols),
                                  ref.decode_mxfp4(packed, scales, rows, cols))
    np.testing.assert_array_equal(rs.mxfp4_matmul(x, packed, scales, rows, cols),
                                  ref.mxfp4_matmul(x, packed, scales, rows, cols))


def test_quantizer_roundtrip_bounds(rs):
    g = np.random.default_rng(3)
    w = g.normal(0, 0.02, size=(64, 256)).astype(np.float32)
    packed, scales = rs.quantize_mxfp4(w)
    dec = rs.decode_mxfp4(packed, scales, 64, 256)
    blocks = np.abs(w).reshape(64, 8, 32).max(axis=2)
    step = np.ldexp(1.0, scales.astype(np.int32) - 127)           # 2^s
    # amax <= 6 * 2^s and not representable one exponent lower
    assert np.all(blocks <= 6 * step) and np.all(blocks > 3 * step)
    # error at most half the coarsest grid spacing (2 * 2^s) per block
    err = np.abs(dec - w).reshape(64, 8, 32).max(axis=2)
    assert np.all(err <= step)


def test_e2m1_terms_exact_decomposition(rs):
    g = np.random.default_rng(5)
    for scale in (1.0, 1e-3, 37.0):
        x = (g.normal(size=32) * scale).astype(np.float32)
        for nterms in (1, 2, 4, 6, 8):
            packed, scales, res = rs.e2m1_terms(x, nterms)
            recon = np.zeros(32, np.float64)
            for t in range(nterms):
                recon += rs.decode_mxfp4(packed[t], scales[t:t + 1], 1, 32)[0].astype(np.float64)
            resid = np.abs(x.astype(np.float64) - recon).max()
            assert resid == pytest.approx(res, rel=0, abs=0)
            # each term removes at least two bits of the block maximum
            assert resid <= np.abs(x).max() * 2.0 ** (-2 * nterms + 1)


_E2M1_GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def _rne_e2m1(v):
    """Round to nearest on the E2M1 grid, ties to the even code (mantissa bit
    0), saturating at 6; the sign bit only on a nonzero code."""
    a = abs(float(v))
    d = np.abs(_E2M1_GRID - min(a, 6.0))
    best = np.flatnonzero(d == d.min())
    code = int(best[0]) if len(best) == 1 else int(best[best % 2 == 0][0])
    return code | (8 if (np.signbit(v) and code) else 0)


def test_e2m1_split_rounding_is_round_half_even(rs):
    """The split's per-element rule is round-half-even onto the E2M1 grid with
    saturation at 6, and a negative value that rounds to zero gets code 0.
    That is what lets the device split use the hardware conversion
    (cvt.rn.satfinite.e2m1x2.f32, plus a fix-up of -0 codes) and stay
    bit-identical. A block whose maximum is 6 has scale exponent 0, so its
    first term's codes are the rounding of the values themselves."""
    g = np.random.default_rng(17)
    ties = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])
    near = np.concatenate([np.nextafter(ties.astype(np.float32), np.float32(0)),
                           np.nextafter(ties.astype(np.float32), np.float32(7))])
    vals = np.concatenate([np.arange(-384, 385) / 64.0, ties, -ties, near, -near, g.uniform(-6, 6, 500),
                           [0.0, -0.0, -1e-30, 1e-30, -0.2, 5.999, -5.5]]).astype(np.float32)
    for i in range(0, len(vals), 31):
        chunk = vals[i:i + 31]
        block = np.zeros(32, np.float32)
        block[0] = 6.0
        block[1:1 + len(chunk)] = chunk
        packed, scales, _ = rs.e2m1_terms(block, 1)
        assert scales[0] == 127
        for j in range(32):
            nib = (int(packed[0][j // 2]) >> (4 * (j % 2))) & 15
            assert nib == _rne_e2m1(block[j]), (block[j], nib)


def test_e2m1_negative_zero_fixup_arithmetic():
    """The device split's fix-up after the hardware conversion
    (experts_tc.cu:e2m1_pack8): mag = w & 0x77777777, and
    (mag + 0x77777777) & 0x88888888 marks the nibbles with a nonzero
    magnitude, so mag | (w & that) keeps a sign bit only there."""
    g = np.random.default_rng(19)
    words = np.concatenate([g.integers(0, 2 ** 32, size=20000, dtype=np.uint64),
                            [0x88888888, 0x80000008, 0xF0F0F0F0, 0x08080808, 0]]).astype(np.uint64)
    for w in words.tolist():
        mag = w & 0x77777777
        fixed = mag | (w & ((mag + 0x77777777) & 0x88888888))
        want = 0
        for k in range(8):
            n = (w >> (4 * k)) & 15
            want |= (n if n & 7 else 0) << (4 * k)
        assert fixed == want, hex(w)


# ---------------------------------------------------------- activations ----

def test_situ_glu_matches_reference(rs, ref):
    g = np.random.default_rng(7)
    gate = (g.normal(size=1000) * 4).astype(np.float32)
    up = (g.normal(size=1000) * 40).astype(np.float32)
    np.testing.assert_array_equal(rs.situ_glu(gate, up, 4.0, 25.0), ref.situ_glu(gate, up, 4.0, 25.0))
    np.testing.assert_array_equal(rs.situ_glu(gate, up, 4.0), ref.situ_glu(gate, up, 4.0))


def test_swiglu_is_situ_limit(rs, ref):
    # SwiGLU = situ_glu(beta = 2^64, no linear bound), bit for bit
    g = np.random.default_rng(8)
    gate = (g.normal(size=4096) * 3).astype(np.float32)
    up = g.normal(size=4096).astype(np.float32)
    np.testing.assert_array_equal(rs.swiglu(gate, up), ref.situ_glu(gate, up, 2.0 ** 64))


def test_situ_literal(rs):
    # fixtures.py:263 situ_glu([[-1, 2]], [[3, 4]], 1, 1) — recomputed here in float64
    gate = np.array([-1.0, 2.0], np.float32)
    up = np.array([3.0, 4.0], np.float32)
    out = rs.situ_glu(gate, up, 1.0, 1.0)
    sig = 1 / (1 + np.exp(-gate.astype(np.float64)))
    expect = np.tanh(gate) * sig * np.tanh(up)
    np.testing.assert_allclose(out, expect, rtol=1e-6)


# --------------------------------------------------------------- router ----

ROUTER = np.array([0x3F80, 0x0000, 0x0000, 0x3F80, 0xBF80, 0x3F80], np.uint16).reshape(3, 2)
CORRECTION = np.array([0.0, 0.1, -0.05], np.float32)
HIDDEN = np.array([1.2578125, -0.32421875], np.float32)


def test_route_literals(rs):
    # test_official_moe.cpp:86-91
    ids, contrib = rs.route(HIDDEN, ROUTER, CORRECTION, 2)
    assert ids.tolist() == [0, 1]
    assert abs(contrib[0] - 0.6497964859) <= 1e-6 and abs(contrib[1] - 0.3502035439) <= 1e-6
    # :92-100 logits entry point gives identical ids/scores/contributions
    logits = np.array([1.2578125, -0.32421875, -1.58203125], np.float32)
    ids2, c2, s2 = rs.route_logits(logits, CORRECTION, 2, want_scores=True)
    assert ids2.tolist() == ids.tolist() and np.array_equal(c2, contrib)
    # :101-109 ties break to the lower index
    ids3, c3, s3 = rs.route_logits(np.zeros(3, np.float32), np.zeros(3, np.float32), 2,
                                   want_scores=True)
    assert ids3.tolist() == [0, 1] and s3.tolist() == [0.5] * 3 and c3.tolist() == [0.5, 0.5]


@pytest.mark.parametrize("logits,corr,k", [
    ([0.0, np.inf, 0.0], [0, 0, 0], 2),       # non-finite logit
    ([0.0, 0.0, 0.0], [0, 0, 0], 0),          # top_k == 0
    ([0.0, 0.0, 0.0], [0, 0, 0], 4),          # top_k > experts
    ([-3.4028235e38] * 3, [0, 0, 0], 2),      # zero mass
])
def test_route_rejects(rs, logits, corr, k):
    # test_official_moe.cpp:110-127
    with pytest.raises(OracleError):
        rs.route_logits(np.array(logits, np.float32), np.array(corr, np.float32), k)


def test_route_matches_reference_random(rs, ref):
    g = np.random.default_rng(12)
    E, H, K = 64, 512, 8
    router = bf16_words(g.normal(0, 0.02, size=(E, H)))
    corr = g.normal(0, 0.02, size=E).astype(np.float32)
    for _ in range(20):
        x = bf16_normal(g, H)
        a = rs.route(x, router, corr, K)
        b = ref.route(x, router, corr, K)
        assert a[0].tolist() == b[0].tolist()
        np.testing.assert_array_equal(a[1], b[1])


# ---------------------------------------------------------- bucketing ----

def test_expert_major_known_answers(rs):
    # test_expert_major.cpp:24-51
    plan = rs.expert_major_plan(np.array([[2, 1], [1, 3]]), np.array([[0.6, 0.4], [0.7, 0.3]]))
    assert plan["group_expert"].tolist() == [2, 1, 3]
    assert plan["group_offset"].tolist() == [0, 1, 3, 4]
    assert plan["assign_token"].tolist() == [0, 0, 1, 1]
    assert plan["assign_slot"].tolist() == [0, 1, 0, 1]
    assert plan["assign_contrib"].tolist() == pytest.approx([0.6, 0.4, 0.7, 0.3])
    # :52-62
    plan = rs.expert_major_plan(np.array([[4], [5]]), np.array([[1.0], [1.0]]))
    assert plan["group_expert"].tolist() == [4, 5]


@pytest.mark.parametrize("ids,contrib,status", [
    ([[1, 1]], [[0.5, 0.5]], 16),                 # duplicate expert (:81-86)
    ([[1]], [[np.nan]], 16),                      # NaN contribution (:87-93)
    ([[1]], [[np.inf]], 16),                      # Inf contribution (:94-100)
])
def test_expert_major_rejects(rs, ids, contrib, status):
    with pytest.raises(OracleError) as e:
        rs.expert_major_plan(np.array(ids), np.array(contrib, np.float32))
    assert e.value.status == status


def test_expert_major_matches_reference_random(rs, ref):
    g = np.random.default_rng(13)
    T, E, K = 64, 384, 16
    ids = np.stack([g.choice(E, K, replace=False) for _ in range(T)]).astype(np.uint32)
    con = g.random(size=(T, K)).astype(np.float32)
    a = rs.expert_major_plan(ids, con)
    b = ref.expert_major_plan(ids.tolist(), con.tolist())
    for key in a:
        np.testing.assert_array_equal(a[key], b[key])


# ---------------------------------------------------- expert FFN literals --

def test_official_expert_literals(rs):
    # test_official_moe.cpp:57-63 and :134-136 — 2x2 experts, group 2, SiTU(4, 25)
    latent = HIDDEN
    scales = np.array([127, 127], np.uint8)
    experts = {0: ([0x12, 0x21], [0x22, 0x31], [0x12, 0x21]),
               1: ([0x21, 0x12], [0x12, 0x23], [0x12, 0x12])}
    expect = {0: [0.76171875, 0.3984375], 1: [0.81640625, 0.81640625]}
    outs = []
    for e, (gp, up, dp) in experts.items():
        gate = rs.mxfp4_matmul(latent, np.array(gp, np.uint8), scales, 2, 2, 2)
        upv = rs.mxfp4_matmul(latent, np.array(up, np.uint8), scales, 2, 2, 2)
        act = rs.situ_glu(gate, upv, 4.0, 25.0)
        y = rs.round_bf16(rs.mxfp4_matmul(act, np.array(dp, np.uint8), scales, 2, 2, 2))
        assert np.abs(y - expect[e]).max() <= 1e-6
        outs.append(y)
    # :136 mixed_latent
    _, contrib = rs.route(HIDDEN, ROUTER, CORRECTION, 2)
    mixed = rs.routed_combine(np.stack(outs), contrib)
    assert np.abs(mixed - [0.78125, 0.54296875]).max() <= 1e-6


def test_moe_layer_matches_reference_random(rs, ref):
    for act in (ACT_SWIGLU, ACT_SITU):
        layer = make_moe_layer(rs, 21 + act, hidden=128, inter=64, experts=12, top_k=4,
                               shared_inter=64, activation=act)
        x = bf16_normal(np.random.default_rng(22), (6, 128))
        a = rs.moe_layer(layer, x)
        b = ref.moe_layer(layer, x, threads=2)
        for u, v in zip(a, b):
            np.testing.assert_array_equal(u, v)


# ------------------------------------------------------------------ KDA ----

def _kda_weights(g, H, h, d, W=4):
    P = h * d
    n = lambda *s: bf16_words(g.normal(0, 0.1, size=s))
    return dict(hidden=H, heads=h, head_dim=d, conv_width=W, eps=1e-5, gate_lower_bound=-5.0,
                q_proj=n(P, H), k_proj=n(P, H), v_proj=n(P, H),
                q_conv=g.normal(0, 0.5, size=(P, W)).astype(np.float32),
                k_conv=g.normal(0, 0.5, size=(P, W)).astype(np.float32),
                v_conv=g.normal(0, 0.5, size=(P, W)).astype(np.float32),
                f_a_proj=n(d, H), f_b_proj=n(P, d),
                a_log=g.normal(0, 0.3, size=d).astype(np.float32),
                dt_bias=g.normal(0, 0.3, size=P).astype(np.float32),
                b_proj=n(h, H), g_proj=n(P, H),
                o_norm=(1 + g.normal(0, 0.1, size=d)).astype(np.float32), o_proj=n(H, P))


def test_kda_block_matches_reference(rs, ref):
    g = np.random.default_rng(31)
    H, h, d, W = 64, 2, 16, 4
    w = _kda_weights(g, H, h, d, W)
    P = h * d
    state = [np.zeros((W - 1) * P, np.uint16)] * 3 + [np.zeros(h * d * d, np.float32)]
    for _ in range(2):   # two chunks: the second continues from the first's state
        x = g.normal(size=(5, H)).astype(np.float32)
        a_out, a_state = rs.kda_block(w, x, *state)
        b_out, b_state = ref.kda_block(w, x, *state)
        np.testing.assert_array_equal(a_out, b_out)
        for u, v in zip(a_state, b_state):
            np.testing.assert_array_equal(u, v)
        state = list(a_state)


def test_kda_tree_linear_chain_equals_steps(rs):
    g = np.random.default_rng(33)
    h, d, n = 2, 8, 5
    s0 = g.normal(0, 0.1, size=(h, d, d)).astype(np.float32)
    q, k, v = (g.normal(size=(n, h * d)).astype(np.float32) for _ in range(3))
    ld = -np.abs(g.normal(size=(n, h * d))).astype(np.float32)
    be = g.random(size=(n, h)).astype(np.float32)
    out, states = rs.kda_tree(s0, np.arange(-1, n - 1), q, k, v, ld, be, h, d, want_states=True)
    s = s0
    for i in range(n):
        s, o = rs.kda_step(s, q[i], k[i], v[i], ld[i], be[i], h, d)
        np.testing.assert_array_equal(o, out[i])
        np.testing.assert_array_equal(s, states[i])


def test_kda_tree_rejects_forward_parent(rs):
    with pytest.raises(OracleError):
        z = np.zeros((2, 8), np.float32)
        rs.kda_tree(np.zeros((1, 8, 8), np.float32), np.array([-1, 1]), z, z, z, z,
                    np.zeros((2, 1), np.float32), 1, 8)


# ----------------------------------------------------------- acceptance ----

@pytest.mark.parametrize("anchor,drafts,maxd,targets,expect", [
    (10, [11, 12], 2, [11, 12, 13], (2, [11, 12, 13], True)),        # test_speculative.cpp:155-165
    (10, [99, 100], 2, [11, 12, 13], (0, [11], False)),             # :166-176
    (10, [11, 99], 2, [11, 12, 13], (1, [11, 12], False)),          # :177-187
    (10, [11, 12, 99], 3, [11, 12, 13, 14], (2, [11, 12, 13], False)),  # :188-199
    (10, [], 0, [11], (0, [11], True)),                              # :200-209
])
def test_greedy_block_known_answers(rs, ref, anchor, drafts, maxd, targets, expect):
    got = rs.verify_greedy_block(anchor, np.array(drafts, np.uint32), maxd, 128,
                                 np.array(targets, np.uint32))
    assert got == expect
    assert ref.verify_greedy_block(anchor, np.array(drafts, np.uint32), maxd, 128,
                                   np.array(targets, np.uint32)) == expect


@pytest.mark.parametrize("anchor,drafts,maxd,status", [
    (10, [11, 12], 1, 9),     # too many drafts (invalid_extent)
    (128, [], 0, 9),          # anchor out of vocabulary
    (10, [128], 1, 9),        # draft out of vocabulary
])
def test_greedy_block_rejects(rs, anchor, drafts, maxd, status):
    with pytest.raises(OracleError) as e:
        rs.verify_greedy_block(anchor, np.array(drafts, np.uint32), maxd, 128,
                               np.arange(11, 11 + len(drafts) + 1, dtype=np.uint32))
    assert e.value.status == status


def test_greedy_block_target_out_of_vocab(rs):
    # :235-242 target token >= vocabulary -> invalid_state
    with pytest.raises(OracleError) as e:
        rs.verify_greedy_block(10, np.array([11], np.uint32), 1, 128, np.array([11, 128], np.uint32))
    assert e.value.status == 16


def test_greedy_block_equals_token_major(ref):
    # verify_greedy_draft (token-major, target callback) and the block form agree
    g = np.random.default_rng(41)
    V = 50
    table = g.integers(0, V, size=V)
    for _ in range(50):
        anchor = int(g.integers(V))
        p = int(g.integers(0, 6))
        drafts = g.integers(0, V, size=p).astype(np.uint32)
        # make some prefixes accepted
        tok = anchor
        for i in range(p):
            if g.random() < 0.6:
                drafts[i] = table[tok]
            tok = drafts[i]
        targets = [int(table[anchor])] + [int(table[t]) for t in drafts]
        a = ref.verify_greedy_draft(anchor, drafts, p, V, lambda t: (0, int(table[t])))
        b = ref.verify_greedy_block(anchor, drafts, p, V, np.array(targets, np.uint32))
        assert a == b


def test_argmax_first_maximum(rs):
    x = np.array([1.0, 3.0, 2.0, 3.0], np.float32)
    assert rs.argmax(x) == 1


def test_rejection_sampling_distribution(rs):
    # The residual rule makes the committed token at the first position
    # distributed as p, whatever q is: check empirically on a tiny vocab.
    V = 6
    g = np.random.default_rng(51)
    tl = g.normal(size=(2, V)).astype(np.float32)
    dl = g.normal(size=(1, V)).astype(np.float32)
    p = np.exp(tl[0] - tl[0].max()); p /= p.sum()
    q = np.exp(dl[0] - dl[0].max()); q /= q.sum()
    counts = np.zeros(V)
    n = 6000
    for s in range(n):
        d = int(g.choice(V, p=q))
        _, com = rs.verify_rejection(tl, dl, np.array([d], np.uint32), 1.0, 1234, s)
        counts[com[0]] += 1
    assert np.abs(counts / n - p).max() < 0.03


def test_rejection_deterministic(rs):
    g = np.random.default_rng(52)
    V = 300
    tl = g.normal(size=(4, V)).astype(np.float32)
    dl = g.normal(size=(3, V)).astype(np.float32)
    d = np.array([int(np.argmax(tl[i])) for i in range(3)], np.uint32)
    a = rs.verify_rejection(tl, dl, d, 1.0, 9, 3)
    b = rs.verify_rejection(tl, dl, d, 1.0, 9, 3)
    assert a == b and 1 <= len(a[1]) <= 4


def test_prepare_input_matches_reference(rs, ref):
    """attention_residual + rms_norm (official_layer.cpp:42-125) composed in
    the restatement == the reference's prepare_official_moe_input."""
    g = np.random.default_rng(41)
    for n in (64, 256, 7168):
        prefix = bf16_normal(g, n)
        block = (g.normal(size=n) * 3).astype(np.float32)
        norm = bf16_words(1 + g.normal(0, 0.1, size=n))
        proj = bf16_words(g.normal(0, 0.05, size=n))
        post = bf16_words(1 + g.normal(0, 0.1, size=n))
        a = rs.prepare_input(prefix, block, norm, proj, post, 1e-6)
        b = ref.prepare_input(prefix, block, norm, proj, post, 1e-6)
        np.testing.assert_array_equal(a, b)


def test_kda_block_tree_on_a_chain_is_the_block(rs):
    g = np.random.default_rng(43)
    H, h, d, W, N = 64, 2, 16, 4, 5
    w = _kda_weights(g, H, h, d, W)
    P = h * d
    conv = tuple(bf16_words(g.normal(0, 0.5, size=(W - 1) * P)) for _ in range(3))
    rec = g.normal(0, 0.1, size=h * d * d).astype(np.float32)
    x = g.normal(size=(N, H)).astype(np.float32)
    want, st = rs.kda_block(w, x, *conv, rec)
    got = rs.kda_block_tree(w, x, np.arange(-1, N - 1), conv, rec)
    np.testing.assert_array_equal(got, want)
    # a branch sees only its own ancestors: node 3 hangs off node 1
    parent = np.array([-1, 0, 1, 1])
    tree = rs.kda_block_tree(w, x[:4], parent, conv, rec)
    alt, _ = rs.kda_block(w, x[[0, 1, 3]], *conv, rec)
    np.testing.assert_array_equal(tree[3], alt[2])
    c = rs.kda_block_commit(w, x, np.arange(-1, N - 1), N - 1, conv, rec)
    for u, v in zip(c, st):
        np.testing.assert_array_equal(u, v)


# ------------------------------------------------------ routing policy ----

def _same_routing(a, b):
    assert a[0] == b[0]
    if a[0]:
        return
    x, y = a[1], b[1]
    for k in ("full_order", "expert_ids", "weights"):
        np.testing.assert_array_equal(x[k], y[k])
    for k in ("selected_k", "escalated", "normalized_entropy", "support", "mass", "boundary"):
        assert x[k] == y[k], k


@pytest.mark.parametrize("mode,kw", [
    (0, {}), (0, dict(quality_floor_k=16)),
    (1, dict(fixed_k=4)), (1, dict(fixed_k=8, quality_floor_k=12)),
    (2, dict(mass_target=0.75, minimum_gap=0.1)), (2, dict(mass_target=0.9, quality_floor_k=12)),
    (2, dict(mass_target=0.5, minimum_gap=0.0)),
])
def test_select_routing_matches_reference(rs, ref, mode, kw):
    """select_routing (routing_policy.cpp:31-159): restatement == reference
    build, bit for bit, on random sigmoid scores with ties and biases."""
    g = np.random.default_rng(100 + mode)
    for trial in range(40):
        E = int(g.choice([16, 32, 64, 384]))
        scores = (1 / (1 + np.exp(-g.normal(0, 2, size=E)))).astype(np.float32)
        if trial % 4 == 0:   # exact ties broken by index
            scores[: E // 2] = scores[0]
        bias = (g.normal(0, 0.05, size=E) * (trial % 3 != 0)).astype(np.float32)
        K = 16 if mode == 2 else int(g.choice([4, 8, 16]))
        _same_routing(rs.select_routing(scores, bias, K, mode=mode, **kw),
                      ref.select_routing(scores, bias, K, mode=mode, **kw))


def test_select_routing_reference_cases(rs):
    """The cases of the reference's test_routing_policy.cpp, on the restatement."""
    close = lambda a, b: abs(a - b) <= 1e-6
    s = np.array([0.8, 0.8, 0.4, 0.7, 0.2, 0.1], np.float32)
    b = np.array([0, 0, 0.5, 0, 0, 0], np.float32)
    st, d = rs.select_routing(s, b, 4)
    assert st == 0 and d["full_order"].tolist() == [2, 0, 1, 3, 4, 5] and d["expert_ids"].tolist() == [2, 0, 1, 3]
    assert all(close(w, v) for w, v in zip(d["weights"], np.float32([0.4, 0.8, 0.8, 0.7]) / np.float32(2.7)))
    assert close(d["mass"], 1.0)
    st, d = rs.select_routing(s, b, 4, quality_floor_k=16)
    assert st == 0 and d["selected_k"] == 4 and not d["escalated"]
    desc = (1 - np.arange(16) * 0.04).astype(np.float32)
    zero = np.zeros(16, np.float32)
    st, d = rs.select_routing(desc, zero, 16, mode=1, fixed_k=4)
    assert st == 0 and d["selected_k"] == 4 and d["expert_ids"].tolist() == [0, 1, 2, 3]
    assert close(float(np.sum(d["weights"], dtype=np.float32)), 1.0) and d["mass"] < 1.0
    eight = np.full(16, 1e-9, np.float32)
    eight[:8] = 1.0
    st, d = rs.select_routing(eight, zero, 16, mode=2, mass_target=0.75, minimum_gap=0.1)
    assert st == 0 and d["selected_k"] == 8 and d["support"] <= 8.0001 and d["boundary"] > 0.9
    st, d = rs.select_routing(eight, zero, 16, mode=2, mass_target=0.75, minimum_gap=0.0, quality_floor_k=12)
    assert st == 0 and d["selected_k"] == 12 and d["escalated"]
    weak = np.full(16, 1e-9, np.float32)
    weak[:8] = 1.0
    weak[8:13] = 0.1
    st, d = rs.select_routing(weak, zero, 16, mode=2, mass_target=0.8, minimum_gap=0.2)
    assert st == 0 and d["selected_k"] == 16
    assert rs.select_routing(desc, zero, 16, mode=1, fixed_k=2)[0] != 0
    assert rs.select_routing(desc, zero, 12, mode=1, fixed_k=16)[0] != 0
    assert rs.select_routing(desc, zero, 16, mode=2, mass_target=float("nan"))[0] != 0
    bad = desc.copy()
    bad[0] = 1.1
    assert rs.select_routing(bad, zero, 16)[0] != 0
    assert rs.select_routing(zero, zero, 16)[0] != 0
    assert rs.select_routing(desc, zero, 16, mode=2, quality_floor_k=5)[0] != 0


def test_latent_moe_matches_reference(rs, ref):
    """LatentMoE: the restatement (prepare_input, then the latent layer, then
    the prefix residual) equals the reference's official_moe_cpu
    (official_moe.cpp:271-344) with its own preparation and routing, bit for
    bit."""
    from oracle import bf16_normal, bf16_words, make_moe_layer
    g = np.random.default_rng(61)
    H, L, T, eps = 256, 128, 4, 1e-6
    layer = make_moe_layer(rs, 62, H, 128, 16, 4, shared_inter=128, latent=L)
    prefix, block = bf16_normal(g, (T, H)), bf16_normal(g, (T, H))
    norm = bf16_words(1 + g.normal(0, 0.1, size=H))
    proj = bf16_words(g.normal(0, 0.05, size=H))
    post = bf16_words(1 + g.normal(0, 0.1, size=H))
    want, want_ids, want_con = ref.official_moe(layer, prefix, block, norm, proj, post, eps)
    layer["latent_eps"] = eps
    hidden = np.stack([rs.prepare_input(prefix[t], block[t], norm, proj, post, eps) for t in range(T)])
    moe, ids, con = rs.moe_layer(layer, hidden)
    got = rs.round_bf16(rs.round_bf16(prefix) + moe)
    np.testing.assert_array_equal(ids, want_ids)
    np.testing.assert_array_equal(con, want_con)
    np.testing.assert_array_equal(got, want)


def test_official_layer_matches_reference(rs, ref):
    """The whole official layer with LatentMoE: the restatement's layer
    composition (attention residual, KDA block, prefix, MoE input, LatentMoE,
    residual) over a chain of positions equals the reference's own
    official_layer_cpu (official_layer.cpp:134-244) bit for bit, outputs,
    routes and the KDA state after the last position."""
    from oracle import bf16_normal, bf16_words, make_layer
    g = np.random.default_rng(63)
    H, h, d, T, W = 256, 2, 64, 4, 4
    P = h * d
    layer = make_layer(rs, 64, H, h, d, 16, 4, 128, 128, latent=128)
    # official_layer_cpu has one epsilon (OfficialKdaConfig::rms_norm_epsilon) for every norm
    layer["moe"]["latent_eps"] = layer["kda"]["eps"] = layer["rms_eps"]
    hidden, block = bf16_normal(g, (T, H)), bf16_normal(g, (T, H))
    conv = tuple(bf16_words(g.normal(0, 0.5, size=(W - 1) * P)) for _ in range(3))
    rec = g.normal(0, 0.05, size=h * d * d).astype(np.float32)
    want, want_ids, (wq, wk, wv, wr) = ref.official_layer(layer, hidden, block, conv, rec)
    got, ids, _, xin = rs.layer_forward(layer, hidden, block, np.arange(-1, T - 1), conv, rec, want_xin=True)
    np.testing.assert_array_equal(ids, want_ids)
    np.testing.assert_array_equal(got, want)
    cq, ck, cv, r = rs.kda_block_commit(layer["kda"], xin, np.arange(-1, T - 1), T - 1, conv, rec)
    for a, b in ((cq, wq), (ck, wk), (cv, wv), (r, wr)):
        np.testing.assert_array_equal(a, b)


def test_two_layer_stack_matches_reference(rs, ref):
    """Layer stacking: the restatement run layer-major (layer 1 over both
    positions, then layer 2 over layer 1's outputs with the same block
    source) equals the reference's official_two_layer_cpu, which runs
    position-major, bit for bit, outputs and both layers' final KDA states."""
    from oracle import bf16_normal, bf16_words, make_layer
    g = np.random.default_rng(65)
    H, h, d, W = 256, 2, 64, 4
    layers = [make_layer(rs, 66 + l, H, h, d, 16, 4, 128, 128, latent=128) for l in range(2)]
    for L in layers:
        L["moe"]["latent_eps"] = L["kda"]["eps"] = L["rms_eps"]
    hidden, block = bf16_normal(g, (2, H)), bf16_normal(g, (2, H))
    convs = [tuple(bf16_words(g.normal(0, 0.5, size=(W - 1) * h * d)) for _ in range(3)) for _ in range(2)]
    recs = [g.normal(0, 0.05, size=h * d * d).astype(np.float32) for _ in range(2)]
    want, want_states = ref.official_two_layer(layers, hidden, block, convs, recs)
    x, parent = hidden, np.arange(-1, 1)
    for l, L in enumerate(layers):
        out, _, _, xin = rs.layer_forward(L, x, block, parent, convs[l], recs[l], want_xin=True)
        state = rs.kda_block_commit(L["kda"], xin, parent, 1, convs[l], recs[l])
        for a, b in zip(state, want_states[l]):
            np.testing.assert_array_equal(a, b)
        x = out
    np.testing.assert_array_equal(x, want)


def test_dense_matvec_and_situ_mlp_match_reference_cpu_backend(rs, ref):
    """The f32 dense product and dense SiTU MLP of the reference CPU backend
    (backend_cpu.cpp:23-47, :107-122, via make_cpu_backend): the restatement
    is bit-identical, over odd shapes and values spanning many binades."""
    g = np.random.default_rng(171)
    for rows, cols in ((1, 1), (7, 33), (130, 257), (64, 1000)):
        w = (g.normal(0, 1, size=(rows, cols)) * np.exp(g.normal(0, 4, size=(rows, cols)))).astype(np.float32)
        x = (g.normal(0, 1, size=cols) * np.exp(g.normal(0, 4, size=cols))).astype(np.float32)
        np.testing.assert_array_equal(rs.dense_matvec(x, w), ref.dense_matvec(x, w))
    inter, cols, out_rows = 48, 96, 80
    gate, up = (g.normal(0, 0.1, size=(inter, cols)).astype(np.float32) for _ in range(2))
    down = g.normal(0, 0.1, size=(out_rows, inter)).astype(np.float32)
    x = g.normal(0, 1, size=cols).astype(np.float32)
    for beta, lin in ((4.0, 0.0), (2.0, 25.0)):
        np.testing.assert_array_equal(rs.dense_situ_mlp(x, gate, up, down, beta, lin),
                                      ref.dense_situ_mlp(x, gate, up, down, beta, lin))


def test_resident_moe_layer_matches_reference_cpu_backend(rs, ref):
    """resident_mxfp4_moe_layer of the reference CPU backend (backend_cpu.cpp:
    305-339): the restated composition is bit-identical."""
    from oracle import make_resident_moe_case
    for seed, lin in ((181, 0.0), (182, 25.0)):
        w, ex, con, x = make_resident_moe_case(rs, seed)
        np.testing.assert_array_equal(rs.resident_moe_layer(w, ex, con, x, 1e-6, 4.0, lin),
                                      ref.resident_moe_layer(w, ex, con, x, 1e-6, 4.0, lin))


def test_plain_layer_matches_reference(rs, ref):
    """The KDA + plain-MoE layer that bench.py's reference arm times
    (ref_shim.cpp:k3xr_plain_layer: the reference's prepare_official_moe_input,
    official_kda_cpu, route_official_moe and expert primitives in
    official_layer_cpu's order) equals the restatement's layer composition
    bit for bit for several sequences on several threads, outputs, routes and
    final KDA states; route_only gives the same routes."""
    from oracle import bf16_normal, bf16_words, make_layer
    g = np.random.default_rng(67)
    H, h, d, T, W, S = 256, 2, 64, 3, 4, 3
    P = h * d
    layer = make_layer(rs, 68, H, h, d, 16, 4, 128, 128)
    layer["kda"]["eps"] = layer["rms_eps"]
    hidden, block = bf16_normal(g, (S, T, H)), bf16_normal(g, (S, T, H))
    conv = np.stack([np.stack([bf16_words(g.normal(0, 0.5, size=(W - 1) * P)) for _ in range(3)])
                     for _ in range(S)])
    rec = g.normal(0, 0.05, size=(S, h, d, d)).astype(np.float32)
    out, ids, conv_after, rec_after = ref.plain_layer(layer, hidden, block, conv, rec, threads=2)
    _, route_ids, _, _ = ref.plain_layer(layer, hidden, block, conv, rec, route_only=True, threads=3)
    np.testing.assert_array_equal(route_ids, ids)
    parent = np.arange(-1, T - 1)
    for s in range(S):
        c = tuple(conv[s])
        want, want_ids, _, xin = rs.layer_forward(layer, hidden[s], block[s], parent, c, rec[s].reshape(-1),
                                                  want_xin=True)
        np.testing.assert_array_equal(out[s], want)
        np.testing.assert_array_equal(ids[s], want_ids)
        cq, ck, cv, r = rs.kda_block_commit(layer["kda"], xin, parent, T - 1, c, rec[s].reshape(-1))
        np.testing.assert_array_equal(conv_after[s], np.stack([cq, ck, cv]))
        np.testing.assert_array_equal(rec_after[s].reshape(-1), r)
