"""The seeded synthetic-workload generator (project-k3x_b200/csrc/synth.cu,
restated in oracle/k3x_oracle.c:k3xo_normal_pair) on the CPU: the C
restatement equals an independent numpy restatement of the same float
operations bit for bit (every numpy float32 operation rounds to nearest,
like the C file compiled without contraction), slices equal the whole, and
the draws are standard normal in distribution. The GPU kernels are pinned
to the C restatement in test_gpu_synth.py."""
import numpy as np

f32 = np.float32


def _mix64(z):
    with np.errstate(over="ignore"):
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def _hexf(s):
    return f32(float.fromhex(s))


def _log(k):
    e = np.floor(np.log2(k.astype(np.float64))).astype(np.int64)   # exact for k < 2^25
    mant = np.where(e <= 23, k.astype(np.uint64) << (23 - e).clip(0).astype(np.uint64),
                    k.astype(np.uint64) >> (e - 23).clip(0).astype(np.uint64))
    m = ((mant & np.uint64(0x7FFFFF)) | np.uint64(0x3F800000)).astype(np.uint32).view(np.float32)
    big = m > _hexf("0x1.6a09e6p+0")
    m = np.where(big, m * f32(0.5), m).astype(f32)
    e = e + big
    s = (m + f32(-1.0)) / (m + f32(1.0))
    s2 = s * s
    p = np.full_like(s, _hexf("0x1.745d18p-4"))
    for c in ("0x1.c71c72p-4", "0x1.24924ap-3", "0x1.99999ap-3", "0x1.555556p-2"):
        p = p * s2 + _hexf(c)
    p = p * s2 + f32(1.0)
    return (e - 24).astype(f32) * _hexf("0x1.62e430p-1") + (f32(2.0) * s) * p


def _cos_sin(k):
    q = k >> np.uint32(22)
    f = (k & np.uint32(0x3FFFFF)).astype(f32) * f32(2.0 ** -24)
    x = f * _hexf("0x1.921fb6p+2")
    x2 = x * x
    c = np.full_like(x, _hexf("-0x1.93974cp-37"))
    for v in ("0x1.1eed8ep-29", "-0x1.27e4fcp-22", "0x1.a01a02p-16", "-0x1.6c16c2p-10", "0x1.555556p-5"):
        c = c * x2 + _hexf(v)
    c = c * x2 + f32(-0.5)
    c = c * x2 + f32(1.0)
    sn = np.full_like(x, _hexf("-0x1.ae7f3ep-41"))
    for v in ("0x1.612462p-33", "-0x1.ae6456p-26", "0x1.71de3ap-19", "-0x1.a01a02p-13", "0x1.111112p-7",
              "-0x1.555556p-3"):
        sn = sn * x2 + _hexf(v)
    sn = (sn * x2) * x + x
    cs = np.select([q == 0, q == 1, q == 2], [c, -sn, -c], sn)
    sc = np.select([q == 0, q == 1, q == 2], [sn, c, -sn], -c)
    return cs, sc


def numpy_pairs(seed, stream, first_pair, n_pairs):
    i = np.arange(first_pair, first_pair + n_pairs, dtype=np.uint64)
    r = _mix64(_mix64(_mix64(np.uint64(seed)) ^ np.uint64(stream)) ^ i)
    k1 = (r >> np.uint64(40)).astype(np.uint32) + np.uint32(1)
    k2 = ((r >> np.uint64(16)) & np.uint64(0xFFFFFF)).astype(np.uint32)
    rad = np.sqrt(f32(-2.0) * _log(k1))
    c, s = _cos_sin(k2)
    return rad * c, rad * s


def test_c_restatement_equals_numpy_restatement(rs):
    for seed, stream in ((1, 10), (3, 71), (0xDEADBEEF, 5)):
        z0, z1 = numpy_pairs(seed, stream, 1000, 20000)
        want = np.stack([z0, z1], axis=1).reshape(-1)
        got = rs.fill_normal_f32(40000, seed, stream, first=2000)
        np.testing.assert_array_equal(got.view(np.uint32), want.astype(f32).view(np.uint32))


def test_slices_equal_the_whole_and_quantisation(rs):
    whole = rs.fill_normal_f32(4096, 7, 3)
    np.testing.assert_array_equal(rs.fill_normal_f32(1001, 7, 3, first=1033), whole[1033:2034])
    words = rs.fill_normal_bf16(4096, 7, 3, sigma=0.5)
    np.testing.assert_array_equal(words, rs.fill_normal_bf16(4096, 7, 3, first=0, sigma=0.5))
    np.testing.assert_array_equal(np.asarray(words, np.uint32),
                                  (rs.round_bf16(f32(0.5) * whole).view(np.uint32) >> 16))
    packed, scales = rs.fill_normal_mxfp4(128, 9, 4, sigma=0.02)
    p2, s2 = rs.fill_normal_mxfp4(16, 9, 4, first=40, sigma=0.02)
    np.testing.assert_array_equal(p2, packed[40 * 16:56 * 16])
    np.testing.assert_array_equal(s2, scales[40:56])
    x = f32(0.02) * rs.fill_normal_f32(128 * 32, 9, 4)
    qp, qs = rs.quantize_mxfp4(x.reshape(128, 32))
    np.testing.assert_array_equal(qp.reshape(-1), packed)
    np.testing.assert_array_equal(qs.reshape(-1), scales)


def test_draws_are_standard_normal(rs):
    z = rs.fill_normal_f32(1 << 20, 11, 1).astype(np.float64)
    assert abs(z.mean()) < 5e-3 and abs(z.std() - 1.0) < 5e-3
    qs = np.quantile(z, [0.025, 0.16, 0.5, 0.84, 0.975])
    np.testing.assert_allclose(qs, [-1.95996, -0.99446, 0.0, 0.99446, 1.95996], atol=0.01)
