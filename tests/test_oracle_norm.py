"""The oracle's RMSNorm and residual add, pinned to the reference's own tests
(bridge-kernels-reference/tests/norm.rs:11-81) for weighted_rms_norm_into
(src/norm.rs:5-18) and residual_add_in_place (src/norm.rs:83-100). CPU only.
"""

import numpy as np

import oracle as orc


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_weighted_rms_norm_matches_the_scalar_definition():
    # tests/norm.rs:11-26 (the into form; close to 1e-6 absolute)
    eps = np.float32(1.0e-5)
    out = orc.rms_norm(np.array([3.0, 4.0], np.float32), np.array([1.0, 2.0], np.float32), eps)
    scale = np.float32(1.0) / np.sqrt(np.float32(25.0 / 2.0) + eps)
    want = np.array([np.float32(3.0) * scale, np.float32(8.0) * scale], np.float32)
    assert np.all(np.abs(out - want) <= 1.0e-6)


def test_rms_norm_is_the_sequential_f32_definition():
    # rms_scale (norm.rs:144-153): one f32 chain of squares, f32 mean, then
    # 1 / sqrt(mean + eps); output (v * scale) * w, each step rounded to f32
    rng = np.random.default_rng(5)
    x = rng.standard_normal(4096).astype(np.float32)
    w = (rng.random(4096) * 2).astype(np.float32)
    eps = np.float32(1.0e-6)
    s = np.float32(0.0)
    for v in x:
        s = np.float32(s + np.float32(v * v))
    scale = np.float32(1.0) / np.sqrt(np.float32(s / np.float32(x.size)) + eps)
    want = (x * scale).astype(np.float32) * w
    np.testing.assert_array_equal(bits(orc.rms_norm(x, w, eps)), bits(want))


def test_residual_add_is_in_place_and_exact():
    # tests/norm.rs:41-46
    values = np.array([1.0, -2.0, 3.5], np.float32)
    assert orc.residual_add_status(values, np.array([2.0, 1.0, -0.5], np.float32)) == 0
    np.testing.assert_array_equal(values, np.array([3.0, -1.0, 3.0], np.float32))


def test_norm_and_residual_validation_are_atomic():
    # tests/norm.rs:48-81: every error leaves the output untouched
    sentinel = np.array([0x7FC000A5, 0x80000000], np.uint32).view(np.float32)
    out = sentinel.copy()
    st = orc.rms_norm_status(np.array([1.0, 2.0], np.float32), np.array([1.0], np.float32), 1.0e-5, out)
    assert st == 10  # DimensionMismatch (RMSNorm weight, expected 2, actual 1)
    d = orc.last_detail()
    assert (d.expected, d.actual) == (2, 1)
    np.testing.assert_array_equal(bits(out), bits(sentinel))

    st = orc.rms_norm_status(np.array([1.0, np.nan], np.float32), np.array([1.0, 1.0], np.float32), 1.0e-5, out)
    assert st == 12 and orc.last_detail().index == 1  # NonFiniteValue (RMSNorm input, index 1)
    np.testing.assert_array_equal(bits(out), bits(sentinel))

    values = np.array([1.0, 0.0], np.float32)
    before = bits(values).copy()
    out = values.copy()
    mx = np.finfo(np.float32).max
    assert orc.rms_norm_status(values, np.array([mx, mx], np.float32), 1.0e-5, out) != 0
    np.testing.assert_array_equal(bits(out), before)

    residual = np.array([mx, 1.0], np.float32)
    before = bits(residual).copy()
    assert orc.residual_add_status(residual, np.array([mx, 2.0], np.float32)) != 0
    np.testing.assert_array_equal(bits(residual), before)


def test_rms_norm_parameter_checks():
    out = np.zeros(2, np.float32)
    x, w = np.ones(2, np.float32), np.ones(2, np.float32)
    assert orc.rms_norm_status(np.zeros(0, np.float32), np.zeros(0, np.float32), 1e-5, out[:0]) == 15  # empty
    assert orc.rms_norm_status(x, w, 0.0, out) == 15  # epsilon must be > 0
    assert orc.rms_norm_status(x, w, float("inf"), out) == 12  # epsilon finite
    assert orc.rms_norm_status(x, np.array([1.0, np.inf], np.float32), 1e-5, out) == 12  # weight finite
