"""The CPU restatement against the reference's own known-answer tests
(vectors in tests/golden/reference_kats.json, extracted by make_golden.py)."""

import numpy as np
import pytest


def test_ladder_matches_the_published_bisection_order(oracle_lib, kats):
    assert oracle_lib.ladder_order(20) == kats["ladder_order_20"]
    for depth, layers in kats["ladder_select_20"].items():
        assert oracle_lib.ladder_select(20, int(depth)) == layers
    assert oracle_lib.ladder_select(8, 2) == kats["ladder_select_8_2"]
    for layers, depth in kats["ladder_rejects"]:
        assert oracle_lib.ladder_select(layers, depth) is None
    assert oracle_lib.ladder_select(20, 8) == kats["depth8_layers"]


def test_whistle_sized_ladders_nest(oracle_lib):
    eight, four = oracle_lib.ladder_select(8, 8), oracle_lib.ladder_select(8, 4)
    assert set(four) <= set(eight)


def _dense_hadamard(x):
    n = len(x)
    rows = np.array([[(-1.0) ** bin(r & c).count("1") for c in range(n)] for r in range(n)])
    return rows @ x.astype(np.float64) / np.sqrt(n)


def test_walsh_matches_the_dense_hadamard_matrix(oracle_lib, kats):
    w = kats["walsh"]
    for size in w["sizes"]:
        x = np.array([(((i * w["mul"] + size) % w["mod"]) - w["offset"]) / w["div"] for i in range(size)], dtype=np.float32)
        out = oracle_lib.walsh(x)
        expected = _dense_hadamard(x)
        worst = np.max(np.abs(out - expected) / (1.0 + np.abs(expected)))
        assert worst < w["tolerance"], (size, worst)


def test_walsh_is_an_involution(oracle_lib):
    x = np.sin(np.arange(128, dtype=np.float32) * np.float32(0.37))
    assert np.all(np.abs(oracle_lib.walsh(oracle_lib.walsh(x)) - x) < 1e-5)


@pytest.mark.parametrize("mode", [0, 1])
def test_kronecker_32_matches_double_precision(oracle_lib, kats, mode):
    k = kats["kronecker"]
    n = k["size"]

    def make(seed):
        return np.array([(((i * k["mul"] + seed * k["seed_mul"]) % k["mod"]) - k["offset"]) / k["div"]
                         for i in range(n * n)], dtype=np.float32)

    x, left, right = (make(s) for s in k["seeds"])
    X, Lm, Rm = (a.astype(np.float64).reshape(n, n) for a in (x, left, right))
    expected = (Lm.T @ (X @ Rm)).astype(np.float32).ravel()
    actual = oracle_lib.kronecker(x, left, right, mode)
    worst = np.max(np.abs(expected - actual) / (1.0 + np.abs(expected)))
    assert worst < k["tolerance"]


def test_fast_exp_is_within_the_reference_tolerance(oracle_lib, kats):
    f = kats["fast_exp"]
    x, worst = np.float32(f["start"]), 0.0
    while x <= f["stop"]:
        exact = np.exp(np.float64(x))
        worst = max(worst, abs((oracle_lib.fast_exp(x) - exact) / exact))
        x = np.float32(x + np.float32(f["step"]))
    assert worst < f["tolerance"]
    assert oracle_lib.fast_exp(0.0) == 1.0
    assert 0.0 <= oracle_lib.fast_exp(-200.0) < 1e-30


def test_softmax_matches_the_exact_distribution(oracle_lib, kats):
    s = kats["softmax"]
    logits = np.array(s["logits"], dtype=np.float32)
    p = oracle_lib.softmax(logits)
    exact = np.exp(logits.astype(np.float64) - logits.max())
    exact /= exact.sum()
    assert np.max(np.abs(p - exact)) < s["tolerance"]
    assert abs(float(np.sum(p, dtype=np.float32)) - 1.0) < s["tolerance"]


def test_half_to_f32_covers_every_class(oracle_lib):
    bits = np.arange(1 << 16, dtype=np.uint16)
    ours = np.array([oracle_lib.half_to_f32(int(b)) for b in bits[::97]], dtype=np.float32)
    numpy = bits[::97].view(np.float16).astype(np.float32)
    same = (ours == numpy) | (np.isnan(ours) & np.isnan(numpy))
    assert same.all()


def test_sinkhorn_is_doubly_stochastic(oracle_lib):
    rng = np.random.default_rng(3)
    x = oracle_lib.sinkhorn(rng.standard_normal(16).astype(np.float32), 4, 20)
    m = x.reshape(4, 4)
    assert np.allclose(m.sum(0), 1.0, atol=1e-5) and np.allclose(m.sum(1), 1.0, atol=1e-3)


def test_quantise_int8_rounds_half_to_even_and_clamps(oracle_lib):
    codes, scale = oracle_lib.quantise_int8(np.array([127.0, 0.5, 1.5, -2.5, -127.0], dtype=np.float32))
    assert scale == 1.0 and list(codes) == [127, 0, 2, -2, -127]
    codes, scale = oracle_lib.quantise_int8(np.zeros(8, dtype=np.float32))
    assert scale == 1.0 and not codes.any()
    fq = oracle_lib.fake_quantise_int8(np.array([1.0, -0.3, 0.0], dtype=np.float32))
    assert fq[0] == np.float32(1.0)


def test_zero_centred_norm_with_zero_gain_is_unit_rms(oracle_lib):
    x = np.random.default_rng(0).standard_normal(512).astype(np.float32)
    y = oracle_lib.zero_centred_norm(x, np.zeros(512, dtype=np.float32))
    assert abs(float(np.sqrt(np.mean(y.astype(np.float64) ** 2))) - 1.0) < 1e-5


def test_rotary_preserves_pair_norms(oracle_lib):
    x = np.random.default_rng(1).standard_normal(64).astype(np.float32)
    y = oracle_lib.rotary(x, 17)
    before = x[:32] ** 2 + x[32:] ** 2
    after = y[:32] ** 2 + y[32:] ** 2
    assert np.allclose(before, after, rtol=1e-5)
    assert np.array_equal(oracle_lib.rotary(x, 0), x)
