"""Properties of the oracle's restated math (SLEEF expf, exp_u20, softmax helpers)."""
import numpy as np

import oracle


def _ulp_error(y, x):
    exact = np.exp(x.astype(np.float64))
    ok = (exact > 1.2e-38) & (exact < 3e38)
    ulp = np.spacing(np.abs(exact[ok]).astype(np.float32)).astype(np.float64)
    return np.abs(y.astype(np.float64)[ok] - exact[ok]) / ulp


def test_sleef_expf_within_published_one_ulp():
    # SLEEF xexpf is documented as 1.0-ULP accurate (src/sleef.rs:497-515).
    x = np.random.default_rng(1).uniform(-103, 88, 400_000).astype(np.float32)
    assert _ulp_error(oracle.sleef_expf(x), x).max() <= 1.0


def test_exp_u20_within_two_ulp_and_groups_fall_back():
    # exp_u20 (src/sleef.rs:1227-1256): about 2 ULP; a 4-lane group with any |x| > 87.3 uses
    # SLEEF expf for all four lanes.
    x = np.random.default_rng(2).uniform(-87, 87, 400_000).astype(np.float32)
    assert _ulp_error(oracle.exp_u20(x), x).max() <= 2.0
    g = np.array([0.5, -1.25, 2.0, -100.0], np.float32)
    assert oracle.exp_u20(g).tobytes() == oracle.sleef_expf(g).tobytes()
    assert oracle.sleef_expf(np.array([-104.5, 100.5], np.float32)).tolist() == [0.0, np.inf]


def test_softmax_lastdim_matches_numpy_and_backward_formula():
    rng = np.random.default_rng(3)
    x = rng.normal(size=(7, 13)).astype(np.float32) * 4
    y = oracle.softmax_lastdim(x)
    e = np.exp(x.astype(np.float64) - x.max(-1, keepdims=True))
    np.testing.assert_allclose(y, e / e.sum(-1, keepdims=True), rtol=2e-6, atol=2e-6)
    g = rng.normal(size=x.shape).astype(np.float32)
    d = oracle.softmax_backward_lastdim(g, y)
    ref = (g - (g * y).sum(-1, keepdims=True)) * y
    np.testing.assert_allclose(d, ref, rtol=1e-5, atol=1e-6)


def test_bmm_matches_numpy():
    rng = np.random.default_rng(4)
    a = rng.normal(size=(3, 9, 16)).astype(np.float32)
    b = rng.normal(size=(3, 16, 11)).astype(np.float32)
    np.testing.assert_allclose(oracle.bmm(a, b), a.astype(np.float64) @ b, rtol=1e-5, atol=1e-5)
    small_a, small_b = a[:, :2, :5], b[:, :5, :3]
    np.testing.assert_allclose(oracle.bmm(small_a, small_b), small_a.astype(np.float64) @ small_b,
                               rtol=1e-5, atol=1e-5)
