"""The FMA-pipe exp2 used for part of the softmax (csrc/ifa4_ptx.cuh ``exp2_poly_pair``),
replayed step by step in numpy float32: round-to-integer with the 1.5*2^23 constant, the
degree-3 polynomial on [-1/2, 1/2], and the exponent-field add.  Checked against exp2."""
import numpy as np

C = np.array([0.9999280572, 0.6932609677, 0.2426111251, 0.0551716685], dtype=np.float32)


def exp2_poly(x):
    x = np.maximum(np.asarray(x, np.float32), np.float32(-125.0))
    r = np.float32(12582912.0)
    t = (x + r).astype(np.float32)
    f = (x - (t - r)).astype(np.float32)
    p = ((C[3] * f + C[2]) * f + C[1]) * f + C[0]
    bits = p.astype(np.float32).view(np.uint32) + (t.view(np.uint32) << np.uint32(23))
    return bits.view(np.float32)


def test_relative_error_below_bf16_half_ulp():
    x = np.linspace(-124.0, 8.0, 2_000_001, dtype=np.float32)
    y = exp2_poly(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(y / ref - 1.0)
    assert rel.max() < 1.0e-4  # bf16 half-ulp is 2^-9 = 1.95e-3


def test_integer_inputs_and_signs():
    x = np.arange(-124, 9, dtype=np.float32)
    np.testing.assert_allclose(exp2_poly(x), np.exp2(x), rtol=1e-4)
    assert np.all(exp2_poly(np.float32([-1e30, -np.inf])) < 1e-37)  # clamped, never negative


def test_minimax_polynomial_equioscillates():
    f = np.linspace(-0.5, 0.5, 200001)
    err = np.polyval(C[::-1].astype(np.float64), f) / np.exp2(f) - 1.0
    assert abs(err.max() + err.min()) < 1e-6  # balanced extrema (minimax)
    assert np.abs(err).max() < 7.6e-5
