"""The GELU forms of the single-pass two-SM GEMM epilogue (gemm_epi.cuh
gelu_erf_fast / gelu_tanh_fast), restated in numpy f32 and checked against the
exact functions the reference uses (libffwd/cuda.cu bias_gelu 2616-2708: erf
GELU, and the tanh form of gelu_new).  CPU only: the device code computes the
same expressions with ex2.approx and a fast divide (relative errors near 2^-22),
which the GPU parity tests cover end to end."""

import math

import numpy as np

# -2 log2(e) q(x), q the odd quintic with sigmoid(q(x)) ~ 0.5 (1 + erf(x / sqrt 2))
C1, C3, C5 = -2.3017271, -0.10617733, 9.1122725e-4
T1, T3 = -2.3022082, -0.1029432  # -2 log2(e) sqrt(2/pi) and x 0.044715


def gelu_erf_fast(x):
    x = x.astype(np.float32)
    c = np.clip(x, np.float32(-8.5), np.float32(8.5))
    c2 = c * c
    e = c * ((np.float32(C5) * c2 + np.float32(C3)) * c2 + np.float32(C1))
    return x / (np.float32(1) + np.exp2(e.astype(np.float64)).astype(np.float32))


def gelu_tanh_fast(x):
    x = x.astype(np.float32)
    e = x * (np.float32(T3) * x * x + np.float32(T1))
    return x / (np.float32(1) + np.exp2(e.astype(np.float64)).astype(np.float32))


def gelu_erf(x):
    x = x.astype(np.float64)
    return 0.5 * x * (1.0 + np.vectorize(math.erf)(x / math.sqrt(2.0)))


def gelu_tanh(x):
    x = x.astype(np.float64)
    return 0.5 * x * (1.0 + np.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x ** 3)))


def test_erf_form_error_bound():
    x = np.linspace(-20.0, 20.0, 400001)
    err = np.abs(gelu_erf_fast(x) - gelu_erf(x))
    assert err.max() <= 6e-5
    # far below the rounding of the 16-bit outputs it feeds (2^-9 relative)
    big = x > 1.0  # (the negative tail is checked by the absolute bound: GELU -> 0 there)
    assert (err[big] / np.abs(gelu_erf(x[big]))).max() <= 2.0 ** -9
    assert np.isfinite(gelu_erf_fast(np.array([-1e30, -100.0, 0.0, 100.0, 1e30]))).all()


def test_tanh_form_matches():
    x = np.linspace(-20.0, 20.0, 400001)
    assert np.abs(gelu_tanh_fast(x) - gelu_tanh(x)).max() <= 2e-6


def test_constants():
    l2e = 1.0 / math.log(2.0)
    assert abs(T1 - (-2.0 * l2e * math.sqrt(2.0 / math.pi))) < 1e-6
    assert abs(T3 - T1 * 0.044715) < 1e-6
