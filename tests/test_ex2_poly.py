"""CPU check of the FMA-pipe exp2 used by the softmax kernels (csrc/common.cuh
ex2_poly), restated step for step in numpy float32: the magic-number rounding,
the degree-3 polynomial and the exponent-field insertion."""

import numpy as np


def ex2_poly(x: np.ndarray) -> np.ndarray:
    x = np.maximum(x.astype(np.float32), np.float32(-126.0))
    magic = np.float32(12582912.0)
    t = (x + magic).astype(np.float32)
    j = (t - magic).astype(np.float32)
    f = (x - j).astype(np.float32)
    p = np.float32(0.0551716573536396) * f + np.float32(0.2426111400127411)
    p = (p.astype(np.float32) * f + np.float32(0.6932609677314758)).astype(np.float32)
    p = (p * f + np.float32(0.9999280571937561)).astype(np.float32)
    bits = p.view(np.int32) + (t.view(np.int32) << 23)
    return bits.astype(np.int32).view(np.float32)


def test_relative_error_over_softmax_range():
    # arguments seen by the softmax: (-inf, 8] (lazy rescaling allows up to 2^8)
    x = np.linspace(-100.0, 8.0, 2_000_001, dtype=np.float32)
    got = ex2_poly(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(got / ref - 1.0)
    assert rel.max() < 1e-4, rel.max()


def test_masked_and_tiny_arguments_vanish():
    x = np.array([-np.inf, -1e30, -200.0, -126.0], dtype=np.float32)
    got = ex2_poly(x)
    assert np.all(np.isfinite(got))
    assert np.all(got <= np.float32(2.0 ** -125))
    # they round to exactly zero in the fp16 P operand
    assert np.all(got.astype(np.float16) == 0)


def test_integer_arguments_are_exact_powers():
    x = np.arange(-60, 9, dtype=np.float32)
    got = ex2_poly(x).astype(np.float64)
    assert np.all(np.abs(got / np.exp2(x.astype(np.float64)) - 1) < 1e-4)
