"""The FMA-pipe exp2 of the CTA-pair prefill kernel's softmax (ex2_pair_fma in backburner_b200/csrc/pa_prefill.cuh),
restated step by step in float32 numpy: rint by the 1.5 * 2^23 addition, a degree-3 polynomial for 2^f on
[-0.5, 0.5], the exponent added as an integer. Pins the fitted coefficients' accuracy (P is rounded to f16 after it,
relative step 2^-11 = 4.9e-4) over the softmax's input range t = s * log2(e) - m <= 8 (the lazy-max threshold)."""
import numpy as np

C3, C2, C1, C0 = np.float32(0.0551716648), np.float32(0.2426111251), np.float32(0.6932609677), np.float32(0.9999280572)
BIG = np.float32(12582912.0)


def ex2_pair_fma(t):
    t = np.maximum(np.asarray(t, np.float32), np.float32(-125.0))
    tt = (t + BIG).astype(np.float32)
    r = (tt - BIG).astype(np.float32)
    f = (t - r).astype(np.float32)
    p = (C3 * f + C2).astype(np.float32)
    p = (p * f + C1).astype(np.float32)
    p = (p * f + C0).astype(np.float32)
    bits = (tt.view(np.uint32).astype(np.uint64) * 0x800000 + p.view(np.uint32).astype(np.uint64)) & 0xFFFFFFFF
    return bits.astype(np.uint32).view(np.float32)


def test_relative_error_over_the_softmax_range():
    t = np.linspace(-60.0, 8.0, 2_000_001, dtype=np.float32)
    got = ex2_pair_fma(t).astype(np.float64)
    ref = np.exp2(t.astype(np.float64))
    assert np.max(np.abs(got - ref) / ref) < 8e-5


def test_masked_and_tiny_inputs_round_to_zero_in_f16():
    got = ex2_pair_fma(np.array([-np.inf, -1e30, -200.0, -125.0], np.float32))
    assert np.all(got > 0) and np.all(got < 1e-37)
    assert np.all(got.astype(np.float16) == 0)


def test_integers_are_exact_powers_up_to_the_polynomial_constant():
    n = np.arange(-30, 9, dtype=np.float32)
    got = ex2_pair_fma(n)
    assert np.allclose(got, np.exp2(n) * C0, rtol=1e-7)
