"""The attention kernel's FMA-pipe 2^x (ex2_poly2, mako-image_b200/csrc/sm100.cuh): its constants are the
minimax-relative-error fit of tests/ex2_fit.py, and evaluated the kernel's way in fp32 they stay within the stated
7.5e-5 relative error (below bf16's 3.9e-3 rounding of P) over the exponents the softmax produces: x = s - m with
m the running row maximum, so x <= 8 (the lazy-rescaling threshold) and anything below -126 flushes to zero."""

import os

import numpy as np

from tests.ex2_fit import ex2_poly_f32, kernel_coefficients, remez_exp2

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _coeffs():
    with open(os.path.join(ROOT, "mako-image_b200", "csrc", "sm100.cuh")) as f:
        return kernel_coefficients(f.read())


def test_kernel_constants_are_the_minimax_fit():
    c, e = remez_exp2()
    k = _coeffs()
    assert len(k) == 4
    assert np.allclose(k, c[::-1], rtol=2e-5, atol=0), (k, c[::-1])
    assert e < 7.5e-5


def test_relative_error_over_the_softmax_range():
    x = np.concatenate([np.linspace(-126.0, 8.0, 2_000_001, dtype=np.float32),
                        np.float32(0.5) + np.arange(-126, 8, dtype=np.float32)])  # the rounding ties, too
    got = ex2_poly_f32(x, _coeffs()).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got / want - 1.0)
    normal = x >= -125.0  # results at 2^-126 and below lose the implicit bit (and are flushed by bf16 anyway)
    assert rel[normal].max() < 7.6e-5, rel[normal].max()


def test_flush_below_the_clamp():
    got = ex2_poly_f32(np.array([-127.5, -200.0, -1e30], np.float32), _coeffs())
    assert np.all(got >= 0) and np.all(got < 2.0 ** -125)
