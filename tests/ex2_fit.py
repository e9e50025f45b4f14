"""The fit behind the attention kernel's FMA-pipe 2^x (ex2_poly2 in mako-image_b200/csrc/sm100.cuh).

2^x = 2^n * 2^f with n = round(x) and f in [-1/2, 1/2]; 2^f is a degree-3 polynomial whose coefficients minimise
the maximum RELATIVE error on that interval (a minimax fit, found with the Remez exchange algorithm: alternate
between solving for the polynomial that equioscillates on a set of 5 reference points and moving the points to the
extrema of the resulting weighted error). Test infrastructure: run as a script it prints the coefficients; the
tests import `remez_exp2` and `ex2_poly_f32` to check the kernel's constants and their error bound."""

import re

import numpy as np


def remez_exp2(degree=3, lo=-0.5, hi=0.5, iters=30):
    """Coefficients c[0..degree] (constant first) of the minimax-relative-error polynomial for 2^f on [lo, hi], and
    the equioscillation error."""
    n = degree + 2
    k = np.arange(n)
    x = 0.5 * (lo + hi) + 0.5 * (hi - lo) * np.cos(np.pi * (n - 1 - k) / (n - 1))  # Chebyshev extrema
    grid = np.linspace(lo, hi, 200001)
    c, E = None, 0.0
    for _ in range(iters):
        # p(x_i) - 2^x_i = (-1)^i E 2^x_i  <=>  sum_j c_j x_i^j - (-1)^i E 2^x_i = 2^x_i
        A = np.zeros((n, n))
        for j in range(degree + 1):
            A[:, j] = x ** j
        A[:, degree + 1] = -((-1.0) ** k) * np.exp2(x)
        sol = np.linalg.solve(A, np.exp2(x))
        c, E = sol[:degree + 1], sol[degree + 1]
        err = np.polyval(c[::-1], grid) / np.exp2(grid) - 1.0
        # new reference: the extremum of each sign run of the error
        sign = np.sign(err)
        edges = np.flatnonzero(np.diff(sign)) + 1
        runs = np.split(np.arange(grid.size), edges)
        ext = [r[np.argmax(np.abs(err[r]))] for r in runs]
        if len(ext) < n:
            break
        while len(ext) > n:  # drop the smaller end extremum
            ext = ext[1:] if abs(err[ext[0]]) < abs(err[ext[-1]]) else ext[:-1]
        x = grid[ext]
    return c, abs(E)


def kernel_coefficients(source_text):
    """The four constants of ex2_poly2, highest degree first, as written in the kernel source."""
    body = source_text[source_text.index("ex2_poly2(float2 x)"):]
    body = body[:body.index("\n}\n")]
    vals = [float(v) for v in re.findall(r"make_float2\(([0-9.]+)f, \1f\)", body)]
    return vals[-4:]  # the polynomial's constants follow the rounding constants


def ex2_poly_f32(x, coeffs_high_first):
    """The kernel's evaluation in fp32: clamp at -126, n by the 1.5 * 2^23 rounding trick, f = x - n, Horner with
    fused multiply-adds (one rounding each, emulated in float64), 2^n added to the exponent bits."""
    f32 = np.float32
    x = np.maximum(np.asarray(x, f32), f32(-126.0))
    magic = f32(12582912.0)
    t = (x + magic).astype(f32)
    nn = (t - magic).astype(f32)
    f = (x - nn).astype(f32)
    c3, c2, c1, c0 = (f32(v) for v in coeffs_high_first)

    def fma(a, b, c):
        return (a.astype(np.float64) * b.astype(np.float64) + np.float64(c)).astype(f32)

    p = fma(np.full_like(f, c3), f, c2)
    p = fma(p, f, c1)
    p = fma(p, f, c0)
    bits = p.view(np.int32) + ((t.view(np.int32) - np.int32(0x4B400000)) << 23)
    return bits.view(f32)


if __name__ == "__main__":
    c, e = remez_exp2()
    print("coefficients (highest degree first):", ", ".join(f"{v!r}" for v in c[::-1]), "max rel error", e)
