"""Derives the erfc coefficients of the 16-bit GELU kernel (xn_act.cu, kErfcF).

erfc(a) = exp(-a^2) * F(a) with F(a) = erfc(a) * exp(a^2), a smooth function
on [0, 4]. F is fitted as a polynomial of degree 7 in t = 1 / (1 + a / 2)
(t in [1/3, 1]) by least squares on relative error at 6000 Chebyshev nodes,
in float64, and the monomial coefficients in t are rounded to f32. Prints the
coefficients (constant term first) and the fit's relative error.

Run: python random-things_b200/csrc/fit_gelu_erfc.py
"""
import math

import numpy as np

P, DEG, TOP, NODES = 0.5, 7, 4.0, 6000


def main() -> None:
    f = lambda a: math.erfc(a) * math.exp(a * a)  # noqa: E731
    tlo, thi = 1 / (1 + P * TOP), 1.0
    k = np.arange(NODES)
    xs = np.cos(np.pi * (k + 0.5) / NODES)
    tv = tlo + (xs + 1) * (thi - tlo) / 2
    y = np.array([f((1 / t - 1) / P) for t in tv])
    w = 1 / np.abs(y)
    c, *_ = np.linalg.lstsq(np.vander(xs, DEG + 1, increasing=True) * w[:, None], y * w, rcond=None)
    poly_t = np.polynomial.Polynomial(c)(np.polynomial.Polynomial([-(tlo + thi) / (thi - tlo), 2 / (thi - tlo)]))
    coef = poly_t.coef.astype(np.float32)
    a = np.linspace(0.0, TOP, 40001)
    t = 1 / (1 + P * a)
    err = np.max(np.abs(np.polynomial.polynomial.polyval(t, coef.astype(np.float64)) / np.array([f(v) for v in a]) - 1))
    print(", ".join(f"{float(v).hex()}f" for v in coef))
    print(f"max relative error of the f32 coefficients: 2^{math.log2(err):.1f}")


if __name__ == "__main__":
    main()
