"""Coefficients of poly_exp2_pair (fgw_common.cuh): 2^f on [-0.5, 0.5] by a degree-3 polynomial.

Lawson's iteratively reweighted least squares on the relative error p(f) / 2^f - 1 over a dense grid: each round
solves a weighted least-squares fit and multiplies every point's weight by its absolute error, which drives the
fit to the minimax (equal-ripple) solution. Prints the float32 coefficients, highest degree first, and the
largest relative error; the kernel header holds the printed values.

    python fgw_b200/csrc/fit_exp2_poly.py
"""
import numpy as np


def fit(degree=3, points=20001, rounds=200):
    f = np.linspace(-0.5, 0.5, points)
    target = np.exp2(f)
    basis = np.vander(f, degree + 1, increasing=True) / target[:, None]  # relative-error design
    weights = np.ones_like(f)
    for _ in range(rounds):
        root = np.sqrt(weights)
        coef, *_ = np.linalg.lstsq(basis * root[:, None], root, rcond=None)
        err = basis @ coef - 1.0
        weights = weights * np.abs(err)
        weights /= weights.sum()
    coef32 = coef.astype(np.float32)
    rel = np.abs(np.polyval(coef32[::-1].astype(np.float64), f) / target - 1.0).max()
    return coef32[::-1], rel


if __name__ == "__main__":
    c, rel = fit()
    print(" ".join(f"{x:.9g}f" for x in c), f"max relative error {rel:.3g}")
