"""Fit the polynomial used by the kernel's FMA-pipe exp2 (exp2_poly_x2 in sm100_ptx.cuh).

Method: range reduction 2^x = 2^n * 2^f with n = rint(x), f = x - n in [-1/2, 1/2]
(the Cody-Waite split, with one term because n is exact in fp32), then a
degree-3 polynomial for 2^f that minimises the maximum relative error. The
minimax fit comes from Lawson's algorithm, an iteratively reweighted least
squares on a dense grid. Running this file prints the fp32 coefficients and the
realised error of fp32 Horner evaluation. The kernel's constants must equal
them (tests/test_exp2_poly.py checks).
"""
import numpy as np


def fit(deg: int = 3, lo: float = -0.5, hi: float = 0.5, iters: int = 200):
    x = np.linspace(lo, hi, 20001)
    y = np.exp2(x)
    w = np.ones_like(x)
    V = np.vander(x, deg + 1, increasing=True)
    for _ in range(iters):
        A = V / y[:, None] * np.sqrt(w)[:, None]
        c, *_ = np.linalg.lstsq(A, np.sqrt(w), rcond=None)
        err = np.abs(V @ c / y - 1)
        w = w * err
        w /= w.sum()
    return c.astype(np.float32)


def horner_f32(c: np.ndarray, f: np.ndarray) -> np.ndarray:
    p = np.full_like(f, c[-1], dtype=np.float32)
    for k in range(len(c) - 2, -1, -1):
        p = (p * f + c[k]).astype(np.float32)
    return p


if __name__ == "__main__":
    c = fit()
    f = np.linspace(-0.5, 0.5, 100001, dtype=np.float32)
    rel = np.abs(horner_f32(c, f).astype(np.float64) / np.exp2(f.astype(np.float64)) - 1).max()
    print("coefficients (c0..c3):", [float(v) for v in c], "max rel err %.3e" % rel)
