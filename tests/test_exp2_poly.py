"""The kernel's FMA-pipe exp2 (exp2_poly_x2 in blackflash_b200/csrc/sm100_ptx.cuh).

Checks that the constants compiled into the kernel are the ones the fit script
(blackflash_b200/csrc/fit_exp2.py) produces, and emulates the device routine
bit for bit in numpy (fp32 rounding at each step, integer exponent add) to bound
its error over the argument range the softmax produces (x <= 8 after the lazy
rescale, arbitrarily negative otherwise)."""
import os
import re
import sys

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(REPO, "blackflash_b200", "csrc"))
import fit_exp2  # noqa: E402

HDR = os.path.join(REPO, "blackflash_b200", "csrc", "sm100_ptx.cuh")


def kernel_coeffs():
    text = open(HDR).read()
    return [float(re.search(rf"kExp2C{i} = ([0-9.eE+-]+)f;", text).group(1)) for i in range(4)]


def emulate(x: np.ndarray, c) -> np.ndarray:
    c = [np.float32(v) for v in c]
    x = np.maximum(x.astype(np.float32), np.float32(-126.0))
    magic = np.float32(12582912.0)
    t = (x + magic).astype(np.float32)
    n = (t - magic).astype(np.float32)
    f = (x - n).astype(np.float32)
    p = (f * c[3] + c[2]).astype(np.float32)
    p = (p * f + c[1]).astype(np.float32)
    p = (p * f + c[0]).astype(np.float32)
    bits = (p.view(np.uint32).astype(np.uint64) + (t.view(np.uint32).astype(np.uint64) << np.uint64(23))) & np.uint64(0xFFFFFFFF)
    return bits.astype(np.uint32).view(np.float32)


def test_kernel_constants_equal_fit():
    np.testing.assert_array_equal(np.array(kernel_coeffs(), np.float32), fit_exp2.fit())


def test_relative_error_bound_on_softmax_range():
    x = np.linspace(-60.0, 8.0, 400001).astype(np.float32)
    y = emulate(x, kernel_coeffs()).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(y / ref - 1)
    assert rel.max() < 1e-4  # far below bf16 rounding of P (2^-9)


def test_underflow_is_tiny_nonnegative_and_finite():
    x = np.array([-126.0, -127.0, -200.0, -1e30, -np.inf], np.float32)
    y = emulate(x, kernel_coeffs())
    assert np.all(np.isfinite(y)) and np.all(y >= 0) and np.all(y < 2.0 ** -125)
