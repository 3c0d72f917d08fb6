"""Derive the exp2 polynomial used by the prefill softmax (prefill_sm100.cuh, exp2_poly2).

Method (published, restated here): Cody & Waite range reduction (W. J. Cody, W. Waite,
"Software Manual for the Elementary Functions", 1980) writes 2^x = 2^n * 2^f with
n = round(x) and f = x - n in [-1/2, 1/2]; 2^f is approximated by a polynomial whose
coefficients minimise the maximum relative error (the minimax / Chebyshev criterion of
Remez's exchange algorithm). Here the minimax problem is solved directly as a linear
programme on a dense grid of f, with the constant term fixed to 1 so that 2^0 is exact.

The kernel evaluates the polynomial in FP32 with fused multiply-adds (Horner), then adds
n << 23 to the bit pattern. `python fit_exp2_poly.py` prints the coefficients as FP32 hex
literals and the relative error bound of the FP32 evaluation; the CPU test
tests/test_exp2_poly.py re-checks that bound against numpy's exp2.
"""
from __future__ import annotations

import numpy as np
from scipy.optimize import linprog

DEGREE = 3


def fit(degree: int = DEGREE, n_grid: int = 20001):
    f = np.linspace(-0.5, 0.5, n_grid)
    target = np.exp2(f)
    # variables: c1..c_deg, E ; minimise E subject to |1 + sum c_k f^k - 2^f| <= E * 2^f
    powers = np.stack([f ** k for k in range(1, degree + 1)], axis=1)
    a_ub = np.vstack([np.hstack([powers, -target[:, None]]),
                      np.hstack([-powers, -target[:, None]])])
    b_ub = np.concatenate([target - 1.0, 1.0 - target])
    cost = np.zeros(degree + 1)
    cost[-1] = 1.0
    res = linprog(cost, A_ub=a_ub, b_ub=b_ub, bounds=[(None, None)] * degree + [(0, None)],
                  method="highs")
    assert res.success, res.message
    return res.x[:degree].astype(np.float32)


def eval_fp32(coeffs: np.ndarray, x: np.ndarray) -> np.ndarray:
    """Mirror of the device evaluation: magic-number rounding, Horner in FP32, exponent add."""
    # Clamp at -127: then n = -127, f = 0, p = 1 and the exponent add gives exactly +0.0,
    # so masked scores (-inf) produce exact zeros.
    x = np.maximum(np.asarray(x, dtype=np.float32), np.float32(-127.0))
    magic = np.float32(12582912.0)  # 1.5 * 2^23: x + magic rounds x to an integer
    t = (x + magic).astype(np.float32)
    r = (t - magic).astype(np.float32)
    f = (x - r).astype(np.float32)
    p = np.float32(coeffs[-1])
    for c in coeffs[-2::-1]:
        p = (p.astype(np.float64) * f + c).astype(np.float32)  # one rounding per FMA
    p = (p.astype(np.float64) * f + 1.0).astype(np.float32)
    bits = p.view(np.uint32) + (t.view(np.uint32) << np.uint32(23))
    return bits.astype(np.uint32).view(np.float32)


def main():
    c = fit()
    x = np.linspace(-30.0, 8.0, 400001, dtype=np.float32)
    rel = np.abs(eval_fp32(c, x).astype(np.float64) / np.exp2(x.astype(np.float64)) - 1.0)
    for k, v in enumerate(c, start=1):
        print(f"c{k} = {v!r}  (0x{np.float32(v).view(np.uint32):08x})")
    print(f"max relative error of the FP32 evaluation on [-30, 8]: {rel.max():.3e}")


if __name__ == "__main__":
    main()
