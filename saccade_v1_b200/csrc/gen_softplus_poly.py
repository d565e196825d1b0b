"""Fits the polynomial of the scan kernels' softplus (scan_common.cuh, softplus_poly).

softplus(x) = max(x, 0) + log1p(e) with e = 2^(-|x| log2 e) in (0, 1], and
log1p(e) = e P(e) with P a polynomial of degree `deg` (default 5, the
kernels' choice: 8.5e-6 relative error; 6 gives 1.4e-6, 7 gives 3.3e-7).  P is the
minimax fit of the relative error of e P(e) against log1p(e) on (0, 1],
found by the Remez exchange algorithm in binary64 (log1p(e) / e is smooth
and tends to 1 as e -> 0, so the relative error is that of P against
log1p(e) / e).  The coefficients are then rounded to FP32, and the FP32
Horner evaluation (one fused multiply-add per step, emulated exactly in
binary64) is measured on a dense grid.

    python saccade_v1_b200/csrc/gen_softplus_poly.py [deg]

prints the coefficients from the highest degree down (the order of the
Horner steps in softplus_poly) and the measured maximum relative error.
"""
import sys

import numpy as np


def target(e):
    return np.log1p(e) / e


def remez(deg: int, lo=1e-12, hi=1.0, iters=60):
    """Minimax P (coefficients c_0..c_deg, low to high) of max |P(e) / target(e) - 1| on [lo, hi]."""
    n = deg + 1
    m = n + 1
    xs = 0.5 * (lo + hi) - 0.5 * (hi - lo) * np.cos(np.pi * np.arange(m) / (m - 1))
    grid = np.concatenate([np.geomspace(lo, 1e-3, 2000), np.linspace(1e-3, hi, 400001)])
    c = None
    for _ in range(iters):
        A = np.zeros((m, m))
        rhs = np.zeros(m)
        for i, x in enumerate(xs):
            t = target(x)
            A[i, :n] = [x ** k for k in range(n)]
            A[i, n] = (-1) ** i * t
            rhs[i] = t
        sol = np.linalg.solve(A, rhs)
        c = sol[:n]
        err = np.polyval(c[::-1], grid) / target(grid) - 1
        # New reference points: the extremum of each sign-alternating run.
        sign = np.sign(err)
        cuts = np.nonzero(np.diff(sign) != 0)[0] + 1
        runs = np.split(np.arange(grid.size), cuts)
        ext = [r[np.argmax(np.abs(err[r]))] for r in runs]
        if len(ext) < m:
            break
        # keep m alternating extrema with the largest |err|
        while len(ext) > m:
            drop = 0 if abs(err[ext[0]]) < abs(err[ext[-1]]) else len(ext) - 1
            ext.pop(drop)
        xs = grid[np.array(ext)]
    return c


def fma_f32(a, b, c):
    """FP32 fused multiply-add: the binary64 product of two FP32 values is exact; one rounding to FP32."""
    return np.float32(np.float64(a) * np.float64(b) + np.float64(c))


def horner_f32(coeffs_high_first, e):
    q = fma_f32(coeffs_high_first[0], e, coeffs_high_first[1])
    for k in coeffs_high_first[2:]:
        q = fma_f32(q, e, k)
    return q


def main() -> None:
    deg = int(sys.argv[1]) if len(sys.argv) > 1 else 5
    c = remez(deg)
    high = [np.float32(v) for v in c[::-1]]
    e = np.concatenate([np.geomspace(2.0 ** -40, 1e-3, 20000), np.linspace(1e-3, 1.0, 200001)]).astype(np.float32)
    e64 = e.astype(np.float64)
    q = horner_f32(high, e)
    got = np.float32(np.float64(e) * np.float64(q))  # e * P(e), one FP32 rounding (the FMA with max(x, 0) = 0)
    rel = np.abs(got.astype(np.float64) / np.log1p(e64) - 1)
    print("coefficients, highest degree first (FP32):")
    for v in high:
        print(f"  {float(v):.8e}f")
    print(f"max relative error of e*P(e) in FP32: {rel.max():.3e}")


if __name__ == "__main__":
    main()
