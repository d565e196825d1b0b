"""Fits the polynomial p(f) ~ 2^f on f in [-1/2, 1/2] used by the bulk scan's
FMA-pipe exponential (scan_bulk.cu, exp2_poly).

Method: Cody-Waite style reduction 2^x = 2^j * 2^f with j = rint(x), then a
minimax polynomial for 2^f, obtained here by the Remez exchange algorithm on
the relative error (float64).  The coefficients are rounded to FP32 and the
resulting FP32 Horner evaluation is checked on a dense grid.

    python saccade_v1_b200/csrc/gen_exp2_poly.py [degree]
"""
import sys

import numpy as np


def remez_rel(deg: int, lo=-0.5, hi=0.5, iters=40):
    # p(f) = sum_{k=0..deg} c_k f^k, minimise max |p(f)/2^f - 1| (Remez exchange).
    n = deg + 1  # unknown coefficients c_0..c_deg; plus the levelled error E
    m = n + 1    # reference points
    xs = 0.5 * (lo + hi) - 0.5 * (hi - lo) * np.cos(np.pi * np.arange(m) / (m - 1))
    grid = np.linspace(lo, hi, 400001)
    c = None
    for _ in range(iters):
        A = np.zeros((m, m))
        rhs = np.zeros(m)
        for i, x in enumerate(xs):
            t = 2.0 ** x
            A[i, :n] = [x ** k for k in range(n)]
            A[i, n] = (-1) ** i * t
            rhs[i] = t
        sol = np.linalg.solve(A, rhs)
        c = sol[:n]
        err = sum(c[k] * grid ** k for k in range(n)) / 2.0 ** grid - 1
        s = np.sign(err)
        idx = [0] + list(np.nonzero(np.diff(s))[0] + 1) + [len(grid)]
        ext = [grid[a + np.argmax(np.abs(err[a:b]))] for a, b in zip(idx[:-1], idx[1:]) if b > a]
        if len(ext) != m:
            break
        xs = np.array(ext)
    return c


def horner_f32(coef32, f):
    p = np.float32(coef32[-1])
    for c in coef32[-2::-1]:
        p = (p * f + np.float32(c)).astype(np.float32)
    return p


def main():
    deg = int(sys.argv[1]) if len(sys.argv) > 1 else 5
    c = remez_rel(deg)
    c32 = c.astype(np.float32)
    f = np.linspace(-0.5, 0.5, 1000001).astype(np.float32)
    rel = np.abs(horner_f32(c32, f).astype(np.float64) / 2.0 ** f.astype(np.float64) - 1)
    print(f"degree {deg}: max relative error of the FP32 evaluation {rel.max():.3e}")
    for k, v in enumerate(c32):
        print(f"  c{k} = {float(v)!r}f  // 0x{np.float32(v).view(np.uint32):08x}")


if __name__ == "__main__":
    main()
