"""Derivation of the polynomial exp2 constants in sparse_q.cu.

The Sparse-Q epilogue computes part of its 2^y values on the FMA pipe:
y = j + f with j = rint(y) and |f| <= 1/2, 2^f from a polynomial, 2^j added
into the exponent field.  The polynomial is the one of least maximum RELATIVE
error |p(f) / 2^f - 1| on [-1/2, 1/2], found here by the Remez exchange
algorithm (equioscillation on deg + 2 reference points, re-chosen each round
at the extrema of the error curve).

    python exp2_poly_fit.py [degree]

prints the fp32 coefficients (c0 first) and the maximum relative error of the
fp32 Horner evaluation on a dense grid.  tests/test_exp2_poly.py checks that
the constants compiled into sparse_q.cu are this fit and meet its bound.
"""

from __future__ import annotations

import sys

import numpy as np

LO, HI = -0.5, 0.5


def remez(degree: int, iterations: int = 60) -> np.ndarray:
    """Coefficients (c0..c_degree, float64) of the minimax relative-error fit of 2^f."""
    n = degree + 2
    ref = (LO + HI) / 2 + (HI - LO) / 2 * np.cos(np.pi * np.arange(n)[::-1] / (n - 1))
    grid = np.linspace(LO, HI, 200_001)
    coeffs = np.zeros(degree + 1)
    for _ in range(iterations):
        # p(x_i) - 2^x_i = (-1)^i * E * 2^x_i on the reference points
        system = np.zeros((n, n))
        system[:, : degree + 1] = ref[:, None] ** np.arange(degree + 1)[None, :]
        system[:, degree + 1] = -((-1.0) ** np.arange(n)) * 2.0 ** ref
        solution = np.linalg.solve(system, 2.0 ** ref)
        coeffs = solution[: degree + 1]
        err = np.polyval(coeffs[::-1], grid) / 2.0 ** grid - 1.0
        # extrema of the error curve, merged into alternating signs
        turn = np.flatnonzero(np.diff(np.sign(np.diff(err))) != 0) + 1
        points = np.concatenate(([0], turn, [grid.size - 1]))
        xs, vs = [grid[points[0]]], [err[points[0]]]
        for i in points[1:]:
            if np.sign(err[i]) == np.sign(vs[-1]):
                if abs(err[i]) > abs(vs[-1]):
                    xs[-1], vs[-1] = grid[i], err[i]
            else:
                xs.append(grid[i])
                vs.append(err[i])
        while len(xs) > n:
            drop = 0 if abs(vs[0]) < abs(vs[-1]) else -1
            xs.pop(drop)
            vs.pop(drop)
        if len(xs) < n:
            break
        ref = np.array(xs)
    return coeffs


def fp32_max_relative_error(coeffs: np.ndarray, samples: int = 2_000_001) -> float:
    """Max |p(f)/2^f - 1| of the fp32 Horner evaluation the kernel performs (FMA per step)."""
    c = np.asarray(coeffs, dtype=np.float32)
    f = np.linspace(LO, HI, samples).astype(np.float32)
    acc = np.full_like(f, c[-1])
    for k in range(c.size - 2, -1, -1):
        # fp32 fma: exact product and sum, one rounding
        acc = (acc.astype(np.float64) * f.astype(np.float64) + np.float64(c[k])).astype(np.float32)
    return float(np.max(np.abs(acc.astype(np.float64) / np.exp2(f.astype(np.float64)) - 1.0)))


def main() -> None:
    degree = int(sys.argv[1]) if len(sys.argv) > 1 else 3
    coeffs = remez(degree).astype(np.float32)
    print("coefficients (c0 first):", ", ".join(repr(float(v)) for v in coeffs))
    print(f"max relative error (fp32 Horner): {fp32_max_relative_error(coeffs):.3e}")


if __name__ == "__main__":
    main()
