"""Derive the polynomial used by the kernel's FMA-pipe exp2.

Method (Cody & Waite argument reduction + minimax polynomial, as in J.-M. Muller,
"Elementary Functions: Algorithms and Implementation", chapters 3 and 11):

    2^x = 2^j * 2^f,   j = round-to-nearest(x),   f = x - j in [-1/2, 1/2],

and 2^f is replaced by the degree-n polynomial p minimising the relative error
max |p(f) / 2^f - 1| on [-1/2, 1/2], found here with the Remez exchange algorithm
(equioscillation at n + 2 points).  The kernel evaluates p by Horner's rule with
packed fp32 FMAs and applies 2^j by adding j << 23 to the bit pattern of p(f).

P (the softmax numerator) is rounded to bf16 (relative step 2^-8) before the PV
product, so a relative error near 1e-4 is far below what the output can resolve.

``python exp2_poly.py`` prints the coefficients (c0..cn, low order first) and the
achieved relative error bound.
"""

from __future__ import annotations

import numpy as np

LO, HI = -0.5, 0.5


def _error(coeffs: np.ndarray, x: np.ndarray) -> np.ndarray:
    return np.polynomial.polynomial.polyval(x, coeffs) / np.exp2(x) - 1.0


def remez(degree: int, iterations: int = 60, grid: int = 200001) -> tuple[np.ndarray, float]:
    """Relative-error minimax coefficients (low order first) and the error bound."""
    n = degree
    k = np.arange(n + 2)
    nodes = 0.5 * (LO + HI) + 0.5 * (HI - LO) * np.cos(np.pi * (n + 1 - k) / (n + 1))
    dense = np.linspace(LO, HI, grid)
    coeffs = np.zeros(n + 1)
    for _ in range(iterations):
        # p(x_i) - 2^x_i = (-1)^i E 2^x_i  ->  sum_k c_k x_i^k - (-1)^i E 2^x_i = 2^x_i
        a = np.zeros((n + 2, n + 2))
        for i, x in enumerate(nodes):
            a[i, : n + 1] = x ** np.arange(n + 1)
            a[i, n + 1] = -((-1) ** i) * np.exp2(x)
        sol = np.linalg.solve(a, np.exp2(nodes))
        coeffs = sol[: n + 1]
        err = _error(coeffs, dense)
        # New reference: one extremum of |err| per sign-alternating run.
        sign = np.sign(err)
        runs = np.split(np.arange(dense.size), np.flatnonzero(np.diff(sign)) + 1)
        extrema = [run[np.argmax(np.abs(err[run]))] for run in runs if run.size]
        if len(extrema) < n + 2:
            break
        while len(extrema) > n + 2:  # drop the smallest end extremum
            if abs(err[extrema[0]]) < abs(err[extrema[-1]]):
                extrema.pop(0)
            else:
                extrema.pop()
        new_nodes = dense[np.array(extrema)]
        if np.allclose(new_nodes, nodes, atol=1e-12, rtol=0):
            break
        nodes = new_nodes
    bound = float(np.abs(_error(coeffs, dense)).max())
    return coeffs, bound


def float32_coefficients(degree: int = 3) -> tuple[list[float], float]:
    """Coefficients rounded to fp32 and the relative error bound of the fp32 set."""
    coeffs, _ = remez(degree)
    c32 = coeffs.astype(np.float32).astype(np.float64)
    x = np.linspace(LO, HI, 400001)
    return [float(c) for c in c32], float(np.abs(_error(c32, x)).max())


def main() -> int:
    for degree in (3, 4):
        coeffs, bound = float32_coefficients(degree)
        print(f"degree {degree}: relative error bound {bound:.3e}")
        for i, c in enumerate(coeffs):
            print(f"  c{i} = {np.float32(c).item()!r:>24}  ({np.float32(c).view(np.uint32):#010x})")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
