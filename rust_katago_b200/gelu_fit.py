"""Derive the GELU polynomial used by the kernels (kb_numeric.cuh: kb_gelu) and
restated by the CPU oracle (oracle/kb_oracle.c: or_gelu).

GELU(x) = x * Phi(x), Phi the standard normal CDF.  For |x| <= 4,
Phi(x) = 0.5 + x * P(t) with t = x^2, and P(t) = 0.5 * erf(sqrt(t/2)) / sqrt(t)
is approximated by a degree-10 polynomial in s = t/8 - 1 (s in [-1, 1]):
a least-squares Chebyshev fit on 40001 points, converted to the monomial
basis and rounded to float32.  The kernels evaluate P at s = min(x^2/8 - 1, 1)
and saturate Phi to [0, 1], so beyond |x| = 4 Phi reaches exactly 0 or 1
(|Phi - {0,1}| < 3.2e-5 there).  Max |GELU error| / max(1, |x|) < 3.2e-5,
far below the bf16/fp16 resolution of the stored activations.

Run: python -m rust_katago_b200.gelu_fit   (prints the coefficients as hex floats)
"""

import math

import numpy as np
from numpy.polynomial import chebyshev as C

DEGREE = 10
T_MAX = 16.0


def coefficients() -> list[float]:
    t = np.linspace(0.0, T_MAX, 40001)
    safe = np.where(t == 0, 1.0, t)
    erf = np.vectorize(math.erf)
    f = np.where(t == 0, 1.0 / math.sqrt(2.0 * math.pi), 0.5 * erf(np.sqrt(safe / 2.0)) / np.sqrt(safe))
    s = t / (T_MAX / 2.0) - 1.0
    c = C.chebfit(s, f, DEGREE)
    return [float(np.float32(v)) for v in C.cheb2poly(c)]


if __name__ == "__main__":
    for i, v in enumerate(coefficients()):
        print(f"c{i} = {v.hex()}  # {v!r}")
