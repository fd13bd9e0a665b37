"""Derive the GELU polynomial used by the kernels (kb_numeric.cuh: kb_gelu) and
restated by the CPU oracle (oracle/kb_oracle.c: or_gelu).

GELU(x) = x * Phi(x), Phi the standard normal CDF.  For |x| <= 4,
Phi(x) = 0.5 + x * P(t) with t = x^2, and P(t) = 0.5 * erf(sqrt(t/2)) / sqrt(t)
is approximated by a degree-7 polynomial in t on [0, 16].  The error that
matters is that of GELU itself relative to max(1, |x|):
|x * x * (P - f)| / max(1, |x|) = w(t) |P - f| with w(t) = min(t, sqrt(t)),
so the fit is a weighted minimax one: Lawson's iteratively reweighted least
squares (C. L. Lawson, 1961) in the scaled variable s = t/8 - 1 (for the
conditioning of the solve), converted to monomials in t in float64 and
rounded to float32.  The kernels evaluate P at t = min(x^2, 16) by Horner's
rule and saturate Phi to [0, 1], so beyond |x| = 4 Phi reaches exactly 0 or 1
(|Phi - {0,1}| < 3.2e-5 there).  Max |GELU error| / max(1, |x|) < 3.2e-5
(the polynomial alone: 1.9e-5), far below the bf16/fp16 resolution of the
stored activations.

Run: python -m rust_katago_b200.gelu_fit   (prints the coefficients as hex
floats and the float32-evaluated error on a dense grid)
"""

import math

import numpy as np
from numpy.polynomial import polynomial as P

DEGREE = 7
T_MAX = 16.0
LAWSON_ITERS = 200


def _target(t: np.ndarray) -> np.ndarray:
    erf = np.vectorize(math.erf)
    safe = np.where(t == 0, 1.0, t)
    return np.where(t == 0, 1.0 / math.sqrt(2.0 * math.pi), 0.5 * erf(np.sqrt(safe / 2.0)) / np.sqrt(safe))


def coefficients() -> list[float]:
    """Float32 coefficients c0..c7 of P(t) = sum c_k t^k."""
    t = np.linspace(0.0, T_MAX, 20001)
    f = _target(t)
    w = np.minimum(t, np.sqrt(t))
    w[0] = 1e-3  # the error vanishes at t = 0 whatever P(0) is; keep the system regular
    s = t / (T_MAX / 2.0) - 1.0
    vand = np.vander(s, DEGREE + 1, increasing=True)
    lw = np.ones_like(t)
    best_err, best = math.inf, None
    for _ in range(LAWSON_ITERS):
        sw = np.sqrt(lw) * w
        c, *_ = np.linalg.lstsq(vand * sw[:, None], f * sw, rcond=None)
        e = np.abs(vand @ c - f) * w
        if e.max() < best_err:
            best_err, best = e.max(), c.copy()
        lw = lw * e
        lw /= lw.sum()
    # monomials in t: s = t * (2 / T_MAX) - 1, Horner on the polynomial in s
    pt = np.zeros(1)
    for k in range(DEGREE, -1, -1):
        pt = P.polyadd(P.polymul(pt, [-1.0, 2.0 / T_MAX]), [best[k]])
    return [float(np.float32(v)) for v in pt]


def gelu_f32(x: np.ndarray, c: list[float]) -> np.ndarray:
    """The kernels' evaluation in float32 (each fused multiply-add rounded once)."""
    xf = x.astype(np.float32)
    t = np.minimum(xf * xf, np.float32(T_MAX))
    p = np.float32(c[-1])
    for k in range(len(c) - 2, -1, -1):
        p = (np.float64(p) * np.float64(t) + np.float64(c[k])).astype(np.float32)
    phi = np.clip((np.float64(xf) * np.float64(p) + 0.5).astype(np.float32), 0.0, 1.0)
    return xf * phi


if __name__ == "__main__":
    coeffs = coefficients()
    for i, v in enumerate(coeffs):
        print(f"c{i} = {v.hex()}  # {v!r}")
    xs = np.linspace(-8.0, 8.0, 400001)
    exact = xs * 0.5 * (1.0 + np.vectorize(math.erf)(xs / math.sqrt(2.0)))
    err = np.abs(gelu_f32(xs, coeffs).astype(np.float64) - exact) / np.maximum(1.0, np.abs(xs))
    print(f"max |GELU error| / max(1, |x|) = {err.max():.3e}")
