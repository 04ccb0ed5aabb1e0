"""Fit the erfc approximation of the exact-erf GELU kernels (rowops.cu).

    python kernscope_b200/csrc/fit_gelu_erfc.py

Form (Press et al., Numerical Recipes, section 6.2, "erfcc": erfc written as
t * exp(-z^2 + P(t)) with t = 1 / (1 + a z)):

    erfc(z) = r * 2^((P(r) - z^2) * log2(e)),  r = 1 / (1 + A z),  z in [0, 4],

with this repository's own coefficients: P of degree 6 in r, fitted by least
squares to ln(erfc(z) / r) + z^2 on 40001 points of [0, 4] and reweighted
toward minimax (Lawson iterations); A = 0.55.  Relative error of erfc in
exact arithmetic: 3.2e-7.  The script prints the float32 coefficients as
they appear in rowops.cu and checks, in a float32 emulation of the kernel's
operation order (r and the power of two taken as correctly rounded, then
perturbed by one and two ulps), that the GELU of every bf16 input with
2^-9 <= |t| < 8 equals the reference formula bit for bit
(refs.py:59-63: x = fp32(t * fp32(1/sqrt 2)), e = fp32(erf(double x)),
bf16(fp32(0.5 t) * fp32(1 + e))).  z >= 4 needs no fit: there erfc < 2^-25,
so fp32(1 - erfc) is 1 as the reference's fp32(erf) is.
"""

from __future__ import annotations

import math

import numpy as np

A = 0.55
DEGREE = 6


def fit(a: float = A, degree: int = DEGREE, zmax: float = 4.0) -> np.ndarray:
    from scipy.special import erfc

    z = np.linspace(0.0, zmax, 40001)
    r = 1.0 / (1.0 + a * z)
    target = np.log(erfc(z) / r) + z * z
    w = np.ones_like(z)
    for _ in range(40):
        m = np.vander(r, degree + 1, increasing=True) * w[:, None]
        c, *_ = np.linalg.lstsq(m, target * w, rcond=None)
        err = np.polynomial.polynomial.polyval(r, c) - target
        w = w * np.abs(err) ** 0.5 + 1e-30
        w /= w.max()
    return c.astype(np.float32)


def _fma(a, b, c):
    return (a.astype(np.float64) * b + c).astype(np.float32)  # one rounding: f32 x f32 is exact in f64


def gelu_emulated(t: np.ndarray, c: np.ndarray, a: float = A, rcp_ulps: int = 0, ex2_ulps: int = 0) -> np.ndarray:
    """float32 emulation of the kernel's operation order."""
    f = np.float32
    x = (t * f(1.0 / math.sqrt(2.0))).astype(f)
    z = np.minimum(np.abs(x), f(4.0))
    r = (f(1.0) / _fma(np.full_like(z, a), z, f(1.0))).astype(f)
    for _ in range(abs(rcp_ulps)):
        r = np.nextafter(r, f(np.inf) if rcp_ulps > 0 else f(-np.inf)).astype(f)
    p = np.full_like(r, c[-1])
    for k in range(len(c) - 2, -1, -1):
        p = _fma(p, r, np.full_like(r, c[k]))
    e = np.exp2((_fma(-z, z, p) * f(1.4426950408889634)).astype(f)).astype(f)
    for _ in range(abs(ex2_ulps)):
        e = np.nextafter(e, f(np.inf) if ex2_ulps > 0 else f(-np.inf)).astype(f)
    w = (f(1.0) - (r * e).astype(f)).astype(f)
    s = np.where(x >= 0, (f(1.0) + w).astype(f), (f(1.0) - w).astype(f))
    return ((f(0.5) * t).astype(f) * s).astype(f)


def gelu_reference(t: np.ndarray) -> np.ndarray:
    f = np.float32
    x = (t * f(1.0 / math.sqrt(2.0))).astype(f)
    e = np.array([math.erf(float(v)) for v in x]).astype(f)
    return ((f(0.5) * t).astype(f) * (f(1.0) + e).astype(f)).astype(f)


def main() -> int:
    import ml_dtypes

    c = fit()
    print("A =", A, " coefficients c0..c6 (float32):")
    print(", ".join(f"{v:.9g}f" for v in c))
    mags = np.arange(0x3B00, 0x4100, dtype=np.uint32)
    codes = np.concatenate([mags, mags | 0x8000]).astype(np.uint16)
    t = codes.view(ml_dtypes.bfloat16).astype(np.float32)
    ref = gelu_reference(t).astype(ml_dtypes.bfloat16).view(np.uint16)
    worst = 0
    for ru in (0, 1, -1):
        for eu in (0, 2, -2):
            got = gelu_emulated(t, c, rcp_ulps=ru, ex2_ulps=eu).astype(ml_dtypes.bfloat16).view(np.uint16)
            worst = max(worst, int((got != ref).sum()))
    print(f"bf16 codes of the fitted range that differ from the reference (worst over ulp perturbations): {worst}")
    return 0 if worst == 0 else 1


if __name__ == "__main__":
    raise SystemExit(main())
