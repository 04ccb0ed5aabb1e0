"""CPU: the exact-erf GELU of the bias_gelu kernels, checked on all bf16 codes.

The kernels (rowops.cu, gelu_erf) evaluate the reference GELU (refs.py:59-63:
x = fp32(t * fp32(1/sqrt 2)), e = fp32(erf(double x)), y = bf16(fp32(0.5 t)
* fp32(1 + e))) with an fp32 erfc of their own in place of the double erf
(coefficients fitted by kernscope_b200/csrc/fit_gelu_erfc.py), and y = 0.5 t
directly below |t| = 2^-9.  This checks, over all 65536 bf16 inputs, a float32
emulation of the kernel's operation order, with the coefficients read from
rowops.cu, against the reference: bit-identical for every finite input, also
with the approximate reciprocal and power of two off by one and two ulps.
The GPU tests run the kernels themselves on the same 65536 codes.
"""

from __future__ import annotations

import os
import re
import sys

import ml_dtypes
import numpy as np
import pytest

from oracle import refs as orf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "kernscope_b200", "csrc")
SMALL = 0x3B00  # bf16 bits of 2^-9


def _kernel_coefficients():
    src = open(os.path.join(CSRC, "rowops.cu")).read()
    a = float(re.search(r"kErfcA = ([-0-9.e]+)f", src).group(1))
    p = [float(re.search(rf"kErfcP{i} = ([-0-9.e]+)f", src).group(1)) for i in range(7)]
    return a, np.array(p, dtype=np.float32)


def _fit_module():
    sys.path.insert(0, CSRC)
    try:
        import fit_gelu_erfc
    finally:
        sys.path.pop(0)
    return fit_gelu_erfc


def _codes():
    bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    return bits, bits.view(ml_dtypes.bfloat16)


@pytest.mark.parametrize("rcp_ulps,ex2_ulps", [(0, 0), (1, 2), (1, -2), (-1, 2), (-1, -2)])
def test_emulated_kernel_equals_reference_on_every_finite_code(rcp_ulps, ex2_ulps):
    fit = _fit_module()
    a, c = _kernel_coefficients()
    bits, t = _codes()
    tf = t.astype(np.float32)
    finite = np.isfinite(tf)
    with np.errstate(invalid="ignore", over="ignore"):
        ref = orf.gelu_erf(t).view(np.uint16)
        y = fit.gelu_emulated(tf, c, a=a, rcp_ulps=rcp_ulps, ex2_ulps=ex2_ulps)
    small = (bits & 0x7FFF) < SMALL
    y = np.where(small, np.float32(0.5) * tf, y).astype(ml_dtypes.bfloat16).view(np.uint16)
    bad = finite & (y != ref)
    assert not bad.any(), [hex(int(b)) for b in bits[bad][:8]]


def test_fitted_form_relative_error():
    """The committed coefficients are the fit's, and erfc is within 4e-7
    relative on [0, 4] in exact arithmetic."""
    from scipy.special import erfc

    fit = _fit_module()
    a, c = _kernel_coefficients()
    assert a == fit.A and np.allclose(c, fit.fit(), rtol=1e-6, atol=1e-7)
    z = np.linspace(0.0, 4.0, 20001)
    r = 1.0 / (1.0 + a * z)
    approx = r * np.exp(np.polynomial.polynomial.polyval(r, c.astype(np.float64)) - z * z)
    assert np.max(np.abs(approx / erfc(z) - 1.0)) < 4e-7


def test_small_inputs_take_half_t():
    """Below 2^-9, |0.5 t e| is under half a bf16 ulp of 0.5 t: the reference
    returns bf16(0.5 t) (zeros and subnormals included)."""
    bits, t = _codes()
    small = (bits & 0x7FFF) < SMALL
    with np.errstate(invalid="ignore"):
        ref = orf.gelu_erf(t[small]).view(np.uint16)
    y = (np.float32(0.5) * t[small].astype(np.float32)).astype(ml_dtypes.bfloat16).view(np.uint16)
    assert np.array_equal(y, ref)


def test_large_inputs_closed_form():
    """From |t| = 8 up to the largest finite bf16, erf(x) rounds to 1 in fp32:
    the reference returns t for t > 0 and -0 for t < 0, the closed form the
    whole-code table (rowops.cu, gelu_erf_code) stores for those codes."""
    bits, t = _codes()
    mag = bits & 0x7FFF
    big = (mag >= 0x4100) & (mag < 0x7F80)
    ref = orf.gelu_erf(t[big]).view(np.uint16)
    want = np.where(bits[big] & 0x8000, np.uint16(0x8000), bits[big])
    assert np.array_equal(ref, want)


def test_code_table_routes_cover_every_code():
    """The table's three routes (0.5 t below 2^-9, the closed form from 8 up,
    the formula between and for inf/NaN) equal the reference on every code."""
    fit = _fit_module()
    a, c = _kernel_coefficients()
    bits, t = _codes()
    tf = t.astype(np.float32)
    mag = bits & 0x7FFF
    with np.errstate(invalid="ignore", over="ignore"):
        formula = fit.gelu_emulated(tf, c, a=a).astype(ml_dtypes.bfloat16).view(np.uint16)
        half = (np.float32(0.5) * tf).astype(ml_dtypes.bfloat16).view(np.uint16)
        ref = orf.gelu_erf(t).view(np.uint16)
    closed = np.where(bits & 0x8000, np.uint16(0x8000), bits)
    table = np.where(mag < SMALL, half, np.where((mag >= 0x4100) & (mag < 0x7F80), closed, formula))
    fref = ref.view(ml_dtypes.bfloat16).astype(np.float32)
    ftab = table.view(ml_dtypes.bfloat16).astype(np.float32)
    same = (table == ref) | (np.isnan(fref) & np.isnan(ftab))
    assert same.all(), [hex(int(b)) for b in bits[~same][:8]]
