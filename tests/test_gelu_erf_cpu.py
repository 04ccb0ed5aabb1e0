"""CPU: the closed-form rules of the exact-erf GELU kernels.

The kernels evaluate the reference GELU (refs.py:59-63: x = fp32(t *
fp32(1/sqrt 2)), e = fp32(erf(double x)), y = bf16(fp32(0.5 t) * fp32(1 +
e))) on every bf16 value t exactly: a table of the reference's outputs for
2^-9 <= |t| < 8, built on the device from double-precision erf, and two
closed forms outside it.  This checks, over all 65536 bf16 codes, that the
closed forms equal the reference and that each table entry's erf value lies
far enough from an fp32 rounding midpoint that any erf accurate to a few
double ulps gives the reference's e.
"""

from __future__ import annotations

import math

import ml_dtypes
import numpy as np

from oracle import refs as orf

TAB_LO, TAB_HI = 0x3B00, 0x4100  # bf16 bits of 2^-9 and 8


def _codes():
    bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    return bits, bits.view(ml_dtypes.bfloat16)


def _same_bits(a, b):
    fa = a.view(ml_dtypes.bfloat16).astype(np.float32)
    fb = b.view(ml_dtypes.bfloat16).astype(np.float32)
    return (a == b) | (np.isnan(fa) & np.isnan(fb))


def test_closed_forms_outside_the_table_equal_the_reference():
    bits, t = _codes()
    with np.errstate(invalid="ignore"):
        ref = orf.gelu_erf(t).view(np.uint16)
        tf = t.astype(np.float32)
        mag = bits & 0x7FFF
        small = mag < TAB_LO
        big = mag >= TAB_HI
        y_small = (np.float32(0.5) * tf).astype(ml_dtypes.bfloat16).view(np.uint16)
        y_big = np.where(tf > 0, tf, tf * np.float32(0.0)).astype(ml_dtypes.bfloat16).view(np.uint16)
    assert small.sum() + big.sum() + (TAB_HI - TAB_LO) * 2 == 1 << 16
    assert _same_bits(y_small[small], ref[small]).all()
    assert _same_bits(y_big[big], ref[big]).all()


def test_table_entries_are_robust_to_erf_rounding():
    mags = np.arange(TAB_LO, TAB_HI, dtype=np.uint32).astype(np.uint16)
    t = mags.view(ml_dtypes.bfloat16).astype(np.float32)
    x = t * np.float32(1.0 / math.sqrt(2.0))
    worst = np.inf
    for xi in x:
        e = math.erf(float(xi))
        f = np.float32(e)
        for nb in (np.nextafter(f, np.float32(np.inf)), np.nextafter(f, np.float32(-np.inf))):
            mid = (float(f) + float(nb)) / 2.0
            worst = min(worst, abs(e - mid) / (abs(e) * 2.0 ** -52))
    assert worst > 1000.0, worst  # double ulps between erf and the nearest fp32 midpoint


def test_one_erf_serves_both_signs():
    """e(-t) = -e(t): the table computes erf once per magnitude."""
    mags = np.arange(TAB_LO, TAB_HI, dtype=np.uint32).astype(np.uint16)
    pos = mags.view(ml_dtypes.bfloat16)
    neg = (mags | 0x8000).view(ml_dtypes.bfloat16)
    xp = pos.astype(np.float32) * np.float32(1.0 / math.sqrt(2.0))
    xn = neg.astype(np.float32) * np.float32(1.0 / math.sqrt(2.0))
    assert np.array_equal(xn, -xp)
    ep = np.array([np.float32(math.erf(float(v))) for v in xp])
    en = np.array([np.float32(math.erf(float(v))) for v in xn])
    assert np.array_equal(en, -ep)
