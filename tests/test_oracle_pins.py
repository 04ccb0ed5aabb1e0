"""Pin the CPU oracle against golden vectors written by the reference itself.

Every ``tests/golden/*.npz`` was produced by the reference harness
(``tests/golden/make_fixtures.py``).  The oracle must regenerate the same
inputs and the same bf16 outputs bit for bit; the verdict restatement must
accept the golden output and reject a sign-flipped one, like the reference
tests (``tests/golden/test_golden.py:61-110``).
"""

from __future__ import annotations

import os

import ml_dtypes
import numpy as np
import pytest

from conftest import fixture_paths, load_fixture
from oracle import inputs as oin
from oracle import metrics as om
from oracle import refs as orf

PATHS = fixture_paths()


def _bits(a):
    return np.asarray(a).view(np.uint16)


@pytest.mark.parametrize("path", PATHS, ids=[os.path.basename(p) for p in PATHS])
def test_inputs_bit_identical(path):
    fx = load_fixture(path)
    inp = oin.generate_inputs(fx["family"], fx["shape"], seed=fx["seed"])
    for k, v in inp.items():
        assert v.dtype == ml_dtypes.bfloat16
        np.testing.assert_array_equal(_bits(v), _bits(fx[k]), err_msg=k)


@pytest.mark.parametrize("path", PATHS, ids=[os.path.basename(p) for p in PATHS])
def test_reference_output_bit_identical(path):
    fx = load_fixture(path)
    inp = {k: fx[k] for k in fx if k not in ("expected", "shape", "seed", "causal", "family")}
    out = oin.reference_output(fx["family"], inp, causal=fx["causal"])
    assert out.shape == oin.output_shape(fx["family"], fx["shape"])
    np.testing.assert_array_equal(_bits(out), _bits(fx["expected"]))


@pytest.mark.parametrize("path", PATHS, ids=[os.path.basename(p) for p in PATHS])
def test_verdict_accepts_golden_rejects_flipped(path):
    fx = load_fixture(path)
    exp = fx["expected"]
    assert om.verdict(exp, exp)["pass"]
    bad = np.asarray(exp).astype(np.float32).ravel().copy()
    bad[::2] = -bad[::2]
    v = om.verdict(bad.reshape(exp.shape), exp)
    if np.any(np.asarray(exp).astype(np.float32).ravel()[::2] != 0):
        assert not v["pass"]
    for key in ("cosine", "max_rel_err", "pcc"):
        assert key in v


def test_seed_determinism():
    a = oin.generate_inputs("matmul", (8, 8, 8), seed=1)
    b = oin.generate_inputs("matmul", (8, 8, 8), seed=1)
    c = oin.generate_inputs("matmul", (8, 8, 8), seed=2)
    np.testing.assert_array_equal(_bits(a["a"]), _bits(b["a"]))
    assert not np.array_equal(_bits(a["a"]), _bits(c["a"]))


def test_verdict_thresholds_inclusive():
    r = np.arange(1, 9, dtype=np.float32)
    a = r * np.float32(1.0 + 1e-2 - 1e-6)
    assert om.verdict(a, r)["pass"]
    a2 = r * np.float32(1.0 + 1.2e-2)
    assert not om.verdict(a2, r)["pass"]


def test_tanh_gelu_close_to_erf():
    t = np.linspace(-4, 4, 4097).astype(np.float32)
    d = np.abs(orf.gelu_tanh(t).astype(np.float64) - orf.gelu_erf(t).astype(np.float64))
    assert d.max() < 2e-2  # bf16 rounding of both plus the 4.7e-4 model gap


def test_baseline_rows_reproducible():
    full = oin.baseline_inputs("softmax", (3000, 64), seed=1)["x"]
    part = oin.baseline_inputs("softmax", (3000, 64), seed=1, row0=1500, nrows=700)["x"]
    np.testing.assert_array_equal(_bits(full[1500:2200]), _bits(part))
    fa = oin.baseline_inputs("attention", (1, 3, 16, 16, 8), seed=4)
    fb = oin.baseline_inputs("attention", (1, 3, 16, 16, 8), seed=4, row0=1, nrows=1)
    np.testing.assert_array_equal(_bits(fa["q"][1:2]), _bits(fb["q"]))
    u = oin.baseline_inputs("reduction_full", (5_000_000,), seed=2)["x"]
    v = oin.baseline_inputs("reduction_full", (5_000_000,), seed=2, row0=4_000_000, nrows=10)["x"]
    np.testing.assert_array_equal(u[4_000_000:4_000_010], v)
