"""CPU: the tuner's in-process correctness gate is the reference's gate.

The reference gate (tools/tune/src/driver_pipeline_impl.h:1223-1235, through
kernels/templates/tests/run_hip_gate.py:81-213) draws its inputs with
tests/golden/kernscope_golden/inputs.py:73-106, computes the expected output
with refs.py and judges with metrics.verdict.  The tuner's gate does all of
it in C++ (kernscope_b200/host/golden.cpp, families.cpp); these tests hold
that C++ against the fixtures the reference harness itself wrote
(tests/golden/*.npz) and against the oracle's restatement of metrics.py:

* inputs: the C++ generator (numpy's default_rng stream restated) gives
  the fixtures' inputs bit for bit at their shapes and seeds;
* reference: fed the fixtures' inputs, the C++ reference gives the fixtures'
  expected bf16 outputs bit for bit except where fp32 summation order
  differs (numpy's BLAS matmul and SIMD exp); those elements are counted,
  and each is within one bf16 ulp or, for an output near zero where the
  sum cancels, within 2^-16 of the output's rms;
* verdict: the C++ gate verdict gives metrics.verdict's cosine,
  max_rel_err and pcc and the same pass/fail on passing, borderline and
  failing outputs.
"""

from __future__ import annotations

import os

import ml_dtypes
import numpy as np
import pytest

from conftest import fixture_paths, load_fixture
from oracle import metrics as om

PATHS = fixture_paths()


@pytest.fixture(scope="module")
def tune():
    from kernscope_b200 import tune as t

    return t


def _key(fx):
    if fx["family"] == "attention":
        return "flash_attention:causal" if fx["causal"] else "flash_attention"
    return fx["family"]


def _bits(a):
    return np.asarray(a).view(np.uint16).ravel()


def _golden(tune, fx, **kw):
    return tune.query("golden", family=_key(fx), shape=[int(v) for v in fx["shape"]], seed=int(fx["seed"]), **kw)


def _fixture_inputs(fx, names):
    return {k: [int(v) for v in _bits(fx[k])] for k in names}


@pytest.mark.parametrize("path", PATHS, ids=[os.path.basename(p) for p in PATHS])
def test_gate_inputs_are_the_reference_inputs(tune, path):
    fx = load_fixture(path)
    r = _golden(tune, fx)
    assert set(r["inputs"]) == {k for k in fx if k not in ("expected", "shape", "seed", "causal", "family")}
    for name, bits in r["inputs"].items():
        np.testing.assert_array_equal(np.asarray(bits, dtype=np.uint16), _bits(fx[name]), err_msg=name)


MISMATCHES = {}


@pytest.mark.parametrize("path", PATHS, ids=[os.path.basename(p) for p in PATHS])
def test_gate_reference_matches_reference_outputs(tune, path):
    fx = load_fixture(path)
    names = [k for k in fx if k not in ("expected", "shape", "seed", "causal", "family")]
    r = _golden(tune, fx, inputs=_fixture_inputs(fx, names))
    got = np.asarray(r["expected"], dtype=np.uint16)
    exp = _bits(fx["expected"])
    assert got.shape == exp.shape
    diff = np.nonzero(got != exp)[0]
    MISMATCHES[os.path.basename(path)] = (len(diff), got.size)
    # bit-exact except where summation order differs: at most 0.05 % of the outputs
    assert len(diff) <= max(2, got.size // 2000), (len(diff), got.size)
    g = got.view(ml_dtypes.bfloat16).astype(np.float64)
    e = exp.view(ml_dtypes.bfloat16).astype(np.float64)
    rms = float(np.sqrt(np.mean(e * e)))
    for i in diff:
        one_ulp = abs(int(got[i].view(np.int16)) - int(exp[i].view(np.int16))) == 1
        near_zero = abs(g[i] - e[i]) <= 2.0 ** -16 * rms
        assert one_ulp or near_zero, (int(i), g[i], e[i], rms)
    # and the fixture's output passes the gate against the C++ reference
    v = _golden(tune, fx, inputs=_fixture_inputs(fx, names), verdict_got=[int(x) for x in exp])["verdict"]
    assert v["pass"], v


def test_gate_reference_mismatch_counts():
    """Summary of the previous test: the elements that differ are few, and
    only in families whose numpy reference uses BLAS or SIMD exp."""
    if len(MISMATCHES) < len(PATHS):
        pytest.skip("runs after the per-fixture comparison")
    total = sum(n for n, _ in MISMATCHES.values())
    elems = sum(m for _, m in MISMATCHES.values())
    print(f"\nC++ gate reference vs reference fixtures: {total} of {elems} bf16 outputs differ: "
          + ", ".join(f"{k} {n}" for k, (n, _) in sorted(MISMATCHES.items()) if n))
    assert total <= elems // 2000
    for name, (n, _) in MISMATCHES.items():
        if n:
            assert name.startswith(("softmax", "attention", "matmul")), name


def _verdict_cases(fx):
    exp = np.asarray(fx["expected"]).astype(np.float32)
    flip = exp.ravel().copy()
    flip[::2] = -flip[::2]
    return [("exact", exp), ("scaled 1.004", exp * np.float32(1.004)), ("scaled 1.02", exp * np.float32(1.02)),
            ("flipped", flip.reshape(exp.shape))]


@pytest.mark.parametrize("path", PATHS, ids=[os.path.basename(p) for p in PATHS])
def test_gate_verdict_is_the_reference_verdict(tune, path):
    fx = load_fixture(path)
    names = [k for k in fx if k not in ("expected", "shape", "seed", "causal", "family")]
    inputs = _fixture_inputs(fx, names)
    cpp_ref = np.asarray(_golden(tune, fx, inputs=inputs)["expected"], dtype=np.uint16).view(ml_dtypes.bfloat16)
    for label, out in _verdict_cases(fx):
        got_bits = np.asarray(out, dtype=np.float32).astype(ml_dtypes.bfloat16).view(np.uint16).ravel()
        got_vals = got_bits.view(ml_dtypes.bfloat16)
        v = _golden(tune, fx, inputs=inputs, verdict_got=[int(x) for x in got_bits])["verdict"]
        ref = om.verdict(got_vals, cpp_ref)  # metrics.py on the same pair
        assert v["pass"] == ref["pass"], (label, v, ref)
        assert abs(v["cosine"] - ref["cosine"]) <= 1e-5, label
        assert abs(v["pcc"] - ref["pcc"]) <= 1e-5, label
        assert abs(v["max_rel_err"] - ref["max_rel_err"]) <= 1e-6 * max(1.0, ref["max_rel_err"]), label
