"""The reference generator's own kernels on the B200 (oracle/ref_gpu.py).

The reference tuner's auto-grid kernels, generated and compiled for sm_100a
by oracle/ref_tune/build_ref_kernels.py, run at the benchmark shapes through
the same launcher the benchmark's reference arm uses.  These tests check the
harness: every runnable family has at least one config that passes the
oracle gate, and the two families the reference cannot run at the benchmark
shapes report why (softmax: the kernel covers block*vec_width <= 4096 of the
8192 columns although its validator accepts the shape; attention: every
d = 128 config needs more static shared memory than CUDA's 48 KB, or is
rejected by the validator)."""

from __future__ import annotations

import pytest

ref_gpu = pytest.importorskip("oracle.ref_gpu")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(ref_gpu.index() is None, reason="reference kernels not built")]


@pytest.mark.parametrize("family", ["layernorm", "bias_gelu", "matmul"])
def test_reference_kernels_pass_the_gate(family):
    r = ref_gpu.run_family(family, reps=1)
    assert "value" in r, r
    assert r["value"] > 0 and r["configs_timed"] >= 1


def test_reference_softmax_cannot_cover_8192_columns():
    r = ref_gpu.run_family("softmax", reps=1)
    assert r.get("unavailable") == "no reference config passed the gate", r


def test_reference_attention_d128_does_not_build():
    r = ref_gpu.run_family("flash_attention", reps=1)
    assert "unavailable" in r and all(x.startswith(("nvcc:", "validator:")) for x in r["reasons"]), r
