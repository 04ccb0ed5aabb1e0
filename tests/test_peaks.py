"""kernscope-bench: the roofline peak CLI (counterpart of the reference's
tools/bench/main.cpp).  CPU: usage and environment exit codes.  GPU: every
probe measures, the peaks clear the sanity floors and stay below the
hardware's nominal limits, and the JSONL db holds records with provenance."""

from __future__ import annotations

import json
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "kernscope_b200", "lib", "kernscope-bench")


def _run(*args, **kw):
    return subprocess.run([CLI, *args], capture_output=True, text=True, timeout=600, **kw)


def test_usage_and_version():
    r = _run("--version")
    assert r.returncode == 0 and "kernscope-bench" in r.stdout
    assert _run().returncode == 2
    assert _run("peak-nothing").returncode == 2
    assert _run("peak-bw", "--sizes", "0").returncode == 2


def test_no_device_is_an_environment_error():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    r = _run("peak-bw")
    assert r.returncode == 2 and "no CUDA device" in r.stderr


@pytest.mark.gpu
def test_peaks_measured_with_provenance(tmp_path, cuda_ok):
    db = tmp_path / "peaks.jsonl"
    r = _run("all", "--sizes", "64,1024", "--json", "--db", str(db))
    assert r.returncode == 0, r.stdout + r.stderr
    out = json.loads(r.stdout)
    p = out["peaks"]
    assert out["arch"] == "sm_100a" and out["floors_ok"]
    assert 3000 < p["hbm_gbs"] < 8000          # HBM3e, nominal 7.7-8 TB/s
    assert 500 < p["bf16_tflops"] < 2500       # dense bf16, nominal 2.25 PF
    assert 20 < p["fp32_tflops"] < 90
    assert p["smem_gbs"] > 10000
    fams = {m["family"] for m in out["measurements"]}
    assert fams == {"peak_bw_d2d", "peak_bw_read", "peak_flops_bf16", "peak_flops_fp32", "peak_smem"}
    # the 64 MiB size is L2-resident and excluded from the HBM peak
    small = [m for m in out["measurements"] if m["label"].endswith(" 64 MiB")]
    assert small and not any(m["hbm_resident"] for m in small)
    recs = [json.loads(ln) for ln in open(db)]
    assert len(recs) == len(out["measurements"])
    for rec in recs:
        assert rec["gpu_arch"] == "sm_100a" and rec["provenance"]["mode"] == "measured"
        assert rec["config"]["measured"] is True and rec["timings"]["median"] > 0
