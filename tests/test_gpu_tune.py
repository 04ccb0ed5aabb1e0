"""GPU: the live tuning pipeline (the reference's acceptance suite,
tools/tune/tests/tune_driver_test.cpp:71-176): every config pre-screened,
gated against the CPU reference and benchmarked; an injected wrong-result
variant fails the gate and is discarded; best == minimum measured median and
the db agrees; a second run with the same tunecache replays everything
without touching the GPU; --emit-repro builds and runs; --arch auto."""

from __future__ import annotations

import json
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

FAST = {"warmup_ms": 2.0, "rep_ms": 10.0}


@pytest.fixture(scope="module")
def tune(cuda_ok):
    from kernscope_b200 import tune as t

    return t


def _best_checks(ev):
    measured = [v for v in ev["variants"] if "timings" in v]
    assert measured
    # the driver's order: median, then p20, then p80, then enumeration index
    best = min(measured, key=lambda v: (v["timings"]["median"], v["timings"]["p20"], v["timings"]["p80"]))
    assert ev["best"]["config"] == best["config"]
    assert [v for v in ev["variants"] if v["best"]][0]["config"] == best["config"]
    return best


def test_softmax_pipeline_gate_injection_and_cache(tune, tmp_path):
    db, cache = str(tmp_path / "sm.jsonl"), str(tmp_path / "sm.cache.json")
    opts = dict(kernel_family="softmax", shape=[1024, 8192], arch="sm_100a", db=db, cache=cache, **FAST)
    rc, ev = tune.run(inject_gate_failure=2, **opts)
    assert rc == 0 and ev["status"] == "ok" and ev["live"]
    s = ev["summary"]
    assert s["variants_total"] == 24 and s["prescreen_rejected"] >= 1
    assert s["golden_gate_failed"] == 1  # exactly the injected variant
    failed = [v for v in ev["variants"] if v["status"] == "golden_gate_failed"]
    assert len(failed) == 1 and "golden gate failed" in failed[0]["reason"]
    assert s["benchmarked"] == s["variants_total"] - s["prescreen_rejected"] - 1
    best = _best_checks(ev)
    assert best["gate"]["pass"] and best["achieved_gbps"] > 1000
    # db: one record per fresh measurement, query_best agrees
    recs = [json.loads(ln) for ln in open(db)]
    assert len(recs) == s["benchmarked"]
    q = tune.query("db_roundtrip", path=str(tmp_path / "copy.jsonl"), records=recs,
                   query={"gpu_arch": "sm_100a", "kernel_family": "softmax", "shape_hash": ev["shape_hash"]})
    assert q["best"]["config"] == ev["best"]["config"]
    # second run: everything replayed from the tunecache, nothing launched
    rc2, ev2 = tune.run(**opts)
    assert rc2 == 0 and ev2["summary"]["cached"] == 24 and ev2["summary"]["compiled"] == 0
    assert ev2["best"]["config"] == ev["best"]["config"]


@pytest.mark.parametrize("family,shape,extra", [
    ("matmul", [512, 512, 512], {}),
    ("layernorm", [2048, 4096], {}),
    ("bias_gelu", [1024, 4096], {"gelu": "tanh"}),
    ("reduction", [1 << 24], {}),
    ("reduction", [4099, 512], {}),
    ("flash_attention", [1, 4, 512, 128], {"causal": True}),
    ("flash_attention", [1, 4, 512, 64], {"causal": True}),
    ("flash_attention", [96, 160, 32], {}),
])
def test_family_pipelines(tune, tmp_path, family, shape, extra):
    rc, ev = tune.run(kernel_family=family, shape=shape, arch="sm_100a", cache=str(tmp_path / "c.json"),
                      db=str(tmp_path / "d.jsonl"), **FAST, **extra)
    assert rc == 0, ev.get("message")
    assert ev["summary"]["golden_gate_failed"] == 0 and ev["summary"]["benchmarked"] >= 1
    best = _best_checks(ev)
    assert best["gate"]["pass"]


def test_cli_arch_auto_and_repro(tune, tmp_path):
    r = subprocess.run([tune.CLI, "--kernel", "matmul", "--shape", "256,256,256", "--arch", "auto", "--json",
                        "--emit-repro", str(tmp_path / "repro")], capture_output=True, text=True, cwd=tmp_path)
    assert r.returncode == 0, r.stderr
    ev = json.loads(r.stdout)
    assert ev["gpu_arch"] == "sm_100a" and ev["status"] == "ok"
    repo = os.path.dirname(os.path.dirname(os.path.dirname(tune.CLI)))  # <repo>/kernscope_b200/lib/kernscope-tune
    run = subprocess.run(["bash", str(tmp_path / "repro" / "run.sh")], capture_output=True, text=True,
                         env={**os.environ, "KERNSCOPE_B200_ROOT": repo})
    assert run.returncode == 0 and "ok" in run.stdout, run.stdout + run.stderr


def test_report_contract_matmul_512(tune, tmp_path):
    """The reference's numeric report contract (tools/tune/tests/check_report.py)
    on the --json evidence of a matmul 512^3 tune.  The config keys differ by
    design (the sm_100a space: tile_m, tile_n, tile_k, stages, acc_stages,
    group_m); every other clause is the reference's."""
    r = subprocess.run([tune.CLI, "--kernel", "matmul", "--shape", "512,512,512", "--arch", "sm_100a", "--json",
                        "--db", str(tmp_path / "d.jsonl"), "--cache", str(tmp_path / "c.json")],
                       capture_output=True, text=True, cwd=tmp_path)
    assert r.returncode == 0, r.stderr
    ev = json.loads(r.stdout)
    assert set(ev["best"]["config"]) == {"tile_m", "tile_n", "tile_k", "stages", "acc_stages", "group_m"}
    rl = ev["roofline"]
    assert rl["ok"] and 0.0 < rl["position"] <= 1.0 and rl["bound"] in ("compute", "memory", "latency")
    assert 0.0 < ev["occupancy"] <= 1.0 and ev["occupancy.limiter"]
    assert len(ev["variants"]) >= 20
    medians = [v["timings"]["median"] for v in ev["variants"] if "timings" in v]
    assert medians and medians == sorted(medians) and min(medians) > 0
    assert ev["speedup"] >= 1.0 and ev["baseline"]["timings"]["median"] > 0
    assert ev["schema_version"] == 1 and ev["gpu_arch"] == "sm_100a" and ev["grid_size"] == len(ev["variants"])
