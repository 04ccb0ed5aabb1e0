"""The tuner pipeline end to end on the CPU, through a mock device runtime.

``tests/mock/mock_runtime.cpp`` is preloaded into a child process that runs
``kernscope_b200.tune.run``: the tuner's device calls then operate on host
memory, launches compute each family on the CPU (independently of the
tuner's own gate references), and events read a fake clock whose per-kernel
durations the test sets.  This covers, without a GPU, what the reference
covers with its MockRuntime and StubRuntime (libs/gpuruntime/include/
kernscope/gpu.h:257-330, libs/bench/tests/bench_test.cpp) and its driver
acceptance test (tools/tune/tests/tune_driver_test.cpp:71-228): selection of
the fastest config, the gate rejecting a wrong kernel, a launch failing in
the middle of the repetitions, the L2 flush before every timed launch, the
tunecache replay without launches, and a host without a device.
"""

from __future__ import annotations

import json
import os
import shutil
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MOCK_SRC = os.path.join(ROOT, "tests", "mock", "mock_runtime.cpp")
MOCK_SO = os.path.join(ROOT, "tests", "mock", "_build", "libks_mock_runtime.so")
REAL_LIB = os.path.join(ROOT, "kernscope_b200", "lib", "libkernscope_b200.so")
FLUSH_BYTES = 2 * (126 << 20)  # the bench's L2 flush: twice the L2 the mock reports

pytestmark = pytest.mark.skipif(not os.path.exists(REAL_LIB), reason="libkernscope_b200.so not built")


@pytest.fixture(scope="module")
def mock_so():
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    os.makedirs(os.path.dirname(MOCK_SO), exist_ok=True)
    subprocess.run(["g++", "-std=c++17", "-O2", "-shared", "-fPIC", "-Wall", "-Wextra", "-Werror",
                    "-I", os.path.join(ROOT, "include"), MOCK_SRC, "-o", MOCK_SO, "-ldl"], check=True)
    return MOCK_SO


def run_tune(mock, tmp_path, env=None, tag="run", **opts):
    """tune.run(**opts) in a child process with the mock preloaded; returns
    (exit code, evidence, op log)."""
    log = tmp_path / f"{tag}.ops.jsonl"
    e = dict(os.environ, PYTHONPATH=ROOT, LD_PRELOAD=mock, KS_MOCK_REAL_LIB=REAL_LIB, KS_MOCK_LOG=str(log))
    e.update(env or {})
    opts = dict(dict(warmup_ms=2, rep_ms=5), **opts)
    code = ("import json, sys\nfrom kernscope_b200 import tune\n"
            "rc, ev = tune.run(**json.loads(sys.argv[1]))\nprint(json.dumps({'rc': rc, 'ev': ev}))\n")
    p = subprocess.run([sys.executable, "-c", code, json.dumps(opts)], env=e, capture_output=True, text=True,
                       timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
    out = json.loads(p.stdout.strip().splitlines()[-1])
    ops = [json.loads(line) for line in log.read_text().splitlines()] if log.exists() else []
    return out["rc"], out["ev"], ops


def by_symbol(ev):
    return {v["symbol"]: v for v in ev["variants"]}


SOFTMAX = dict(kernel_family="softmax", shape=[64, 1024])
FAST = "kernscope_b200_softmax_b256_v8_onepass"


def test_picks_the_fastest_and_records_it(mock_so, tmp_path):
    db, cache = tmp_path / "db.jsonl", tmp_path / "cache.json"
    rc, ev, ops = run_tune(mock_so, tmp_path, env={"KS_MOCK_TIMES": f"{FAST}=0.25"}, db=str(db), cache=str(cache),
                           **SOFTMAX)
    assert rc == 0 and ev["status"] == "ok" and ev["live"] is True
    assert ev["best"]["symbol"] == FAST
    assert ev["best"]["timings"]["median"] == pytest.approx(0.25)
    medians = [v["timings"]["median"] for v in ev["variants"] if v["status"] == "benchmarked"]
    assert len(medians) == ev["summary"]["benchmarked"] >= 10 and min(medians) == pytest.approx(0.25)
    from kernscope_b200 import tune

    best = tune.query("db_load", path=str(db))["best"]
    assert len(best) == 1 and best[0]["config"] == ev["best"]["config"]
    assert any(o["op"] == "launch" and o["detail"] == FAST for o in ops)


def test_every_timed_launch_follows_an_l2_flush(mock_so, tmp_path):
    """bench.cpp's repetition: flush memset, event, launch, event."""
    rc, ev, ops = run_tune(mock_so, tmp_path, **SOFTMAX)
    assert rc == 0
    timed = 0
    for i in range(1, len(ops) - 2):
        if ops[i]["op"] == "event_record" and ops[i + 1]["op"] == "launch" and ops[i + 2]["op"] == "event_record":
            timed += 1
            assert ops[i - 1]["op"] == "memset" and ops[i - 1]["bytes"] == FLUSH_BYTES
    assert timed >= ev["summary"]["benchmarked"]
    flushes = [o for o in ops if o["op"] == "memset" and o["bytes"] == FLUSH_BYTES]
    assert len(flushes) == timed


def test_cache_replay_launches_nothing(mock_so, tmp_path):
    db, cache = tmp_path / "db.jsonl", tmp_path / "cache.json"
    env = {"KS_MOCK_TIMES": f"{FAST}=0.25"}
    rc1, ev1, _ = run_tune(mock_so, tmp_path, env=env, tag="first", db=str(db), cache=str(cache), **SOFTMAX)
    rc2, ev2, ops2 = run_tune(mock_so, tmp_path, env=env, tag="second", db=str(db), cache=str(cache), **SOFTMAX)
    assert rc1 == rc2 == 0
    assert ev2["summary"]["cached"] == ev2["summary"]["variants_total"]
    assert not [o for o in ops2 if o["op"] == "launch"]
    assert ev2["best"]["symbol"] == ev1["best"]["symbol"] == FAST


def test_gate_rejects_a_kernel_that_writes_zeros(mock_so, tmp_path):
    bad = "kernscope_b200_softmax_b128_v4_onepass"
    rc, ev, _ = run_tune(mock_so, tmp_path, env={"KS_MOCK_ZERO": bad}, **SOFTMAX)
    v = by_symbol(ev)
    assert rc == 0 and v[bad]["status"] == "golden_gate_failed"
    assert ev["summary"]["golden_gate_failed"] == 1
    assert all(x["status"] in ("benchmarked", "prescreen_rejected") for s, x in v.items() if s != bad)


def test_launch_failure_during_the_repetitions(mock_so, tmp_path):
    bad = "kernscope_b200_softmax_b512_v8_onepass"
    rc, ev, ops = run_tune(mock_so, tmp_path, env={"KS_MOCK_FAIL": f"{bad}:5"}, **SOFTMAX)
    v = by_symbol(ev)
    assert rc == 0 and v[bad]["status"] == "bench_failed", v[bad]
    assert ev["summary"]["bench_failed"] == 1
    assert sum(o["op"] == "launch" and o["detail"] == bad for o in ops) == 5  # gate + warm + calibration ...
    assert ev["best"]["symbol"] != bad


def test_no_device_runs_the_pre_screen_only(mock_so, tmp_path):
    rc, ev, ops = run_tune(mock_so, tmp_path, env={"KS_MOCK_DEVICES": "0"}, **SOFTMAX)
    assert ev["live"] is False
    assert not [o for o in ops if o["op"] in ("launch", "malloc")]
    assert all(v["status"] in ("compiled", "prescreen_rejected") for v in ev["variants"])


@pytest.mark.parametrize("family,shape", [
    ("matmul", [128, 128, 128]),
    ("flash_attention", [1, 2, 128, 128]),
    ("layernorm", [64, 1024]),
    ("bias_gelu", [64, 1024]),
    ("reduction", [256, 256]),
    ("reduction", [65536]),
])
def test_every_family_passes_its_gate_against_independent_cpu_math(mock_so, tmp_path, family, shape):
    """The mock computes each family with its own loops; the tuner's gate
    references and verdicts must accept every config."""
    rc, ev, _ = run_tune(mock_so, tmp_path, kernel_family=family, shape=shape)
    assert rc == 0 and ev["status"] == "ok"
    assert ev["summary"]["benchmarked"] >= 1 and ev["summary"]["golden_gate_failed"] == 0
    assert all(v["status"] in ("benchmarked", "prescreen_rejected") for v in ev["variants"])
