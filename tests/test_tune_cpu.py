"""CPU tests of the C++20 tuner host side (no GPU): keys, config spaces and
pre-screen, occupancy, roofline, db and tunecache persistence, CLI exit codes.
Mirrors the reference's no-gpu suites (tools/tune/tests/*_gen_test.cpp,
tune_driver_test.cpp:181-228, libs/{occupancy,roofline,db}/tests)."""

from __future__ import annotations

import json
import os
import subprocess

import pytest

tune = pytest.importorskip("kernscope_b200.tune")


def fnv1a64(s: str) -> str:
    h = 0xCBF29CE484222325
    for b in s.encode():
        h ^= b
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return f"fnv1a64:{h:016x}"


def test_shape_hash_and_cache_key():
    h = tune.query("shape_hash", family="matmul", shape=[512, 512, 512])
    assert h == fnv1a64("matmul:512,512,512")
    k = tune.query("cache_key", arch="sm_100a", family="matmul", shape_hash=h)
    assert k == f"sm_100a:matmul:{h}"


def test_matmul_space():
    auto = tune.query("enumerate", family="matmul", shape=[8192, 8192, 8192])
    assert len(auto) == 34 and all(v["valid"] for v in auto)
    assert sum(v["config"]["tile_m"] == 256 for v in auto) == 10  # 4 CTA pairs, 6 one-CTA 256-row tiles
    assert sum(v["config"].get("cta_group") == 1 for v in auto) == 6
    assert sum(v["config"]["group_m"] < 0 for v in auto) == 11  # N-band rasters
    full = tune.query("enumerate", family="matmul", shape=[8192, 8192, 8192], full=True)
    assert len(full) == 372
    bad = [v for v in full if not v["valid"]]
    # 5 and 6 stages of 128x256 tiles, and 4 stages of one-CTA 256x256 tiles, exceed 227 KB; two
    # accumulators of a one-CTA 256x256 tile exceed 512 TMEM columns
    assert len(bad) == 48
    assert all("stages" in v["reason"] or "TMEM" in v["reason"] for v in bad)


def test_rowop_spaces_and_rejections():
    sm = tune.query("enumerate", family="softmax", shape=[4096, 8192])
    assert len(sm) == 24
    rej = {v["symbol"]: v["reason"] for v in sm if not v["valid"]}
    assert "kernscope_b200_softmax_b128_v8_onepass" in rej and "registers" in rej["kernscope_b200_softmax_b128_v8_onepass"]
    assert len(tune.query("enumerate", family="softmax", shape=[4096, 8192], full=True)) == 64
    red = tune.query("enumerate", family="reduction", shape=[1 << 28])
    assert all(v["valid"] for v in red)
    fa = tune.query("enumerate", family="flash_attention", shape=[8, 32, 8192, 128], causal=True)
    assert len(fa) == 3 and all(v["valid"] and v["symbol"].endswith("_causal") for v in fa)
    assert {v["config"]["tile_m"] for v in fa} == {128, 256}
    v = tune.query("validate", family="softmax", shape=[4, 100], config={"block": 256, "vec_width": 8, "mode": "onepass"})
    assert not v["valid"] and "vec_width" in v["reason"]


def test_occupancy_model():
    # persistent GEMM: 192 threads, ~197 KB shared, 512 TMEM columns -> 1 CTA/SM
    o = tune.query("occupancy", regs=64, smem=197 * 1024, block=192, tmem=512)
    assert o["blocks_per_sm"] == 1
    o = tune.query("occupancy", regs=64, smem=0, block=256, tmem=0)
    assert o["blocks_per_sm"] == 4 and o["limiter"] == "registers" and abs(o["occupancy"] - 0.5) < 1e-12
    o = tune.query("occupancy", regs=32, smem=0, block=1024, tmem=0)
    assert o["blocks_per_sm"] == 2 and o["occupancy"] == 1.0
    o = tune.query("occupancy", regs=64, smem=0, block=128, tmem=256)
    assert o["blocks_per_sm"] == 2 and o["limiter"] == "tmem"
    assert tune.query("occupancy", regs=300, smem=0, block=128)["blocks_per_sm"] == 0


def test_roofline_model():
    g = tune.query("roofline", family="matmul", m=8192, n=8192, k=8192)
    assert g["flops"] == 2 * 8192 ** 3 and g["bound"] == "compute"
    fa = tune.query("roofline", family="flash_attention", m=256, n=8192, d=128, causal=True)
    assert fa["flops"] == 4 * 128 * 256 * 8192 * 8193 // 2
    sm = tune.query("roofline", family="softmax", n=4096 * 8192, k=8192)
    assert sm["bytes"] == 4096 * 8192 * 4 and sm["bound"] == "memory"
    bg = tune.query("roofline", family="bias_gelu", n=16384 * 16384, k=16384)
    assert bg["bytes"] == 16384 * 16384 * 4 + 16384 * 2
    assert bg["reference_model_bytes"] == 3 * 16384 * 16384 * 2
    p = tune.query("peaks")
    assert p["hbm_gbs"] > 1000 and p["bf16_tflops"] > 500


def test_db_roundtrip(tmp_path):
    rec = lambda med, cfg: {"schema_version": 1, "gpu_arch": "sm_100a", "kernel_family": "softmax",
                            "shape_hash": "fnv1a64:0", "config": cfg,
                            "timings": {"median": med, "p20": med * 0.9, "p80": med * 1.1},
                            "provenance": {"timestamp": "2026-12-01T00:00:00Z", "tool_version": "t", "mode": "measured"}}
    path = str(tmp_path / "db.jsonl")
    out = tune.query("db_roundtrip", path=path, records=[rec(0.03, {"block": 256}), rec(0.02, {"block": 128})],
                     query={"gpu_arch": "sm_100a", "kernel_family": "softmax", "shape_hash": "fnv1a64:0"})
    assert out["saved"] and len(out["records"]) == 2 and out["warnings"] == 0
    assert out["best"]["config"] == {"block": 128}
    lines = open(path).read().strip().splitlines()
    assert all(json.loads(ln)["schema_version"] == 1 for ln in lines)


def test_prescreen_only_run_and_cache_replay(tmp_path):
    """No GPU: the pipeline stops after the pre-screen (no_live_gpu when a live
    run is requested, ok with live_bench False) and writes the tunecache; a
    second run replays every config from the cache."""
    cache = str(tmp_path / "c.json")
    rc, ev = tune.run(kernel_family="softmax", shape=[4096, 8192], arch="sm_100a", live_bench=False, cache=cache,
                      db=str(tmp_path / "db.jsonl"))
    assert rc == 0 and ev["summary"]["variants_total"] == 24 and ev["summary"]["cached"] == 0
    assert ev["summary"]["compiled"] + ev["summary"]["prescreen_rejected"] == 24
    c = json.load(open(cache))
    assert c["schema_version"] == 1
    (key, entry), = c["entries"].items()
    assert key == f"sm_100a:softmax:{fnv1a64('softmax:4096,8192')}"
    assert entry["key"]["shape"] == [4096, 8192] and len(entry["configs"]) == 24
    rc2, ev2 = tune.run(kernel_family="softmax", shape=[4096, 8192], arch="sm_100a", live_bench=False, cache=cache)
    assert ev2["summary"]["cached"] == 24 and ev2["summary"]["compiled"] == 0
    # a different occupancy floor must not replay the cached outcomes
    rc3, ev3 = tune.run(kernel_family="softmax", shape=[4096, 8192], arch="sm_100a", live_bench=False, cache=cache,
                        min_occupancy=0.25)
    assert ev3["summary"]["cached"] == 0


def test_no_viable_config_at_full_occupancy(tmp_path):
    rc, ev = tune.run(kernel_family="matmul", shape=[512, 512, 512], arch="sm_100a", min_occupancy=1.0,
                      cache=str(tmp_path / "c.json"))
    assert rc == 1 and ev["status"] == "no_viable_config"
    assert ev["summary"]["compiled"] == 0 and ev["summary"]["prescreen_rejected"] == ev["summary"]["variants_total"]


def test_cli_exit_codes(tmp_path):
    def cli(*a):
        return subprocess.run([tune.CLI, *a], capture_output=True, text=True, cwd=tmp_path)
    assert cli("--kernel", "nope", "--shape", "1,2", "--arch", "sm_100a").returncode == 2
    assert cli("--kernel", "matmul", "--shape", "0,1,2", "--arch", "sm_100a").returncode == 2
    assert cli("--kernel", "matmul", "--shape", "64,64,64", "--arch", "sm_90").returncode == 2
    assert cli("--verify", "--kernel", "matmul", "--shape", "64,64,64").returncode == 2
    r = cli("--kernel", "layernorm", "--shape", "16384,4096", "--arch", "sm_100a", "--no-bench", "--json")
    assert r.returncode == 0
    ev = json.loads(r.stdout)
    # default db reports/tune/<family>-<hash>.jsonl, cache next to it
    assert ev["kernel_family"] == "layernorm" and ev["db"]["path"].startswith("reports/tune/layernorm-")
    assert os.path.exists(os.path.join(tmp_path, ev["cache"]["path"]))
    r = cli("--kernel", "matmul", "--shape", "512,512,512", "--arch", "sm_100a", "--min-occupancy", "1.0", "--text")
    assert r.returncode == 1 and "no viable config" in r.stdout
    assert cli("--version").returncode == 0


def test_reproducer_source_mentions_config():
    g = tune.query("geometry", family="matmul", shape=[8192, 8192, 8192],
                   config={"tile_m": 128, "tile_n": 256, "tile_k": 64, "stages": 4, "acc_stages": 2, "group_m": 8})
    assert g["grid_x"] == 148 and g["block_x"] == 192 and g["tmem_columns"] == 512
    assert "ks_matmul_launch" in g["source"] and "{128, 256, 64, 4, 2, 8, 0}" in g["source"]
    assert g["gate_shape"] == [64, 64, 64]


def test_exceptions_do_not_cross_the_c_abi():
    """A library exception (here get_arch's unknown-arch error) becomes an
    error status of the C entry point, not a terminated process."""
    with pytest.raises(ValueError, match="unknown arch"):
        tune.query("occupancy", arch="gfx9999", regs=32, smem=0, block=128)
    rc, ev = tune.run(kernel_family="softmax", shape=[64, 1024], arch="gfx9999", live_bench=False)
    assert rc == 2 and "unknown arch" in ev.get("message", "") + ev.get("error", "")
