"""The tuner's host logic pinned against the reference tuner itself (CPU).

``oracle/_ref/ref_tune_check`` is linked from the reference's own host
sources (``oracle/ref_tune/Makefile``) and answers the same questions as
``kernscope_b200.tune.query``: workload keys (tools/tune/src/driver.cpp
make_shape_hash / make_cache_key), the roofline model
(libs/roofline/src/roofline.cpp compute_flops / compute_bytes_moved), the
occupancy model (libs/occupancy/src/occupancy.cpp compute_occupancy), the
timing quantile (libs/bench/src/bench.cpp quantile) and the JSONL db reader
(libs/db/src/db.cpp Database::load / query_best). Every case here compares
the two answers. The module is skipped where the checker was not built
(it needs the reference checkout at build time).
"""

from __future__ import annotations

import glob
import json
import os
import re
import subprocess

import numpy as np
import pytest

tune = pytest.importorskip("kernscope_b200.tune")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CHECK = os.path.join(ROOT, "oracle", "_ref", "ref_tune_check")
pytestmark = pytest.mark.skipif(not os.access(CHECK, os.X_OK), reason="oracle/_ref/ref_tune_check not built")


def ref(*args) -> dict:
    out = subprocess.run([CHECK, *map(str, args)], capture_output=True, text=True, timeout=60, check=True)
    return json.loads(out.stdout)


SHAPES = [
    ("matmul", [512, 512, 512]),
    ("matmul", [8192, 8192, 8192]),
    ("matmul", [65536, 8192, 8192]),
    ("flash_attention", [8, 32, 8192, 128]),
    ("flash_attention", [1, 1, 256, 64]),
    ("softmax", [4096, 8192]),
    ("layernorm", [16384, 4096]),
    ("bias_gelu", [16384, 16384]),
    ("reduction", [268435456]),
    ("reduction", [256, 256]),
    ("softmax", [1]),
]


@pytest.mark.parametrize("family,shape", SHAPES)
@pytest.mark.parametrize("arch", ["sm_100a", "gfx1101"])
def test_keys_match_reference(family, shape, arch):
    r = ref("hash", family, ",".join(map(str, shape)), arch)
    h = tune.query("shape_hash", family=family, shape=shape)
    assert h == r["shape_hash"]
    assert tune.query("cache_key", arch=arch, family=family, shape_hash=h) == r["cache_key"]


ROOFLINE = [
    ("matmul", dict(m=8192, n=8192, k=8192)),
    ("matmul", dict(m=65536, n=8192, k=8192)),
    ("matmul", dict(m=1000, n=24, k=7)),
    ("softmax", dict(n=4096 * 8192)),
    ("layernorm", dict(n=16384 * 4096)),
    ("bias_gelu", dict(n=16384 * 16384)),
    ("reduction", dict(n=1 << 28)),
    ("flash_attention", dict(m=1, n=8192, d=128)),
    ("flash_attention", dict(m=1, n=300, d=64)),
    ("softmax", dict(n=0)),
]


@pytest.mark.parametrize("family,shape", ROOFLINE)
@pytest.mark.parametrize("dtype_bytes", [2, 4])
def test_roofline_model_matches_reference(family, shape, dtype_bytes):
    s = dict(m=0, n=0, k=0, d=0) | shape
    r = ref("roofline", family, s["m"], s["n"], s["k"], s["d"], dtype_bytes)
    ours = tune.query("roofline", family=family, dtype_bytes=dtype_bytes, **shape)
    assert ours["flops"] == r["flops"]
    assert ours["reference_model_bytes"] == r["bytes"]


def test_occupancy_matches_reference_on_sm_100():
    """Launchable (regs, smem, block) triples. One deliberate difference is
    left out: above 255 registers per thread the reference still computes a
    register-limited count, while this tuner reports 0 blocks (no such kernel
    can launch; test_occupancy_refuses_unlaunchable covers it)."""
    rng = np.random.default_rng(7)
    cases = [(64, 0, 128), (168, 100000, 384), (255, 0, 1024), (32, 232448, 128), (255, 0, 256), (16, 0, 32)]
    cases += [(int(rng.integers(8, 256)), int(rng.integers(0, 232448)), 32 * int(rng.integers(1, 33)))
              for _ in range(40)]
    for regs, smem, block in cases:
        r = ref("occupancy", "sm_100", regs, smem, block)
        ours = tune.query("occupancy", arch="sm_100", regs=regs, smem=smem, block=block)
        assert (ours["blocks_per_sm"], ours["warps_resident"], ours["limiter"]) == (
            r["blocks_per_sm"], r["warps_resident"], r["limiter"]), (regs, smem, block)
        assert ours["occupancy"] == pytest.approx(r["occupancy"], abs=1e-12)


def test_occupancy_refuses_unlaunchable():
    assert ref("occupancy", "sm_100", 300, 0, 128)["blocks_per_sm"] == 1
    assert tune.query("occupancy", arch="sm_100", regs=300, smem=0, block=128)["blocks_per_sm"] == 0


def test_quantile_matches_reference():
    rng = np.random.default_rng(3)
    for n in (1, 2, 3, 5, 10, 100, 101):
        s = [round(float(x), 6) for x in rng.random(n)]
        for q in (0.0, 0.2, 0.5, 0.8, 1.0):
            r = ref("quantile", q, ",".join(map(str, s)))["q"]
            assert tune.query("quantile", q=q, samples=s)["q"] == pytest.approx(r, rel=1e-15, abs=1e-15)


DBS = sorted(glob.glob(os.path.join(ROOT, "reports", "tune", "*.jsonl")) +
             glob.glob(os.path.join(ROOT, "reports", "peaks", "*.jsonl")))


@pytest.mark.parametrize("path", DBS, ids=os.path.basename)
def test_reference_reads_our_db(path):
    """Our committed tune and peak records load cleanly in the reference's db
    reader, and both readers pick the same best config per workload."""
    r = ref("db", path)
    ours = tune.query("db_load", path=path)
    assert r["opened"] and not r["warnings"]
    assert ours["records"] == r["records"] > 0
    assert not ours["warnings"]
    assert len(ours["best"]) == len(r["best"])
    for a, b in zip(ours["best"], r["best"]):
        assert {k: a[k] for k in ("gpu_arch", "kernel_family", "shape_hash", "config")} == \
               {k: b[k] for k in ("gpu_arch", "kernel_family", "shape_hash", "config")}
        assert a["median"] == pytest.approx(b["median"], rel=1e-12)


def test_db_reader_skips_the_same_lines(tmp_path):
    """Blank, CRLF, malformed, non-object, future- and fractional-schema,
    incomplete and bad-provenance lines, a config repeated with its members
    reordered, and a tie on the median: both readers keep the same records,
    pick the same best and warn on the same line numbers."""
    good = dict(schema_version=1, gpu_arch="sm_100a", kernel_family="softmax", shape_hash="fnv1a64:0",
                config=dict(block=256, vec_width=8), timings=dict(median=0.5, p20=0.4, p80=0.6),
                provenance=dict(timestamp="2026-01-01T00:00:00Z", tool_version="t", mode="measured"))
    faster = good | dict(config=dict(block=128, vec_width=8), timings=dict(median=0.25, p20=0.2, p80=0.3))
    replaced = good | dict(timings=dict(median=0.1, p20=0.1, p80=0.1))
    # same config as `faster` with its members in the other order: replaces it
    permuted = json.dumps(good | dict(timings=dict(median=0.3, p20=0.3, p80=0.3))).replace(
        '"block": 256, "vec_width": 8', '"vec_width": 8, "block": 128')
    tie = good | dict(config=dict(block=64, vec_width=8), timings=dict(median=0.1, p20=0.1, p80=0.1))
    bad_mode = good | dict(provenance=dict(timestamp="t", tool_version="t", mode="guessed"))
    lines = [json.dumps(good), "", "{not json", json.dumps(good | dict(schema_version=99)), json.dumps(faster),
             json.dumps(replaced), '{"schema_version": 1, "gpu_arch": "sm_100a"}', permuted + "\r",
             json.dumps(tie), json.dumps(bad_mode), json.dumps(good | dict(schema_version=1.5)), "[1, 2]",
             json.dumps(good | dict(shape_hash="fnv1a64:1", schema_version=0))]
    p = tmp_path / "mixed.jsonl"
    p.write_text("\n".join(lines) + "\n")
    r = ref("db", p)
    ours = tune.query("db_load", path=str(p))
    assert ours["records"] == r["records"]
    line_no = lambda msgs: sorted(int(re.search(r"line (\d+)", m).group(1)) for m in msgs)  # noqa: E731
    assert line_no(ours["warnings"]) == line_no(r["warnings"])
    assert [(b["config"], b["median"]) for b in ours["best"]] == [(b["config"], b["median"]) for b in r["best"]]
    assert len(r["warnings"]) == 6 and r["records"] == 4
