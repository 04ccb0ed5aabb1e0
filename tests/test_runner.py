"""ks-template-runner: the reference's gate flow (kernels/templates/tests/
run_hip_gate.py: golden inputs -> raw .bin buffers -> runner -> golden check)
with this library's runner and the committed golden fixtures.  CPU: usage and
environment exit codes.  GPU: every fixture through the runner, checked with
the reference verdict (tensor-core attention: the attention tolerance)."""

from __future__ import annotations

import os
import subprocess

import numpy as np
import pytest

from _util import assert_attention_close, assert_bf16_close
from conftest import fixture_paths, load_fixture

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
RUNNER = os.path.join(ROOT, "kernscope_b200", "lib", "ks-template-runner")

# per family: input arrays in the kernel's argument order, and the scalars
ARGS = {
    "softmax": (("x",), lambda s: [s[0], s[1]]),
    "layernorm": (("x", "gamma", "beta"), lambda s: [s[0], s[1]]),
    "bias_gelu": (("x", "bias"), lambda s: [s[0] * s[1], s[1]]),
    "reduction": (("x",), lambda s: [s[0], s[1]]),
    "matmul": (("a", "b"), lambda s: [s[0], s[1], s[2]]),
    "attention": (("q", "k", "v"), lambda s: [s[0], s[1], s[2]]),
}


def _run(*args):
    return subprocess.run([RUNNER, *map(str, args)], capture_output=True, text=True, timeout=300)


def test_usage_errors():
    assert _run().returncode == 2
    assert _run("--family", "softmax", "--out", "/tmp/x", "--out-size", "16", "--int", "2").returncode == 2
    # no --family and a symbol that names none
    r = _run("--hsaco", "k.hsaco", "--kernel", "kernscope_tune_softmax", "--out", "/tmp/x", "--out-size", "16")
    assert r.returncode == 2 and "--family" in r.stderr
    r = _run("--family", "softmax", "--kernel", "not_a_symbol", "--out", "/tmp/x", "--out-size", "64",
             "--int", "4", "--int", "8")
    assert r.returncode == 2 and "unknown kernel symbol" in r.stderr


def test_no_device_fails_loudly(tmp_path):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    x = tmp_path / "x.bin"
    x.write_bytes(b"\0" * 64)
    r = _run("--family", "softmax", "--in", x, "--out", tmp_path / "o.bin", "--out-size", "64", "--int", "4",
             "--int", "8")
    assert r.returncode == 1 and "no CUDA device" in r.stderr


def test_reference_gate_argv_reaches_the_device(tmp_path):
    """The argument list the reference's gate script builds
    (kernels/templates/tests/run_hip_gate.py: --hsaco, --kernel, --grid,
    --block, --in..., --out, --out-size, --int...) is accepted as it is: the
    family comes from the symbol and --hsaco is ignored.  Without a GPU the
    run gets as far as the device check."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present (the GPU test runs the kernel)")
    x = tmp_path / "x.bin"
    x.write_bytes(b"\0" * 64)
    r = _run("--hsaco", tmp_path / "unused.hsaco", "--kernel", "kernscope_b200_softmax_b256_v8_onepass", "--grid",
             "4", "--block", "256", "--in", x, "--out", tmp_path / "o.bin", "--out-size", "64", "--int", "4",
             "--int", "8")
    assert r.returncode == 1 and "no CUDA device" in r.stderr


def _family(fx):
    return fx["family"]


@pytest.mark.gpu
@pytest.mark.parametrize("path", fixture_paths(), ids=os.path.basename)
def test_gate_flow_through_runner(cuda_ok, tmp_path, path):
    from oracle import refs as orf

    fx = load_fixture(path)
    fam = _family(fx)
    names, ints = ARGS[fam]
    shape = fx["shape"]
    ins = []
    for n in names:
        p = tmp_path / f"{n}.bin"
        p.write_bytes(np.ascontiguousarray(fx[n]).tobytes())
        ins += ["--in", p]
    out = tmp_path / "out.bin"
    exp = fx["expected"]
    extra = ["--causal"] if fx["causal"] else []
    if fam == "bias_gelu":
        extra += ["--gelu", "erf"]  # the reference's exact-erf GELU
    r = _run("--family", fam, *ins, "--out", out, "--out-size", exp.nbytes,
             *sum((["--int", v] for v in ints(shape)), []), *extra, "--grid", "1", "--block", "1")
    assert r.returncode == 0, r.stdout + r.stderr
    got = np.frombuffer(out.read_bytes(), dtype=exp.dtype).reshape(exp.shape)
    if fam == "attention" and shape[2] == 128:
        rho = orf.attention_abs_weight(fx["q"], fx["k"], fx["v"], causal=fx["causal"])
        assert_attention_close(got, exp, rho)
    else:
        assert_bf16_close(got, exp, gate=True)


@pytest.mark.gpu
@pytest.mark.parametrize("symbol", ["kernscope_b200_matmul_m256_n256_k64_s4_a2_g8",
                                    "kernscope_b200_matmul_m128_n64_k64_s3_a1_g1"])
def test_runner_selects_config_by_symbol(cuda_ok, tmp_path, symbol):
    path = [p for p in fixture_paths() if os.path.basename(p).startswith("matmul_64x64x64")][0]
    fx = load_fixture(path)
    (tmp_path / "a.bin").write_bytes(fx["a"].tobytes())
    (tmp_path / "b.bin").write_bytes(fx["b"].tobytes())
    out = tmp_path / "out.bin"
    r = _run("--family", "matmul", "--kernel", symbol, "--in", tmp_path / "a.bin", "--in", tmp_path / "b.bin",
             "--out", out, "--out-size", fx["expected"].nbytes, "--int", 64, "--int", 64, "--int", 64)
    assert r.returncode == 0 and symbol in r.stdout, r.stdout + r.stderr
    got = np.frombuffer(out.read_bytes(), dtype=fx["expected"].dtype).reshape(fx["expected"].shape)
    assert_bf16_close(got, fx["expected"], gate=True)


@pytest.mark.gpu
@pytest.mark.parametrize("fixture,symbol", [("softmax_32x512_s0", "kernscope_b200_softmax_b256_v8_onepass"),
                                            ("matmul_64x64x64_s0", "kernscope_b200_matmul_m128_n256_k64_s4_a2_g16")])
def test_reference_gate_argv(cuda_ok, tmp_path, fixture, symbol):
    """The reference gate script's argument list, unchanged: --hsaco (any
    path), --kernel with one of this library's symbols, no --family."""
    path = [p for p in fixture_paths() if os.path.basename(p).startswith(fixture)][0]
    fx = load_fixture(path)
    names, ints = ARGS[fx["family"]]
    ins = []
    for n in names:
        p = tmp_path / f"{n}.bin"
        p.write_bytes(np.ascontiguousarray(fx[n]).tobytes())
        ins += ["--in", p]
    out = tmp_path / "out.bin"
    exp = fx["expected"]
    r = _run("--hsaco", tmp_path / "module.hsaco", "--kernel", symbol, "--grid", "1", "--block", "1", *ins,
             "--out", out, "--out-size", exp.nbytes, *sum((["--int", v] for v in ints(fx["shape"])), []))
    assert r.returncode == 0 and symbol in r.stdout, r.stdout + r.stderr
    got = np.frombuffer(out.read_bytes(), dtype=exp.dtype).reshape(exp.shape)
    assert_bf16_close(got, exp, gate=True)
