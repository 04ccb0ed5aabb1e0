"""GPU parity: softmax, layernorm, bias_gelu (C ABI via ctypes) vs the oracle.

Golden fixtures (written by the reference harness) are checked with the
reference verdict plus the floor-guarded rel-err <= 1e-2; every config of the
sm_100a space that validates for the shape is exercised; the benchmark shapes
are checked at full size (bias_gelu on sampled rows of the full launch).
"""

from __future__ import annotations

import itertools
import os

import ml_dtypes
import numpy as np
import pytest

from _util import assert_bf16_close, to_numpy, to_torch
from conftest import fixture_paths, load_fixture
from oracle import inputs as oin
from oracle import refs as orf

pytestmark = pytest.mark.gpu

BLOCKS = (128, 256, 512, 1024)
VECS = (1, 2, 4, 8)


def MODES(N):
    return (N.KS_MODE_ONEPASS, N.KS_MODE_TWOPASS, N.KS_MODE_STAGED, N.KS_MODE_CLUSTER)


CLUSTER_SHAPES = [(64, 131072), (256, 32768), (3, 16384), (2, 262144), (1000, 4096), (1, 16), (7, 48)]


def _fx(family):
    return [p for p in fixture_paths() if os.path.basename(p).startswith(family + "_")]


@pytest.fixture(scope="module")
def ks(cuda_ok):
    from kernscope_b200 import native, ops

    return native, ops


# ---------------------------------------------------------------- softmax
@pytest.mark.parametrize("path", _fx("softmax"), ids=os.path.basename)
def test_softmax_golden_all_configs(ks, path):
    N, ops = ks
    fx = load_fixture(path)
    r, c = fx["shape"]
    x = to_torch(fx["x"])
    ran = 0
    for block, vec, mode in itertools.product(BLOCKS, VECS, MODES(N)):
        cfg = N.SoftmaxConfig(block, vec, mode)
        st, _ = N.validate("softmax", cfg, r, c)
        if st != 0:
            continue
        y = to_numpy(ops.softmax(x, cfg=cfg))
        assert_bf16_close(y, fx["expected"], gate=True)
        ran += 1
    assert ran > 0


def test_softmax_baseline_full(ks):
    _, ops = ks
    inp = oin.baseline_inputs("softmax", (4096, 8192), seed=1)
    y = to_numpy(ops.softmax(to_torch(inp["x"])))
    assert_bf16_close(y, orf.softmax(inp["x"]))


@pytest.mark.parametrize("shape", [(1, 8), (3, 24), (7, 4104), (2, 65536), (33, 1000)])
def test_softmax_ragged(ks, shape):
    _, ops = ks
    inp = oin.generate_inputs("softmax", shape, seed=5)
    y = to_numpy(ops.softmax(to_torch(inp["x"])))
    assert_bf16_close(y, orf.softmax(inp["x"]))


@pytest.mark.parametrize("shape", [(4099, 256), (1000, 520), (777, 1024), (70000, 64), (129, 8)])
@pytest.mark.parametrize("block", [128, 256, 1024])
def test_softmax_warp_rows(ks, shape, block):
    """Rows of at most 1024 columns run one row per warp: 1, 2 or 4 chunks
    per lane, partly filled warps, and more rows than resident warps."""
    N, ops = ks
    inp = oin.generate_inputs("softmax", shape, seed=9)
    y = to_numpy(ops.softmax(to_torch(inp["x"]), cfg=N.SoftmaxConfig(block, 8, N.KS_MODE_ONEPASS)))
    assert_bf16_close(y, orf.softmax(inp["x"]))


@pytest.mark.parametrize("shape", CLUSTER_SHAPES)
@pytest.mark.parametrize("block", [256, 512, 1024])
def test_softmax_cluster_rows(ks, shape, block):
    """One row over a cluster of 2 to 8 CTAs: 1, 2 or 4 chunks per thread,
    partly filled CTAs, and the max and sum combined through distributed
    shared memory."""
    N, ops = ks
    cfg = N.SoftmaxConfig(block, 8, N.KS_MODE_CLUSTER)
    st, reason = N.validate("softmax", cfg, *shape)
    if st != 0:
        assert "cluster" in reason
        pytest.skip(reason)
    inp = oin.generate_inputs("softmax", shape, seed=11)
    y = to_numpy(ops.softmax(to_torch(inp["x"]), cfg=cfg))
    assert_bf16_close(y, orf.softmax(inp["x"]))


STAGED_WIDE_SHAPES = [(300, 32768), (5, 16384), (1000, 4096), (149, 24576)]


@pytest.mark.parametrize("shape", STAGED_WIDE_SHAPES)
def test_softmax_staged_wide(ks, shape):
    """1024-thread STAGED CTAs: a 200 KB ring of up to 8 rows, three 64 KB
    rows at 32768 columns, more rows than CTAs."""
    N, ops = ks
    cfg = N.SoftmaxConfig(1024, 8, N.KS_MODE_STAGED)
    assert N.validate("softmax", cfg, *shape)[0] == 0
    inp = oin.generate_inputs("softmax", shape, seed=13)
    y = to_numpy(ops.softmax(to_torch(inp["x"]), cfg=cfg))
    assert_bf16_close(y, orf.softmax(inp["x"]))


def test_softmax_rejects_bad_config(ks):
    N, ops = ks
    st, reason = N.validate("softmax", N.SoftmaxConfig(96, 8, 0), 4, 64)
    assert st == N.KS_ERR_INVALID_CONFIG and "block" in reason
    st, reason = N.validate("softmax", N.SoftmaxConfig(128, 8, 0), 4, 100)
    assert st == N.KS_ERR_INVALID_CONFIG and "vec_width" in reason
    import torch

    x = torch.zeros((4, 100), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(N.KsError):
        ops.softmax(x, cfg=N.SoftmaxConfig(128, 8, 0))


# ---------------------------------------------------------------- layernorm
@pytest.mark.parametrize("path", _fx("layernorm"), ids=os.path.basename)
def test_layernorm_golden_all_configs(ks, path):
    N, ops = ks
    fx = load_fixture(path)
    r, c = fx["shape"]
    x, g, b = (to_torch(fx[k]) for k in ("x", "gamma", "beta"))
    ran = 0
    for block, vec, mode in itertools.product(BLOCKS, VECS, MODES(N)):
        cfg = N.LayerNormConfig(block, vec, mode)
        if N.validate("layernorm", cfg, r, c)[0] != 0:
            continue
        y = to_numpy(ops.layernorm(x, g, b, cfg=cfg))
        assert_bf16_close(y, fx["expected"], gate=True)
        ran += 1
    assert ran > 0


def test_layernorm_baseline_full(ks):
    _, ops = ks
    inp = oin.baseline_inputs("layernorm", (16384, 4096), seed=2)
    y = to_numpy(ops.layernorm(*(to_torch(inp[k]) for k in ("x", "gamma", "beta"))))
    assert_bf16_close(y, orf.layernorm(inp["x"], inp["gamma"], inp["beta"]))


@pytest.mark.parametrize("shape", [(1, 8), (5, 40), (3, 1000), (9, 12288)])
def test_layernorm_ragged(ks, shape):
    _, ops = ks
    inp = oin.generate_inputs("layernorm", shape, seed=6)
    y = to_numpy(ops.layernorm(*(to_torch(inp[k]) for k in ("x", "gamma", "beta"))))
    assert_bf16_close(y, orf.layernorm(inp["x"], inp["gamma"], inp["beta"]))


@pytest.mark.parametrize("shape", [(4099, 256), (1000, 520), (777, 1024), (70000, 64), (129, 8)])
@pytest.mark.parametrize("block", [128, 256, 1024])
def test_layernorm_warp_rows(ks, shape, block):
    N, ops = ks
    inp = oin.generate_inputs("layernorm", shape, seed=10)
    cfg = N.LayerNormConfig(block, 8, N.KS_MODE_ONEPASS)
    y = to_numpy(ops.layernorm(*(to_torch(inp[k]) for k in ("x", "gamma", "beta")), cfg=cfg))
    assert_bf16_close(y, orf.layernorm(inp["x"], inp["gamma"], inp["beta"]))


@pytest.mark.parametrize("shape", CLUSTER_SHAPES)
@pytest.mark.parametrize("block", [256, 512, 1024])
def test_layernorm_cluster_rows(ks, shape, block):
    N, ops = ks
    cfg = N.LayerNormConfig(block, 8, N.KS_MODE_CLUSTER)
    st, reason = N.validate("layernorm", cfg, *shape)
    if st != 0:
        assert "cluster" in reason
        pytest.skip(reason)
    inp = oin.generate_inputs("layernorm", shape, seed=12)
    y = to_numpy(ops.layernorm(*(to_torch(inp[k]) for k in ("x", "gamma", "beta")), cfg=cfg))
    assert_bf16_close(y, orf.layernorm(inp["x"], inp["gamma"], inp["beta"]))


@pytest.mark.parametrize("shape", STAGED_WIDE_SHAPES)
def test_layernorm_staged_wide(ks, shape):
    """1024-thread STAGED CTAs read gamma and beta from global memory."""
    N, ops = ks
    cfg = N.LayerNormConfig(1024, 8, N.KS_MODE_STAGED)
    assert N.validate("layernorm", cfg, *shape)[0] == 0
    inp = oin.generate_inputs("layernorm", shape, seed=14)
    y = to_numpy(ops.layernorm(*(to_torch(inp[k]) for k in ("x", "gamma", "beta")), cfg=cfg))
    assert_bf16_close(y, orf.layernorm(inp["x"], inp["gamma"], inp["beta"]))


# ---------------------------------------------------------------- bias_gelu
@pytest.mark.parametrize("path", _fx("bias"), ids=os.path.basename)
def test_bias_gelu_erf_golden_all_configs(ks, path):
    N, ops = ks
    fx = load_fixture(path)
    r, c = fx["shape"]
    x, b = to_torch(fx["x"]), to_torch(fx["bias"])
    ran = 0
    for block, vec in itertools.product(BLOCKS, VECS):
        cfg = N.BiasGeluConfig(block, vec, N.KS_GELU_ERF)
        if N.validate("bias_gelu", cfg, r * c, c)[0] != 0:
            continue
        y = to_numpy(ops.bias_gelu(x, b, gelu="erf", cfg=cfg))
        assert_bf16_close(y, fx["expected"], gate=True)
        ran += 1
    assert ran > 0


def _same_bf16_bits(a, b):
    a, b = np.asarray(a).view(np.uint16), np.asarray(b).view(np.uint16)
    fa = a.view(ml_dtypes.bfloat16).astype(np.float32)
    fb = b.view(ml_dtypes.bfloat16).astype(np.float32)
    return (a == b) | (np.isnan(fa) & np.isnan(fb))


@pytest.mark.parametrize("vec", [8, 4, 2, 1])
@pytest.mark.parametrize("block", [128, 1024])
def test_bias_gelu_erf_bit_exact_every_bf16_code(ks, vec, block):
    """The exact-erf GELU equals the reference bit for bit on all 65536 bf16
    inputs (zeros, subnormals, infinities and NaN included; NaN compares as
    NaN): t = x + 0 runs every code through the table and both closed forms."""
    N, ops = ks
    x = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16).view(ml_dtypes.bfloat16).reshape(64, 1024)
    bias = np.zeros(1024, dtype=ml_dtypes.bfloat16)
    cfg = N.BiasGeluConfig(block, vec, N.KS_GELU_ERF)
    y = to_numpy(ops.bias_gelu(to_torch(x), to_torch(bias), gelu="erf", cfg=cfg))
    with np.errstate(invalid="ignore"):
        exp = orf.bias_gelu(x, bias)
    assert _same_bf16_bits(y, exp).all(), int((~_same_bf16_bits(y, exp)).sum())


def test_bias_gelu_erf_bit_exact_baseline_rows(ks):
    """C3b rows with the reference's erf GELU: bit-identical to the oracle."""
    _, ops = ks
    shape = (16384, 16384)
    inp = oin.baseline_inputs("bias_gelu", shape, seed=2, row0=0, nrows=256)
    y = to_numpy(ops.bias_gelu(to_torch(inp["x"]), to_torch(inp["bias"]), gelu="erf"))
    assert _same_bf16_bits(y, orf.bias_gelu(inp["x"], inp["bias"])).all()


@pytest.mark.parametrize("shape", [(1000, 16384), (77, 8200), (3, 8), (2, 1 << 21)])
def test_bias_gelu_erf_code_table_shapes(ks, shape):
    """The 1024-thread 8-wide erf kernel (a shared-memory table of every bf16
    code, resident grid over 32-row groups) is bit-identical to the oracle
    with a ragged last row group, a last column CTA with one active thread,
    a single row group, and more column CTAs than SMs."""
    N, ops = ks
    inp = oin.generate_inputs("bias_gelu", shape, seed=21)
    cfg = N.BiasGeluConfig(1024, 8, N.KS_GELU_ERF)
    y = to_numpy(ops.bias_gelu(to_torch(inp["x"]), to_torch(inp["bias"]), gelu="erf", cfg=cfg))
    assert _same_bf16_bits(y, orf.bias_gelu(inp["x"], inp["bias"])).all()


@pytest.mark.parametrize("gelu", ["erf", "tanh"])
def test_bias_gelu_baseline_sampled(ks, gelu):
    _, ops = ks
    shape = (16384, 16384)
    inp = oin.baseline_inputs("bias_gelu", shape, seed=2)
    y = ops.bias_gelu(to_torch(inp["x"]), to_torch(inp["bias"]), gelu=gelu)
    rows = np.r_[0:64, 8000:8064, shape[0] - 64:shape[0]]
    got = to_numpy(y[rows.tolist()])
    ref_fn = orf.bias_gelu_tanh if gelu == "tanh" else orf.bias_gelu
    assert_bf16_close(got, ref_fn(inp["x"][rows], inp["bias"]))


def test_bias_gelu_ragged_total(ks):
    """total not a multiple of cols: the flat walk of the reference (i % cols)."""
    import torch

    N, ops = ks
    cols, total = 24, 24 * 5 + 7
    inp = oin.generate_inputs("bias_gelu", (6, cols), seed=9)
    xflat = inp["x"].reshape(-1)[:total].copy()
    x = to_torch(xflat)
    b = to_torch(inp["bias"])
    out = torch.empty_like(x)
    import ctypes as C

    idx = np.arange(total)
    exp = orf.gelu_erf(orf.to_bf16(xflat.astype(np.float32) + inp["bias"][idx % cols].astype(np.float32)))
    for block, vec in itertools.product((128, 1024), (1, 2, 4, 8)):
        cfg = N.BiasGeluConfig(block, vec, N.KS_GELU_ERF)
        args = N.BiasGeluArgs(x.data_ptr(), b.data_ptr(), out.data_ptr(), total, cols)
        out.zero_()
        N.check("launch", N.lib.ks_bias_gelu_launch(C.byref(cfg), C.byref(args), None))
        torch.cuda.synchronize()
        assert _same_bf16_bits(to_numpy(out), exp).all(), (block, vec)


@pytest.mark.parametrize("rows,chunk", [(4096, 512), (1000, 333), (7, 64)])
def test_host_row_pipeline_matches_device(ks, rows, chunk):
    """Row chunks through the three-stream host pipeline give the same bytes
    as one device launch, over two pipelined steps with new host data."""
    import torch

    _, ops = ks
    cols = 4096
    pipe = ops.HostRowPipeline(rows, chunk_rows=chunk)
    x_dev = torch.empty((rows, cols), dtype=torch.bfloat16, device="cuda")
    y_dev = torch.empty_like(x_dev)
    outs = []
    hosts = [(torch.randn(rows, cols) * (s + 1)).bfloat16().pin_memory() for s in range(2)]
    host_out = [torch.empty((rows, cols), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    for s in range(2):
        pipe.step([hosts[s]], [x_dev], host_out[s], y_dev,
                  lambda r0, r1, st: ops.softmax(x_dev[r0:r1], out=y_dev[r0:r1], stream=st))
    pipe.join()
    torch.cuda.synchronize()
    for s in range(2):
        ref = ops.softmax(hosts[s].cuda()).cpu()
        assert torch.equal(host_out[s], ref)
