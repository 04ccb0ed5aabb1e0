"""GPU parity: the tcgen05 GEMM vs the oracle.

Golden fixtures (reference-written) and the 512^3 configuration C1 with the
reference verdict; every tile/stage/accumulator config; ragged M/N/K; the
CUDA-core path for unaligned shapes; the 8192^3 configuration on a full
128-row panel plus 4096 random elements against an fp32 reference.
"""

from __future__ import annotations

import itertools
import os

import numpy as np
import pytest

from _util import assert_bf16_close, to_numpy, to_torch
from conftest import fixture_paths, load_fixture
from oracle import inputs as oin
from oracle import refs as orf

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ks(cuda_ok):
    from kernscope_b200 import native, ops

    return native, ops


def _configs(N):
    """Every tile/stage/accumulator config: one CTA (tile_m 128), CTA pairs
    (tile_m 256) and one-CTA 256-row tiles (tile_m 256, cta_group 1)."""
    for bm, bn, st, acc, cg in itertools.product((128, 256), (64, 128, 256), (2, 3, 4, 5, 6), (1, 2), (0, 1)):
        if cg == 1 and bm != 256:
            continue
        cfg = N.MatmulConfig(bm, bn, 64, st, acc, 8, cg)
        if N.validate("matmul", cfg, 64, 64, 64)[0] == 0:
            yield cfg


def _fx():
    return [p for p in fixture_paths() if os.path.basename(p).startswith("matmul_")]


@pytest.mark.parametrize("path", _fx(), ids=os.path.basename)
def test_matmul_golden(ks, path):
    N, ops = ks
    fx = load_fixture(path)
    a, b = to_torch(fx["a"]), to_torch(fx["b"])
    for cfg in _configs(N):
        y = to_numpy(ops.matmul(a, b, cfg=cfg))
        assert_bf16_close(y, fx["expected"], gate=True)


def test_matmul_c1_512(ks):
    """C1 (512^3, the reference profile).  The reference's max_rel_err with
    eps 1e-6 is ill-conditioned here: its own driver gates matmul at 64^3
    because a correct fp32-accumulate GEMM drifts past 1e-2 on near-zero
    outputs at K=512 (tools/tune/src/driver_matmul.cpp:58-66).  So at 512^3
    the check is the benchmark tolerance (floor rel-err and norm-wise error
    <= 1e-2) plus the verdict's cosine/pcc thresholds, against the golden and
    against an fp64 product; every element is also within 2 bf16 ulps of the
    fp64 product rounded to bf16."""
    from oracle import metrics as om

    N, ops = ks
    inp = oin.generate_inputs("matmul", (512, 512, 512), seed=0)
    exp = orf.matmul(inp["a"], inp["b"])
    r64 = inp["a"].astype(np.float64) @ inp["b"].astype(np.float64)
    a, b = to_torch(inp["a"]), to_torch(inp["b"])
    for cfg in _configs(N):
        y = to_numpy(ops.matmul(a, b, cfg=cfg))
        assert_bf16_close(y, exp)
        assert_bf16_close(y, orf.to_bf16(r64))
        v = om.verdict(y, exp)
        assert v["cosine"] >= om.COSINE_MIN and v["pcc"] >= om.PCC_MIN, v
        ulp = np.abs(orf.to_bf16(r64).astype(np.float64)) * 2.0 ** -7 + 2.0 ** -133
        assert (np.abs(y.astype(np.float64) - r64) <= ulp + 1e-5).all()


@pytest.mark.parametrize("shape", [(1, 8, 8), (130, 264, 72), (257, 136, 200), (1000, 520, 1032),
                                   (128, 256, 8), (3, 1024, 4096)])
def test_matmul_ragged(ks, shape):
    N, ops = ks
    inp = oin.generate_inputs("matmul", shape, seed=3)
    exp = orf.matmul(inp["a"], inp["b"])
    a, b = to_torch(inp["a"]), to_torch(inp["b"])
    for cfg in (N.MatmulConfig(128, 256, 64, 4, 2, 8), N.MatmulConfig(128, 64, 64, 3, 1, 1),
                N.MatmulConfig(256, 256, 64, 5, 2, 16), N.MatmulConfig(256, 128, 64, 3, 1, 1),
                N.MatmulConfig(256, 256, 64, 3, 1, -8, 1), N.MatmulConfig(256, 128, 64, 4, 2, 3, 1)):
        assert_bf16_close(to_numpy(ops.matmul(a, b, cfg=cfg)), exp)


# (tile_m, stages, acc_stages, cta_group): one CTA, CTA pair, one-CTA 256-row tile
KINDS = [(128, 4, 2, 0), (256, 5, 2, 0), (256, 3, 1, 1)]


@pytest.mark.parametrize("shape", [(1000, 2056, 264), (4096, 1024, 512), (130, 264, 72), (8192, 256, 128)])
@pytest.mark.parametrize("kind", KINDS, ids=lambda t: f"m{t[0]}c{t[3]}")
def test_matmul_nband_raster_bit_identical(ks, shape, kind):
    """Negative group_m walks bands of N-tiles (N-tiles fastest, B loaded
    evict_last).  The raster only reorders the tiles, so every band width
    gives the bits of the M-group raster, including bands wider than the
    N extent and ragged last bands; and every tile kind gives the bits of
    the one-CTA 128-row kernel (each output accumulates K in order)."""
    N, ops = ks
    tm, st, acc, cg = kind
    inp = oin.generate_inputs("matmul", shape, seed=5)
    a, b = to_torch(inp["a"]), to_torch(inp["b"])
    base = to_numpy(ops.matmul(a, b, cfg=N.MatmulConfig(128, 256, 64, 4, 2, 8)))
    assert_bf16_close(base, orf.matmul(inp["a"], inp["b"]))
    for g in (8, -1, -3, -8, -32):
        got = to_numpy(ops.matmul(a, b, cfg=N.MatmulConfig(tm, 256, 64, st, acc, g, cg)))
        assert np.array_equal(got.view(np.uint16), base.view(np.uint16)), g


@pytest.mark.parametrize("shape", [(4096, 4096, 64), (4096, 4096, 192), (4096, 4096, 1024)])
def test_matmul_wide_tiles_many_per_cta_bit_identical(ks, shape):
    """One-CTA 256-row tiles free their accumulator one 128-row half at a
    time, and the next tile's MMAs for the other half wait for it over up to
    stages - 1 K-blocks.  With more tiles than SMs each CTA crosses several
    tile boundaries; K of 1, 3 and 16 K-blocks covers the cases with no
    deferral, with a deferral cut short by the last K-block, and with the
    full one.  Every valid configuration gives the bits of the 128-row
    kernel (each output accumulates K in order)."""
    N, ops = ks
    m, n, k = shape
    inp = oin.generate_inputs("matmul", shape, seed=6)
    a, b = to_torch(inp["a"]), to_torch(inp["b"])
    base = to_numpy(ops.matmul(a, b, cfg=N.MatmulConfig(128, 256, 64, 4, 2, 8)))
    n_cfg = 0
    for bn, st, acc in itertools.product((64, 128, 256), (2, 3, 4, 5, 6), (1, 2)):
        cfg = N.MatmulConfig(256, bn, 64, st, acc, -8, 1)
        if N.validate("matmul", cfg, m, n, k)[0] != 0:
            continue
        assert (m // 256) * (n // bn) > 148  # several tiles per CTA
        got = to_numpy(ops.matmul(a, b, cfg=cfg))
        assert np.array_equal(got.view(np.uint16), base.view(np.uint16)), (bn, st, acc)
        n_cfg += 1
    assert n_cfg >= 6


@pytest.mark.parametrize("shape", [(5, 7, 9), (70, 33, 100), (64, 64, 13)])
def test_matmul_unaligned_simt(ks, shape):
    _, ops = ks
    inp = oin.generate_inputs("matmul", shape, seed=4)
    assert_bf16_close(to_numpy(ops.matmul(to_torch(inp["a"]), to_torch(inp["b"]))),
                      orf.matmul(inp["a"], inp["b"]))


def test_matmul_empty(ks):
    import torch

    _, ops = ks
    a = torch.zeros((0, 64), dtype=torch.bfloat16, device="cuda")
    b = torch.zeros((64, 32), dtype=torch.bfloat16, device="cuda")
    assert ops.matmul(a, b).shape == (0, 32)
    a = torch.zeros((16, 0), dtype=torch.bfloat16, device="cuda")
    b = torch.zeros((0, 32), dtype=torch.bfloat16, device="cuda")
    out = torch.full((16, 32), 7.0, dtype=torch.bfloat16, device="cuda")
    ops.matmul(a, b, out=out)
    assert float(out.abs().max()) == 0.0


@pytest.mark.parametrize("kind", KINDS, ids=lambda t: f"m{t[0]}c{t[3]}")
def test_matmul_8192_sampled(ks, kind):
    """C4 8192^3 with N(0, 1/sqrt(K)) operands: a full 128-row panel and 4096
    random elements against an fp32 reference (rel-err <= 1e-2)."""
    N, ops = ks
    tm, st, acc, cg = kind
    cfg = N.MatmulConfig(tm, 256, 64, st, acc, -8 if cg == 1 else 16, cg)
    m = n = k = 8192
    inp = oin.baseline_inputs("matmul", (m, n, k), seed=3)
    y = ops.matmul(to_torch(inp["a"]), to_torch(inp["b"]), cfg=cfg)
    af, bf = inp["a"].astype(np.float32), inp["b"].astype(np.float32)
    r0 = 4096 + 64  # a panel that straddles two 128-row tiles
    panel = to_numpy(y[r0:r0 + 128])
    assert_bf16_close(panel, orf.to_bf16(af[r0:r0 + 128] @ bf))
    rng = np.random.default_rng(0)
    ri, ci = rng.integers(0, m, 4096), rng.integers(0, n, 4096)
    got = to_numpy(y[ri.tolist(), ci.tolist()])
    exp = orf.to_bf16(np.einsum("ij,ji->i", af[ri], bf[:, ci]))
    assert_bf16_close(got, exp)


def test_matmul_invalid_configs(ks):
    N, _ = ks
    assert N.validate("matmul", N.MatmulConfig(64, 128, 64, 4, 2, 8), 64, 64, 64)[0] == N.KS_ERR_INVALID_CONFIG
    assert N.validate("matmul", N.MatmulConfig(128, 256, 64, 6, 2, 8), 64, 64, 64)[0] == N.KS_ERR_INVALID_CONFIG
    assert N.validate("matmul", N.MatmulConfig(128, 96, 64, 4, 2, 8), 64, 64, 64)[0] == N.KS_ERR_INVALID_CONFIG
    assert N.validate("matmul", N.MatmulConfig(256, 64, 64, 4, 2, 8), 64, 64, 64)[0] == N.KS_ERR_INVALID_CONFIG
    assert N.validate("matmul", N.MatmulConfig(256, 256, 64, 6, 2, 8), 64, 64, 64)[0] == 0
    for g in (0, -33, 65):
        assert N.validate("matmul", N.MatmulConfig(128, 256, 64, 4, 2, g), 64, 64, 64)[0] == N.KS_ERR_INVALID_CONFIG
    assert N.validate("matmul", N.MatmulConfig(128, 256, 64, 4, 2, -32), 64, 64, 64)[0] == 0
    # one-CTA 256-row tiles: three stages of 64 KB fit, four do not; two accumulators of 2 x 256 columns
    # exceed TMEM; cta_group 2 needs tile_m 256; cta_group is 0, 1 or 2
    assert N.validate("matmul", N.MatmulConfig(256, 256, 64, 3, 1, 8, 1), 64, 64, 64)[0] == 0
    assert N.validate("matmul", N.MatmulConfig(256, 256, 64, 4, 1, 8, 1), 64, 64, 64)[0] == N.KS_ERR_INVALID_CONFIG
    assert N.validate("matmul", N.MatmulConfig(256, 256, 64, 3, 2, 8, 1), 64, 64, 64)[0] == N.KS_ERR_INVALID_CONFIG
    assert N.validate("matmul", N.MatmulConfig(256, 128, 64, 4, 2, 8, 1), 64, 64, 64)[0] == 0
    assert N.validate("matmul", N.MatmulConfig(128, 256, 64, 4, 2, 8, 2), 64, 64, 64)[0] == N.KS_ERR_INVALID_CONFIG
    assert N.validate("matmul", N.MatmulConfig(256, 256, 64, 3, 1, 8, 3), 64, 64, 64)[0] == N.KS_ERR_INVALID_CONFIG
