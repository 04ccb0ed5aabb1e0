"""GPU parity: the reduction family vs the oracle.

axis 0 (the reference family) against the golden fixtures with the reference
verdict; the full fp32 sum of 2^28 uniform[0,1) values against an fp64 sum at
rel-err <= 1e-5; determinism run to run; workspace errors.
"""

from __future__ import annotations

import ctypes as C
import itertools
import os

import numpy as np
import pytest

from _util import F32_SUM_TOL, assert_bf16_close, to_numpy, to_torch
from conftest import fixture_paths, load_fixture
from oracle import inputs as oin
from oracle import refs as orf

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ks(cuda_ok):
    from kernscope_b200 import native, ops

    return native, ops


def _fx():
    return [p for p in fixture_paths() if os.path.basename(p).startswith("reduction_")]


@pytest.mark.parametrize("path", _fx(), ids=os.path.basename)
def test_axis0_golden_all_configs(ks, path):
    N, ops = ks
    fx = load_fixture(path)
    r, c = fx["shape"]
    x = to_torch(fx["x"])
    ran = 0
    for block, vec, mode in itertools.product((128, 256, 512, 1024), (1, 2, 4, 8),
                                              (N.KS_MODE_STRIDED, N.KS_MODE_TREE)):
        cfg = N.ReductionConfig(block, vec, mode)
        if c % vec:
            continue
        y = to_numpy(ops.reduction(x, axis=0, cfg=cfg))
        assert_bf16_close(y, fx["expected"], gate=True)
        ran += 1
    assert ran > 0


@pytest.mark.parametrize("shape", [(1, 8), (4099, 24), (65536, 16), (3, 40000), (100000, 1)])
def test_axis0_shapes_f32(ks, shape):
    N, ops = ks
    rng = np.random.default_rng(11)
    xf = rng.uniform(-1, 1, shape).astype(np.float32)
    y = to_numpy(ops.reduction(to_torch(xf), axis=0, out_dtype=__import__("torch").float32))
    exp = np.sum(xf.astype(np.float64), axis=0)
    # fp32 summation in any order: |error| <= (n - 1) * 2^-24 * sum |x| (+ output rounding)
    bound = shape[0] * 2.0 ** -24 * np.sum(np.abs(xf.astype(np.float64)), axis=0) + 2.0 ** -24 * np.abs(exp)
    assert (np.abs(y.astype(np.float64) - exp) <= bound + 1e-30).all()


def test_full_sum_baseline(ks):
    import torch

    N, ops = ks
    n = 1 << 28
    x = oin.baseline_inputs("reduction_full", (n,), seed=2)["x"]
    xt = to_torch(x)
    p64 = torch.zeros(1, dtype=torch.float64, device="cuda")
    y = ops.reduction(xt, axis=-1, partial_f64=p64)
    ref = orf.sum_full_f64(x)
    got = float(to_numpy(y)[0])
    assert abs(got - ref) / abs(ref) <= F32_SUM_TOL
    assert abs(float(p64.item()) - ref) / abs(ref) <= 1e-9
    # deterministic: fixed-order combine gives the same bits every launch
    y2 = ops.reduction(xt, axis=-1)
    assert to_numpy(y2)[0] == to_numpy(y)[0]


@pytest.mark.parametrize("n", [1, 3, 4, 1000, 4097, 1 << 20])
@pytest.mark.parametrize("mode", ["strided", "tree"])
def test_full_sum_small(ks, n, mode):
    N, ops = ks
    rng = np.random.default_rng(n)
    x = rng.random(n, dtype=np.float32)
    cfg = N.ReductionConfig(256, 4, N.MODE_NAMES[mode])
    y = ops.reduction(to_torch(x), axis=-1, cfg=cfg)
    ref = float(np.sum(x.astype(np.float64)))
    assert abs(float(to_numpy(y)[0]) - ref) <= F32_SUM_TOL * abs(ref) + 1e-7


def test_workspace_missing_is_an_error(ks):
    import torch

    N, ops = ks
    x = torch.ones((4096, 64), dtype=torch.bfloat16, device="cuda")
    out = torch.empty(64, dtype=torch.bfloat16, device="cuda")
    cfg = N.ReductionConfig(256, 8, N.KS_MODE_TREE)
    args = ops.reduction_args(x, out, 0, torch.bfloat16)
    need = C.c_size_t(0)
    N.check("ws", N.lib.ks_reduction_workspace_bytes(C.byref(cfg), C.byref(args), C.byref(need)))
    assert need.value > 0
    st = N.lib.ks_reduction_launch(C.byref(cfg), C.byref(args), None)
    assert st == N.KS_ERR_WORKSPACE
