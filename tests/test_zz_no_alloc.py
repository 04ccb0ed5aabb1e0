"""GPU: ks_reduction_launch_noalloc, the reduction for callers that cannot
call cudaMalloc (e.g. a plugin inside a framework that owns all device
memory, or a latency-critical path that cannot take cudaMalloc's device-wide
synchronisation).

Its partials and counters live in a library-owned static device array, so
the test checks, through the C ABI, that two calls in a row give the same
results as ks_reduction_launch with a caller workspace (the array keeps the
previous call's contents, so the second call also shows the launch clears
what must start at zero), and that a shape needing more scratch than the
array holds is refused with KS_ERR_WORKSPACE.  This file is collected last
so that a run stopping at the first failure has run every other test.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from _util import F32_SUM_TOL, assert_bf16_close, to_numpy, to_torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ks(cuda_ok):
    from kernscope_b200 import native, ops

    return native, ops


def _run(N, fn, cfg, args):
    import torch

    N.check(fn, getattr(N.lib, fn)(C.byref(cfg), C.byref(args), C.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()


def test_full_sum_matches_workspace_launch_twice(ks):
    import torch

    N, ops = ks
    cfg = N.ReductionConfig(512, 4, N.KS_MODE_STRIDED)
    rng = np.random.default_rng(123)
    for call, n in enumerate((1 << 24, (1 << 22) + 3)):  # two calls in a row, different sizes
        x = to_torch(rng.random(n, dtype=np.float32))
        ref_out = torch.empty(1, dtype=torch.float32, device="cuda")
        ref_p64 = torch.zeros(1, dtype=torch.float64, device="cuda")
        ws = ops.reduction_workspace(x, axis=-1, cfg=cfg)
        _run(N, "ks_reduction_launch", cfg, ops.reduction_args(x, ref_out, -1, torch.float32, ws, ref_p64))
        out = torch.full((1,), float("nan"), dtype=torch.float32, device="cuda")
        p64 = torch.zeros(1, dtype=torch.float64, device="cuda")
        _run(N, "ks_reduction_launch_noalloc", cfg, ops.reduction_args(x, out, -1, torch.float32, None, p64))
        got, want = float(out.item()), float(ref_out.item())
        assert abs(got - want) <= F32_SUM_TOL * abs(want), (call, got, want)
        assert abs(float(p64.item()) - float(ref_p64.item())) <= 1e-12 * abs(float(ref_p64.item()))


def test_axis0_matches_workspace_launch_twice(ks):
    import torch

    N, ops = ks
    cfg = N.ReductionConfig(256, 8, N.KS_MODE_TREE)
    rng = np.random.default_rng(7)
    for shape in ((65536, 64), (4099, 512)):
        import ml_dtypes

        x = to_torch(rng.uniform(-1, 1, shape).astype(np.float32).astype(ml_dtypes.bfloat16))
        ref = to_numpy(ops.reduction(x, axis=0, cfg=cfg))
        out = torch.empty(shape[1], dtype=torch.bfloat16, device="cuda")
        args = ops.reduction_args(x, out, 0, torch.bfloat16)
        need = C.c_size_t(0)
        N.check("ws", N.lib.ks_reduction_workspace_bytes(C.byref(cfg), C.byref(args), C.byref(need)))
        assert 0 < need.value <= (1 << 20)  # fits the library's scratch array
        _run(N, "ks_reduction_launch_noalloc", cfg, args)
        assert_bf16_close(to_numpy(out), ref)


def test_oversize_is_refused(ks):
    import torch

    N, ops = ks
    cfg = N.ReductionConfig(256, 8, N.KS_MODE_TREE)
    rows, cols = 1 << 16, 1 << 16  # the row split needs far more than 1 MiB of partials
    args = N.ReductionArgs(None, None, rows, cols, N.KS_BF16, N.KS_BF16, 0, None, 0, None)
    need = C.c_size_t(0)
    N.check("ws", N.lib.ks_reduction_workspace_bytes(C.byref(cfg), C.byref(args), C.byref(need)))
    assert need.value > (1 << 20)
    x = torch.zeros(8, dtype=torch.bfloat16, device="cuda")  # never read: refused before launch
    args.x, args.out = x.data_ptr(), x.data_ptr()
    st = N.lib.ks_reduction_launch_noalloc(C.byref(cfg), C.byref(args), None)
    assert st == N.KS_ERR_WORKSPACE
