"""Helpers shared by the tests: numpy <-> torch bf16 and the tolerance checks."""

from __future__ import annotations

import ml_dtypes
import numpy as np

from oracle import metrics as om

BF16 = ml_dtypes.bfloat16
# bf16 outputs: per-element error with the 2^-8*rms floor and norm-wise error
# both <= 1e-2 against the fp32 reference, plus the reference's own verdict.
BF16_TOL = 1e-2
# fp32 full sums: relative error <= 1e-5 against an fp64 sum.
F32_SUM_TOL = 1e-5


def to_torch(a: np.ndarray, device="cuda"):
    import torch

    a = np.ascontiguousarray(a)
    if a.dtype == BF16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).to(device)
    return torch.from_numpy(a.copy()).to(device)


def to_numpy(t) -> np.ndarray:
    import torch

    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(BF16)
    return t.numpy()


def assert_bf16_close(actual, expected, verdict: bool = True, tol: float = BF16_TOL):
    fe = om.floor_rel_err(actual, expected)
    assert fe["max"] <= tol and fe["norm"] <= tol, f"floor rel-err {fe} > {tol}"
    if verdict:
        v = om.verdict(actual, expected)
        assert v["pass"], f"reference verdict failed: {v}"
    return fe
