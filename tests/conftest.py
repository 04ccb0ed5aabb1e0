"""Shared pytest configuration: the ``gpu`` marker and fixture loading."""

from __future__ import annotations

import glob
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def load_fixture(path: str) -> dict:
    """Load a golden npz; bf16 arrays come back as ml_dtypes.bfloat16."""
    import ml_dtypes

    out = {}
    with np.load(path) as z:
        for k in z.files:
            a = z[k]
            if a.dtype == np.uint16:
                a = a.view(ml_dtypes.bfloat16)
            out[k] = a
    out["shape"] = tuple(int(v) for v in out["shape"])
    out["seed"] = int(out["seed"])
    out["causal"] = bool(int(out["causal"]))
    out["family"] = os.path.basename(path).split("_")[0]
    if out["family"] == "bias":
        out["family"] = "bias_gelu"
    return out


def fixture_paths():
    return sorted(glob.glob(os.path.join(GOLDEN, "*.npz")))


@pytest.fixture(scope="session")
def cuda_ok():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return True
