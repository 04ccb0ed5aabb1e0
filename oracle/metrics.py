"""Verdict metrics (CPU oracle; test infrastructure only).

``verdict`` restates kernscope ``tests/golden/kernscope_golden/metrics.py:29-116``:
cosine >= 0.999, max_rel_err <= 1e-2 with eps 1e-6 in the denominator, and
pcc >= 0.99, all inclusive, over flattened fp32 views.

``floor_rel_err`` is the benchmark tolerance: |a - r| / max(|r|, 2^-8 rms(r))
per element (the plain |r| + 1e-6 denominator is unstable for outputs near
zero), together with a norm-wise error ||a - r|| / ||r||.
"""

from __future__ import annotations

import numpy as np

COSINE_MIN = 0.999
MAX_REL_ERR_MAX = 1e-2
PCC_MIN = 0.99
EPS = 1e-6


def _flat(x) -> np.ndarray:
    return np.asarray(x).astype(np.float32).ravel()


def cosine(a, r) -> float:
    x, y = _flat(a), _flat(r)
    nx, ny = float(np.linalg.norm(x)), float(np.linalg.norm(y))
    if nx * ny == 0.0:
        return 1.0 if nx == 0.0 and ny == 0.0 else 0.0
    return float(np.dot(x, y) / (nx * ny))


def max_rel_err(a, r, eps: float = EPS) -> float:
    x, y = _flat(a), _flat(r)
    return float(np.max(np.abs(x - y) / (np.abs(y) + eps)))


def pcc(a, r) -> float:
    x, y = _flat(a), _flat(r)
    xc, yc = x - x.mean(), y - y.mean()
    den = float(np.sqrt(np.sum(xc * xc)) * np.sqrt(np.sum(yc * yc)))
    if den == 0.0:
        return 1.0 if np.array_equal(x, y) else 0.0
    return float(np.sum(xc * yc) / den)


def verdict(a, r) -> dict:
    c, m, p = cosine(a, r), max_rel_err(a, r), pcc(a, r)
    ok = c >= COSINE_MIN and m <= MAX_REL_ERR_MAX and p >= PCC_MIN
    return {"pass": bool(ok), "cosine": c, "max_rel_err": m, "pcc": p,
            "thresholds": {"cosine": COSINE_MIN, "max_rel_err": MAX_REL_ERR_MAX,
                           "pcc": PCC_MIN}}


def floor_rel_err(a, r) -> dict:
    """Per-element error with a 2^-8*rms floor, plus the norm-wise error."""
    x = np.asarray(a).astype(np.float64).ravel()
    y = np.asarray(r).astype(np.float64).ravel()
    rms = float(np.sqrt(np.mean(y * y))) if y.size else 0.0
    den = np.maximum(np.abs(y), rms * 2.0 ** -8)
    den = np.where(den == 0.0, 1.0, den)
    ny = float(np.linalg.norm(y))
    return {"max": float(np.max(np.abs(x - y) / den)) if y.size else 0.0,
            "norm": float(np.linalg.norm(x - y) / ny) if ny else float(np.linalg.norm(x))}
