"""Seeded inputs per family (CPU oracle; test infrastructure only).

``generate_inputs(family, shape, seed)`` restates the reference profile of
kernscope ``tests/golden/kernscope_golden/inputs.py:73-106``: one
``np.random.default_rng(seed)``, fp32/fp64 uniform draws in the same order,
rounded to bf16.  The arrays are bit-identical to the reference's (pinned by
``tests/test_oracle_pins.py``).

``baseline_inputs(workload, ...)`` is the second profile: the distributions
of the benchmark configurations (N(0,2^2) softmax logits, N(0,1) layernorm
activations with gamma N(1,0.1)/beta N(0,0.1), N(0,1)+N(0,0.1) bias_gelu,
uniform[0,1) fp32 for the full sum, N(0,1/sqrt(K)) GEMM operands, N(0,1)
attention Q/K/V).  Large tensors are drawn in row blocks so generation stays
bounded in memory; each block has its own child generator so any block can
be regenerated alone (used to check sampled panels of huge outputs).
"""

from __future__ import annotations

import numpy as np

from .refs import FAMILIES, REFERENCES, attention, to_bf16

DEFAULT_SEED = 0

_ARITY = {"matmul": 3, "bias_gelu": 2, "softmax": 2, "layernorm": 2,
          "reduction": 2, "attention": 3}


def family_arity(family: str) -> int:
    return _ARITY[family]


def output_shape(family: str, shape) -> tuple:
    """Output shape per family (inputs.py:47-59)."""
    if family == "matmul":
        return (shape[0], shape[1])
    if family in ("bias_gelu", "softmax", "layernorm"):
        return tuple(shape)
    if family == "reduction":
        return (shape[1],)
    if family == "attention":
        return (shape[0], shape[2])
    raise KeyError(family)


def generate_inputs(family: str, shape, seed: int = DEFAULT_SEED) -> dict:
    """Reference-profile inputs (inputs.py:73-106): uniform draws -> bf16."""
    if family not in FAMILIES:
        raise KeyError(f"unknown kernel family {family!r}")
    g = np.random.default_rng(seed)
    u = g.uniform
    if family == "matmul":
        m, n, k = shape
        a = to_bf16(u(-1.0, 1.0, (m, k)))
        b = to_bf16(u(-1.0, 1.0, (k, n)))
        return {"a": a, "b": b}
    if family == "bias_gelu":
        r, c = shape
        x = to_bf16(u(-1.0, 1.0, (r, c)))
        return {"x": x, "bias": to_bf16(u(-0.25, 0.25, (c,)))}
    if family == "softmax":
        r, c = shape
        return {"x": to_bf16(u(-2.0, 2.0, (r, c)))}
    if family == "layernorm":
        r, c = shape
        x = to_bf16(u(-1.0, 1.0, (r, c)))
        gamma = to_bf16(u(0.5, 1.5, (c,)))
        beta = to_bf16(u(-0.25, 0.25, (c,)))
        return {"x": x, "gamma": gamma, "beta": beta}
    if family == "reduction":
        r, c = shape
        return {"x": to_bf16(u(-1.0, 1.0, (r, c)))}
    nq, nk, d = shape  # attention
    s = 1.0 / np.sqrt(d)
    q = to_bf16(u(-s, s, (nq, d)))
    k = to_bf16(u(-s, s, (nk, d)))
    return {"q": q, "k": k, "v": to_bf16(u(-1.0, 1.0, (nk, d)))}


def reference_output(family: str, inputs: dict, causal: bool = False):
    """Expected bf16 output (inputs.py:109-120)."""
    if family == "attention" and causal:
        return attention(inputs["q"], inputs["k"], inputs["v"], causal=True)
    return REFERENCES[family](inputs)


# ---------------------------------------------------------------------------
# Baseline profile (benchmark distributions).
# ---------------------------------------------------------------------------

_BLOCK_ROWS = 1024


def _normal_rows(seed: int, stream: int, rows: int, cols: int, sigma: float,
                 mean: float = 0.0, block_rows: int = _BLOCK_ROWS,
                 row0: int = 0, nrows=None) -> np.ndarray:
    """N(mean, sigma) fp32 -> bf16 for rows [row0, row0+nrows) of a
    rows x cols tensor.  Block i of ``block_rows`` rows is drawn from
    ``default_rng([seed, stream, i])`` so any row range is reproducible."""
    nrows = rows - row0 if nrows is None else nrows
    out = np.empty((nrows, cols), dtype=to_bf16(np.zeros(1)).dtype)
    r = row0
    end = row0 + nrows
    while r < end:
        blk = r // block_rows
        b0 = blk * block_rows
        b1 = min(b0 + block_rows, rows)
        g = np.random.default_rng([seed, stream, blk])
        vals = g.standard_normal((b1 - b0, cols), dtype=np.float32)
        vals = vals * np.float32(sigma) + np.float32(mean)
        lo, hi = r - b0, min(end, b1) - b0
        out[r - row0:r - row0 + (hi - lo)] = to_bf16(vals[lo:hi])
        r = b0 + hi
    return out


def _uniform01_f32(seed: int, stream: int, n: int, block: int = 1 << 22,
                   i0: int = 0, count=None) -> np.ndarray:
    count = n - i0 if count is None else count
    out = np.empty(count, dtype=np.float32)
    i = i0
    end = i0 + count
    while i < end:
        blk = i // block
        b0 = blk * block
        b1 = min(b0 + block, n)
        g = np.random.default_rng([seed, stream, blk])
        vals = g.random(b1 - b0, dtype=np.float32)
        lo, hi = i - b0, min(end, b1) - b0
        out[i - i0:i - i0 + (hi - lo)] = vals[lo:hi]
        i = b0 + hi
    return out


def baseline_inputs(workload: str, shape, seed: int, row0: int = 0, nrows=None) -> dict:
    """Inputs of the ``baseline`` profile for one workload.

    ``row0``/``nrows`` select a row range of the leading operand (x, a, or
    the flattened (b,h) heads for attention) without generating the rest.
    """
    if workload == "softmax":
        r, c = shape
        return {"x": _normal_rows(seed, 0, r, c, 2.0, row0=row0, nrows=nrows)}
    if workload == "layernorm":
        r, c = shape
        return {"x": _normal_rows(seed, 0, r, c, 1.0, row0=row0, nrows=nrows),
                "gamma": _normal_rows(seed, 1, 1, c, 0.1, mean=1.0)[0],
                "beta": _normal_rows(seed, 2, 1, c, 0.1)[0]}
    if workload in ("bias_gelu", "bias_gelu_tanh"):
        r, c = shape
        return {"x": _normal_rows(seed, 3, r, c, 1.0, row0=row0, nrows=nrows),
                "bias": _normal_rows(seed, 4, 1, c, 0.1)[0]}
    if workload == "reduction_full":
        (n,) = shape
        return {"x": _uniform01_f32(seed, 5, n, i0=row0, count=nrows)}
    if workload == "matmul":
        m, n, k = shape
        sig = 1.0 / np.sqrt(k)
        return {"a": _normal_rows(seed, 6, m, k, sig, row0=row0, nrows=nrows),
                "b": _normal_rows(seed, 7, k, n, sig)}
    if workload == "attention":
        b, h, nq, nk, d = shape
        heads = b * h
        h0 = row0
        hn = heads - h0 if nrows is None else nrows
        q = _normal_rows(seed, 8, heads * nq, d, 1.0, block_rows=nq,
                         row0=h0 * nq, nrows=hn * nq).reshape(hn, nq, d)
        k_ = _normal_rows(seed, 9, heads * nk, d, 1.0, block_rows=nk,
                          row0=h0 * nk, nrows=hn * nk).reshape(hn, nk, d)
        v = _normal_rows(seed, 10, heads * nk, d, 1.0, block_rows=nk,
                         row0=h0 * nk, nrows=hn * nk).reshape(hn, nk, d)
        return {"q": q, "k": k_, "v": v}
    raise KeyError(workload)
