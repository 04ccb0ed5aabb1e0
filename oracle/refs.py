"""Reference math for the six families (CPU oracle; test infrastructure only).

Rounding contract, as in kernscope ``tests/golden/kernscope_golden/refs.py:1-9``:
inputs are bf16 (round-to-nearest-even), arithmetic is fp32, and each output
is rounded to bf16 once.  Functions below restate ``refs.py:57-142`` with the
same operation order so that the bf16 outputs are bit-identical to the
reference on the same inputs (pinned by ``tests/test_oracle_pins.py``).

Extensions (not in the reference, needed by the B200 configurations):

* ``gelu_tanh`` / ``bias_gelu_tanh`` -- tanh-approximation GELU computed in
  fp64 and rounded to bf16 once;
* ``sum_full_f64`` -- the full fp32 sum judged at rel-err 1e-5 (fp64 sum);
* ``attention_bhnd`` -- batched multi-head attention over [B,H,N,d] that
  applies the single-head reference per (b,h).
"""

from __future__ import annotations

import math

import ml_dtypes
import numpy as np

BF16 = ml_dtypes.bfloat16
F32 = np.float32
_SQRT1_2 = 1.0 / math.sqrt(2.0)

# math.erf is C libm erf at double precision, the same routine the reference
# vectorises (refs.py:41).
_erf64 = np.vectorize(math.erf, otypes=[np.float64])


def to_bf16(x) -> np.ndarray:
    """Round to bf16, round-to-nearest-even (refs.py:44-46)."""
    return np.asarray(x).astype(BF16)


def to_f32(x) -> np.ndarray:
    """Upcast to fp32 (refs.py:49-51)."""
    return np.asarray(x).astype(F32)


def matmul(a, b) -> np.ndarray:
    """C = A @ B, fp32 product of the bf16 operands, bf16 out (refs.py:54-56)."""
    return to_bf16(np.matmul(to_f32(a), to_f32(b)))


def gelu_erf(x) -> np.ndarray:
    """0.5*x*(1+erf(x/sqrt2)); erf in fp64, cast to fp32 before the add
    (refs.py:59-63)."""
    t = to_f32(x)
    e = _erf64(t * F32(_SQRT1_2)).astype(F32)
    return to_bf16(F32(0.5) * t * (F32(1.0) + e))


def bias_gelu(x, bias) -> np.ndarray:
    """GELU_erf(bf16(x + bias)), bias broadcast over the last axis
    (refs.py:66-76)."""
    t = to_bf16(to_f32(x) + to_f32(bias))
    return gelu_erf(t)


def gelu_tanh(x) -> np.ndarray:
    """tanh-approximation GELU 0.5t(1+tanh(sqrt(2/pi)(t+0.044715t^3))), fp64."""
    t = np.asarray(x).astype(np.float64)
    u = math.sqrt(2.0 / math.pi) * (t + 0.044715 * t * t * t)
    return to_bf16(0.5 * t * (1.0 + np.tanh(u)))


def bias_gelu_tanh(x, bias) -> np.ndarray:
    """GELU_tanh(bf16(x + bias)); the fusion point matches ``bias_gelu``."""
    t = to_bf16(to_f32(x) + to_f32(bias))
    return gelu_tanh(t)


def softmax(x) -> np.ndarray:
    """Stable row softmax over the last axis, fp32, bf16 out (refs.py:79-84)."""
    xf = to_f32(x)
    e = np.exp(xf - np.max(xf, axis=-1, keepdims=True))
    return to_bf16(e / np.sum(e, axis=-1, keepdims=True))


def layernorm(x, gamma, beta, eps: float = 1e-5) -> np.ndarray:
    """(x-mean)/sqrt(var+eps)*gamma+beta, biased variance (refs.py:87-99)."""
    xf = to_f32(x)
    mu = xf.mean(axis=-1, keepdims=True)
    var = ((xf - mu) ** 2).mean(axis=-1, keepdims=True)
    y = (xf - mu) / np.sqrt(var + eps) * to_f32(gamma) + to_f32(beta)
    return to_bf16(y)


def reduction(x) -> np.ndarray:
    """Axis-0 sum y[j] = sum_i x[i,j], fp32, bf16 out (refs.py:102-110)."""
    return to_bf16(np.sum(to_f32(x), axis=0))


def sum_full_f64(x) -> float:
    """Full sum of every element in fp64 (the 1e-5 judge for fp32 sums)."""
    return float(np.sum(np.asarray(x, dtype=np.float64)))


def attention(q, k, v, causal: bool = False) -> np.ndarray:
    """Single-head O = softmax(Q K^T / sqrt(d)) V, optional causal mask
    (col > row masked), fp32, bf16 out (refs.py:113-142)."""
    qf, kf, vf = to_f32(q), to_f32(k), to_f32(v)
    d = qf.shape[-1]
    s = np.matmul(qf, kf.T) / math.sqrt(d)
    if causal:
        r = np.arange(s.shape[0])[:, None]
        c = np.arange(s.shape[1])[None, :]
        s = np.where(c > r, -np.inf, s)
    e = np.exp(s - np.max(s, axis=-1, keepdims=True))
    p = e / np.sum(e, axis=-1, keepdims=True)
    return to_bf16(np.matmul(p, vf))


def attention_abs_weight(q, k, v, causal: bool = False) -> np.ndarray:
    """rho = softmax(Q K^T / sqrt(d)) |V| in fp32 (single head).

    The scale of the error of any kernel that feeds P to the tensor cores in
    bf16: |O_kernel - O| <= 2^-9 rho + 2^-9 |O| + fp32 terms, since each
    p_i carries a relative rounding error <= 2^-9 and |O| <= rho."""
    qf, kf, vf = to_f32(q), to_f32(k), to_f32(v)
    s = np.matmul(qf, kf.T) / math.sqrt(qf.shape[-1])
    if causal:
        r = np.arange(s.shape[0])[:, None]
        c = np.arange(s.shape[1])[None, :]
        s = np.where(c > r, -np.inf, s)
    e = np.exp(s - np.max(s, axis=-1, keepdims=True))
    return np.matmul(e / np.sum(e, axis=-1, keepdims=True), np.abs(vf))


def attention_bhnd(q, k, v, causal: bool = False, pairs=None) -> np.ndarray:
    """Multi-head attention over [B,H,N,d]: ``attention`` per (b,h).

    ``pairs`` restricts the work to a list of (b,h) heads; the result then has
    shape [len(pairs), Nq, d] in that order.
    """
    b_, h_ = q.shape[0], q.shape[1]
    sel = pairs if pairs is not None else [(b, h) for b in range(b_) for h in range(h_)]
    outs = [attention(q[b, h], k[b, h], v[b, h], causal=causal) for b, h in sel]
    out = np.stack(outs)
    if pairs is None:
        out = out.reshape(b_, h_, *out.shape[1:])
    return out


# name -> callable(inputs) -> expected output (refs.py:146-153 order).
REFERENCES = {
    "matmul": lambda d: matmul(d["a"], d["b"]),
    "bias_gelu": lambda d: bias_gelu(d["x"], d["bias"]),
    "softmax": lambda d: softmax(d["x"]),
    "layernorm": lambda d: layernorm(d["x"], d["gamma"], d["beta"]),
    "reduction": lambda d: reduction(d["x"]),
    "attention": lambda d: attention(d["q"], d["k"], d["v"]),
}
FAMILIES = tuple(REFERENCES)
