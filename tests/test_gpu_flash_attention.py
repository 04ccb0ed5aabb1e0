"""GPU parity: attention forward vs the oracle.

The reference's single-head golden fixtures (d = 16, 32 on the CUDA-core
path, d = 128 on the tcgen05 path; causal and not) with the reference
verdict; multi-head [B,H,N,d] shapes with ragged sequence lengths; and the
C5 configuration (B8 H32 N8192 d128, causal) on sampled heads of the full
launch.
"""

from __future__ import annotations

import os

import numpy as np
import pytest

from _util import assert_attention_close, assert_bf16_close, to_numpy, to_torch
from conftest import fixture_paths, load_fixture
from oracle import inputs as oin
from oracle import refs as orf

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ks(cuda_ok):
    from kernscope_b200 import native, ops

    return native, ops


def _fx():
    return [p for p in fixture_paths() if os.path.basename(p).startswith("attention_")]


@pytest.mark.parametrize("path", _fx(), ids=os.path.basename)
def test_attention_golden(ks, path):
    _, ops = ks
    fx = load_fixture(path)
    q, k, v = (to_torch(fx[n]) for n in ("q", "k", "v"))
    o = to_numpy(ops.flash_attention(q, k, v, causal=fx["causal"]))
    if fx["shape"][2] == 128:  # tensor-core path: P enters the MMA as bf16
        rho = orf.attention_abs_weight(fx["q"], fx["k"], fx["v"], causal=fx["causal"])
        assert_attention_close(o, fx["expected"], rho)
    else:  # the reference's gate shapes (d = 16, 32): CUDA-core path, full verdict
        assert_bf16_close(o, fx["expected"], gate=True)


def _check_mh(o, q, k, v, causal):
    exp = orf.attention_bhnd(q, k, v, causal=causal)
    b, h = q.shape[:2]
    rho = np.stack([orf.attention_abs_weight(q[i, j], k[i, j], v[i, j], causal=causal)
                    for i in range(b) for j in range(h)]).reshape(exp.shape)
    if q.shape[-1] in (64, 128):  # tensor-core path: P enters the MMA as bf16
        assert_attention_close(o, exp, rho)
    else:
        assert_bf16_close(o, exp)


def _mh(shape, seed, scale=1.0):
    b, h, nq, nk, d = shape
    g = np.random.default_rng(seed)
    mk = lambda n: orf.to_bf16(g.standard_normal((b, h, n, d), dtype=np.float32) * np.float32(scale))
    return mk(nq), mk(nk), mk(nk)


# (tile_m, tile_n): two query tiles per CTA, one with S double-buffered, and
# two query tiles with S in 64-key slots
TILES = [(256, 128), (128, 128), (256, 64)]


@pytest.mark.parametrize("tiles", TILES, ids=lambda t: f"m{t[0]}n{t[1]}")
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("shape", [(1, 1, 256, 256, 128), (2, 3, 384, 384, 128), (1, 2, 300, 300, 128),
                                   (1, 1, 1, 1, 128), (1, 1, 129, 129, 128), (1, 1, 640, 640, 128),
                                   (1, 1, 192, 192, 128), (1, 2, 130, 130, 128)])
def test_attention_multihead(ks, shape, causal, tiles):
    N, ops = ks
    q, k, v = _mh(shape, 7)
    cfg = N.FlashAttentionConfig(tiles[0], tiles[1], 2, int(causal))
    o = to_numpy(ops.flash_attention(to_torch(q), to_torch(k), to_torch(v), causal=causal, cfg=cfg))
    _check_mh(o, q, k, v, causal)


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("shape", [(1, 1, 256, 256, 64), (2, 3, 384, 384, 64), (1, 2, 300, 300, 64),
                                   (1, 1, 1, 1, 64), (1, 1, 129, 129, 64), (1, 2, 200, 520, 64),
                                   (1, 1, 520, 200, 64)])
@pytest.mark.parametrize("tile_n", [128, 64])
def test_attention_d64_tensor_cores(ks, shape, causal, tile_n):
    """d = 64 on the tcgen05 kernels (two query tiles per CTA): one 64-column
    box per tile, P V with N = 64."""
    N, ops = ks
    q, k, v = _mh(shape, 11)
    cfg = N.FlashAttentionConfig(256, tile_n, 2, int(causal))
    o = to_numpy(ops.flash_attention(to_torch(q), to_torch(k), to_torch(v), causal=causal, cfg=cfg))
    _check_mh(o, q, k, v, causal)


@pytest.mark.parametrize("tile_n", [128, 64])
def test_attention_d64_large_logits(ks, tile_n):
    N, ops = ks
    q, k, v = _mh((1, 2, 512, 512, 64), 12, scale=4.0)
    cfg = N.FlashAttentionConfig(256, tile_n, 2, 1)
    o = to_numpy(ops.flash_attention(to_torch(q), to_torch(k), to_torch(v), causal=True, cfg=cfg))
    _check_mh(o, q, k, v, True)


@pytest.mark.parametrize("tiles", TILES, ids=lambda t: f"m{t[0]}n{t[1]}")
@pytest.mark.parametrize("shape", [(1, 2, 200, 520, 128), (1, 1, 520, 200, 128), (2, 1, 64, 1000, 64)])
def test_attention_cross_lengths(ks, shape, tiles):
    N, ops = ks
    q, k, v = _mh(shape, 8)
    cfg = N.FlashAttentionConfig(tiles[0], tiles[1], 2, 0)
    o = to_numpy(ops.flash_attention(to_torch(q), to_torch(k), to_torch(v), causal=False, cfg=cfg))
    _check_mh(o, q, k, v, False)


@pytest.mark.parametrize("tiles", TILES, ids=lambda t: f"m{t[0]}n{t[1]}")
def test_attention_large_logits(ks, tiles):
    """Scores spread far apart force the running-max rescale of O."""
    N, ops = ks
    q, k, v = _mh((1, 2, 512, 512, 128), 9, scale=4.0)
    cfg = N.FlashAttentionConfig(tiles[0], tiles[1], 2, 1)
    o = to_numpy(ops.flash_attention(to_torch(q), to_torch(k), to_torch(v), causal=True, cfg=cfg))
    _check_mh(o, q, k, v, True)


@pytest.mark.parametrize("tiles", TILES, ids=lambda t: f"m{t[0]}n{t[1]}")
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("d", [128, 64])
def test_attention_score_jumps(ks, tiles, causal, d):
    """Scores that jump far above every earlier key of their row: inside a
    128-key tile (key 100, about 2^76 above keys 0-63 in exp2 terms), a
    moderate rise in the next tile (key 200, about 2^13 higher) and another
    far jump in the first half of a later tile (key 300, about 2^100
    higher).  The kernels move their exponent offset and rescale the P and O
    they already hold; a missed rescale leaves earlier terms 2^64 or more
    too large."""
    N, ops = ks
    b, h, n = 1, 2, 512
    g = np.random.default_rng(31)
    q, k, v = (g.standard_normal((b, h, n, d), dtype=np.float32) for _ in range(3))
    q[..., 0] = 10.0  # a component every query shares
    k[..., 100, 0] = 60.0
    k[..., 200, 0] = 70.0
    k[..., 300, 0] = 150.0
    q, k, v = (orf.to_bf16(x) for x in (q, k, v))
    cfg = N.FlashAttentionConfig(tiles[0], tiles[1], 2, int(causal))
    o = to_numpy(ops.flash_attention(to_torch(q), to_torch(k), to_torch(v), causal=causal, cfg=cfg))
    assert np.isfinite(o.astype(np.float32)).all()
    _check_mh(o, q, k, v, causal)


@pytest.mark.parametrize("tile_n", [128, 64])
def test_attention_c5_sampled(ks, tile_n):
    """C5: B8 H32 N8192 d128 causal, Q/K/V ~ N(0,1); heads (0,0) and (7,31)
    of the full launch checked against the oracle."""
    N, ops = ks
    b, h, s, d = 8, 32, 8192, 128
    inp = oin.baseline_inputs("attention", (b, h, s, s, d), seed=4)
    q, k, v = (to_torch(inp[n].reshape(b, h, s, d)) for n in ("q", "k", "v"))
    o = ops.flash_attention(q, k, v, causal=True, cfg=N.FlashAttentionConfig(256, tile_n, 2, 1))
    for bi, hi in ((0, 0), (7, 31)):
        idx = bi * h + hi
        qi, ki, vi = inp["q"][idx], inp["k"][idx], inp["v"][idx]
        exp = orf.attention(qi, ki, vi, causal=True)
        assert_attention_close(to_numpy(o[bi, hi]), exp, orf.attention_abs_weight(qi, ki, vi, causal=True))


def test_attention_invalid(ks):
    N, _ = ks
    a = N.FlashAttentionArgs(None, None, None, None, 1, 1, 128, 128, 512, 0.0)
    assert N.validate("flash_attention", N.FlashAttentionConfig(128, 128, 2, 1), a)[0] == N.KS_ERR_INVALID_CONFIG
    a.d = 128
    assert N.validate("flash_attention", N.FlashAttentionConfig(64, 128, 2, 1), a)[0] == N.KS_ERR_INVALID_CONFIG
    assert N.validate("flash_attention", N.FlashAttentionConfig(128, 128, 2, 1), a)[0] == 0
    assert N.validate("flash_attention", N.FlashAttentionConfig(256, 128, 2, 1), a)[0] == 0
    assert N.validate("flash_attention", N.FlashAttentionConfig(192, 128, 2, 1), a)[0] == N.KS_ERR_INVALID_CONFIG
    assert N.validate("flash_attention", N.FlashAttentionConfig(256, 64, 2, 1), a)[0] == 0
    assert N.validate("flash_attention", N.FlashAttentionConfig(128, 64, 2, 1), a)[0] == N.KS_ERR_INVALID_CONFIG
