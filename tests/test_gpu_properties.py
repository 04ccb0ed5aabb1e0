"""GPU: size-independent properties at the benchmark sizes, no oracle needed.

The sampled oracle checks of the other files cover a few panels/heads of the
largest launches; these cover EVERY output element of them through
properties that hold exactly (or to bf16 rounding) by construction:

* matmul with B a permutation matrix is a column gather of A -- bit-exact,
  which exercises every M-panel, N-tile and K-block of the tcgen05 pipeline;
* attention with all keys equal is a (causal prefix) mean of V -- checks the
  causal mask and the P V accumulation on every query row of C5;
* softmax of a constant row is exactly 1/cols; every softmax row sums to 1;
* layernorm with gamma 1, beta 0 gives rows of mean 0 and variance 1;
* bias_gelu is exact at t = 0 (0) and for t >= 6 (t);
* the full fp32 sum is bitwise reproducible, additive over a split, and
  exact on integer-valued inputs.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ks(cuda_ok):
    import torch

    from kernscope_b200 import native, ops

    torch.manual_seed(0)
    return native, ops, torch


@pytest.mark.parametrize("kind", [(128, 4, 2, 16, 0), (256, 5, 2, 16, 0), (256, 3, 1, -8, 1)],
                         ids=["m128", "pair", "m256c1"])
@pytest.mark.parametrize("m", [8192, 65536])
def test_matmul_permutation_gather_bit_exact(ks, m, kind):
    N, ops, torch = ks
    tile_m, st, acc, grp, cg = kind
    n = k = 8192
    g = torch.Generator(device="cuda").manual_seed(3)
    a = (torch.randn(m, k, generator=g, device="cuda") / 90.5).bfloat16()
    perm = torch.randperm(k, generator=g, device="cuda")
    b = torch.zeros(k, n, dtype=torch.bfloat16, device="cuda")
    b[perm, torch.arange(n, device="cuda")] = 1.0  # C[:, j] = A[:, perm[j]]
    c = ops.matmul(a, b, cfg=N.MatmulConfig(tile_m, 256, 64, st, acc, grp, cg))
    torch.cuda.synchronize()
    assert torch.equal(c, a[:, perm])
    del a, b, c
    torch.cuda.empty_cache()


@pytest.mark.parametrize("causal", [True, False])
def test_attention_equal_keys_is_prefix_mean(ks, causal):
    _, ops, torch = ks
    bsz, h, s, d = (8, 32, 8192, 128) if causal else (2, 8, 4096, 128)
    g = torch.Generator(device="cuda").manual_seed(4)
    q = torch.randn(bsz, h, s, d, generator=g, device="cuda").bfloat16()
    k = torch.randn(bsz, h, 1, d, generator=g, device="cuda").bfloat16().expand(bsz, h, s, d).contiguous()
    v = torch.randn(bsz, h, s, d, generator=g, device="cuda").bfloat16()
    o = ops.flash_attention(q, k, v, causal=causal)
    if causal:
        ref = torch.cumsum(v.float(), dim=2)
        ref /= torch.arange(1, s + 1, device="cuda", dtype=torch.float32).view(1, 1, s, 1)
    else:
        ref = v.float().mean(dim=2, keepdim=True).expand_as(v)
    del q, k, v
    err = (o.float() - ref).abs()
    floor = 2.0 ** -8 * ref.pow(2).mean().sqrt()
    rel = err / torch.maximum(ref.abs(), floor)
    assert float(rel.max()) <= 1e-2
    assert float(err.norm() / ref.norm()) <= 1e-2
    del o, ref, err, rel
    torch.cuda.empty_cache()


def test_softmax_constant_rows_exact_and_row_sums(ks):
    _, ops, torch = ks
    r, c = 4096, 8192
    x = (torch.randn(r, 1, device="cuda") * 4).bfloat16().expand(r, c).contiguous()
    y = ops.softmax(x)
    assert torch.all(y == 2.0 ** -13)  # 1/8192, exact in bf16
    x = (torch.randn(r, c, device="cuda") * 2).bfloat16()
    sums = ops.softmax(x).float().sum(dim=1)
    assert float((sums - 1).abs().max()) <= 1e-2


def test_layernorm_unit_affine_moments(ks):
    _, ops, torch = ks
    r, c = 16384, 4096
    x = (torch.randn(r, c, device="cuda") * 2 + 3).bfloat16()
    one = torch.ones(c, dtype=torch.bfloat16, device="cuda")
    zero = torch.zeros(c, dtype=torch.bfloat16, device="cuda")
    y = ops.layernorm(x, one, zero).float()
    assert float(y.mean(dim=1).abs().max()) <= 1e-2
    assert float((y.var(dim=1, unbiased=False) - 1).abs().max()) <= 1e-2


@pytest.mark.parametrize("gelu", ["erf", "tanh"])
def test_bias_gelu_exact_points(ks, gelu):
    _, ops, torch = ks
    r, c = 16384, 16384
    bias = (torch.randn(c, device="cuda") * 0.1).bfloat16()
    x = (-bias).expand(r, c).contiguous()  # t = x + bias = 0 exactly
    assert torch.all(ops.bias_gelu(x, bias, gelu=gelu) == 0)
    x = (torch.rand(r, c, device="cuda") * 58 + 6.5).bfloat16()
    # one rounding of x + bias: wherever the fp32 sum could round, it is far
    # from a bf16 rounding midpoint, so this equals the kernel's bf16 add
    t = (x.float() + bias.float()).bfloat16()
    assert torch.equal(ops.bias_gelu(x, bias, gelu=gelu), t)


def test_full_sum_reproducible_additive_exact(ks):
    _, ops, torch = ks
    n = 1 << 28
    x = torch.rand(n, device="cuda")
    s1 = ops.reduction(x, axis=-1)
    s2 = ops.reduction(x, axis=-1)
    assert torch.equal(s1, s2)  # fixed combine order: bitwise reproducible
    h = (n // 3) & ~3
    parts = ops.reduction(x[:h], axis=-1).double() + ops.reduction(x[h:], axis=-1).double()
    assert abs(float(parts) - float(s1)) <= 1e-6 * float(s1)
    x.copy_(torch.randint(0, 4, (n,), device="cuda").float())
    exact = int(torch.sum(x.to(torch.int64)))
    # integer partials stay exact in fp64; the fp32 output is one rounding of the exact total
    assert float(ops.reduction(x, axis=-1)) == float(np.float32(exact))
