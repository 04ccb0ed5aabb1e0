"""GPU: runtime ABI and the bounded-wait failure path.

The self-test kernel waits on an mbarrier that nothing completes; the wait is
bounded (a fraction of a second), records the timeout in the device error
word and returns -- the context stays usable, which the follow-up launch
checks.  No fault, trap or hang is involved.
"""

from __future__ import annotations

import ctypes as C

import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def N(cuda_ok):
    from kernscope_b200 import native

    return native


def test_arch_and_counts(N):
    buf = C.create_string_buffer(32)
    N.check("arch", N.lib.ks_gpu_arch(0, buf, 32))
    assert buf.value.decode() == "sm_100a"
    n = C.c_int(0)
    N.check("sms", N.lib.ks_gpu_sm_count(0, C.byref(n)))
    assert n.value == 148
    l2 = C.c_size_t(0)
    N.check("l2", N.lib.ks_gpu_l2_bytes(0, C.byref(l2)))
    assert l2.value > 64 << 20


def test_bounded_wait_selftest(N):
    import torch

    st = N.lib.ks_selftest_bounded_wait(200_000_000, None)  # 0.2 s
    assert st == N.KS_ERR_DEVICE_TIMEOUT
    w = C.c_int(-1)
    N.check("take", N.lib.ks_device_error_take(C.byref(w)))
    assert w.value == 0  # the self-test cleared its record
    # the context is still usable
    from kernscope_b200 import ops

    x = torch.randn((4, 64), device="cuda").to(torch.bfloat16)
    y = ops.softmax(x)
    torch.cuda.synchronize()
    assert torch.allclose(y.float().sum(-1), torch.ones(4, device="cuda"), atol=2e-2)


def test_memcpy_roundtrip(N):
    import numpy as np

    n = 1 << 20
    src = np.arange(n, dtype=np.uint8) * 7
    dst = np.zeros_like(src)
    d = C.c_void_p()
    N.check("malloc", N.lib.ks_gpu_malloc(C.byref(d), n))
    N.check("h2d", N.lib.ks_gpu_memcpy_htod(d, src.ctypes.data, n, None))
    N.check("d2h", N.lib.ks_gpu_memcpy_dtoh(dst.ctypes.data, d, n, None))
    N.check("sync", N.lib.ks_gpu_synchronize())
    N.check("free", N.lib.ks_gpu_free(d))
    assert (src == dst).all()
