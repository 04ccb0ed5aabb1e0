"""CPU: the C-ABI library loads, exports every symbol the header declares, and
rejects invalid configs/args without touching a GPU."""

from __future__ import annotations

import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "kernscope_b200.h")


@pytest.fixture(scope="module")
def N():
    from kernscope_b200 import native

    return native


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ks_[a-z0-9_]+)\s*\(", src)))


def test_header_symbols_exported(N):
    names = _declared()
    assert len(names) >= 40
    for n in names:
        assert hasattr(N.lib, n), f"{n} declared in the header but not exported"
    assert set(names) == set(N.PROTOTYPES), set(names) ^ set(N.PROTOTYPES)


def test_abi_version_and_status(N):
    assert N.lib.ks_abi_version() == 1
    assert N.status_string(0) == "ok"
    assert N.status_string(N.KS_ERR_INVALID_CONFIG) == "invalid_config"
    assert N.status_string(-5) == "launch_failed"  # GpuError::kLaunchFailed


def test_library_built_from_these_sources(N):
    """The loaded library reports the hash of the sources, headers, nvcc flags
    and nvcc version it was compiled from; it must be this tree's."""
    from kernscope_b200 import build

    assert f"src {build.source_hash()}" in N.lib.ks_build_info().decode()


def test_validate_rowops(N):
    assert N.validate("softmax", N.SoftmaxConfig(256, 8, 0), 4096, 8192) == (0, "")
    st, reason = N.validate("softmax", N.SoftmaxConfig(128, 8, 0), 4096, 8192)
    assert st == N.KS_ERR_INVALID_CONFIG and "registers" in reason
    assert N.validate("softmax", N.SoftmaxConfig(128, 8, 1), 4096, 8192)[0] == 0
    assert N.validate("layernorm", N.LayerNormConfig(512, 8, 0), 16384, 4096)[0] == 0
    assert N.validate("layernorm", N.LayerNormConfig(512, 3, 0), 16384, 4096)[0] == N.KS_ERR_INVALID_CONFIG
    assert N.validate("bias_gelu", N.BiasGeluConfig(256, 8, 1), 1 << 28, 16384)[0] == 0
    assert N.validate("bias_gelu", N.BiasGeluConfig(256, 8, 2), 64, 16)[0] == N.KS_ERR_INVALID_CONFIG
    assert N.validate("softmax", N.SoftmaxConfig(256, 8, 0), 0, 64)[0] == N.KS_ERR_INVALID_ARGS


def test_validate_cluster_rows(N):
    C = N.KS_MODE_CLUSTER
    assert N.validate("softmax", N.SoftmaxConfig(1024, 8, C), 64, 131072) == (0, "")
    assert N.validate("layernorm", N.LayerNormConfig(1024, 8, C), 2, 262144) == (0, "")
    assert N.validate("layernorm", N.LayerNormConfig(256, 8, C), 1, 16) == (0, "")
    for cfg, rows, cols in [
        (N.SoftmaxConfig(1024, 4, C), 64, 131072),  # vec 8 only
        (N.SoftmaxConfig(128, 8, C), 64, 8192),  # block below 256
        (N.SoftmaxConfig(256, 8, C), 64, 200),  # 100 columns per CTA is not a multiple of 8
        (N.SoftmaxConfig(256, 8, C), 2, 262144),  # more than 32 columns per thread over 8 CTAs
    ]:
        st, reason = N.validate("softmax", cfg, rows, cols)
        assert st == N.KS_ERR_INVALID_CONFIG and "cluster" in reason, (cfg, rows, cols, reason)


def test_validate_matmul(N):
    assert N.validate("matmul", N.MatmulConfig(128, 256, 64, 4, 2, 8), 8192, 8192, 8192)[0] == 0
    st, reason = N.validate("matmul", N.MatmulConfig(128, 256, 64, 5, 2, 8), 64, 64, 64)
    assert st == N.KS_ERR_INVALID_CONFIG and "stages" in reason


def test_reduction_workspace_sizes(N):
    cfg = N.ReductionConfig(512, 4, N.KS_MODE_STRIDED)
    args = N.ReductionArgs(None, None, 1, 1 << 28, N.KS_F32, N.KS_F32, -1, None, 0, None)
    n = C.c_size_t(0)
    assert N.lib.ks_reduction_workspace_bytes(C.byref(cfg), C.byref(args), C.byref(n)) == 0
    assert 256 < n.value < 1 << 20
    args.in_dtype = N.KS_BF16
    assert N.lib.ks_reduction_workspace_bytes(C.byref(cfg), C.byref(args), C.byref(n)) == N.KS_ERR_INVALID_CONFIG


def test_kernel_symbols(N):
    assert N.kernel_symbol("softmax", N.SoftmaxConfig(256, 8, 0)) == "kernscope_b200_softmax_b256_v8_onepass"
    assert N.kernel_symbol("matmul", N.MatmulConfig(128, 256, 64, 4, 2, 8)) == \
        "kernscope_b200_matmul_m128_n256_k64_s4_a2_g8"
    assert N.kernel_symbol("matmul", N.MatmulConfig(128, 256, 64, 4, 2, -8)) == \
        "kernscope_b200_matmul_m128_n256_k64_s4_a2_nb8"
    assert N.kernel_symbol("matmul", N.MatmulConfig(256, 256, 64, 3, 1, -8, 1)) == \
        "kernscope_b200_matmul_m256_n256_k64_s3_a1_nb8_c1"
    assert N.kernel_symbol("matmul", N.MatmulConfig(256, 256, 64, 5, 2, 16)) == \
        "kernscope_b200_matmul_m256_n256_k64_s5_a2_g16"  # the CTA pair keeps its name
    assert N.kernel_symbol("flash_attention", N.FlashAttentionConfig(128, 128, 2, 1)).endswith("_causal")


def test_launch_without_gpu_reports_error(N):
    """Launch calls with null pointers fail with invalid_args before any CUDA call."""
    cfg = N.SoftmaxConfig(256, 8, 0)
    args = N.SoftmaxArgs(None, None, 4, 64)
    assert N.lib.ks_softmax_launch(C.byref(cfg), C.byref(args), None) == N.KS_ERR_INVALID_ARGS


def _launch_cases(N):
    """(entry point, config, args) with every pointer null, per family."""
    return [
        ("ks_softmax_launch", N.SoftmaxConfig(256, 8, 0), N.SoftmaxArgs(None, None, 64, 64)),
        ("ks_layernorm_launch", N.LayerNormConfig(128, 8, 0), N.LayerNormArgs(None, None, None, None, 64, 64, 1e-5)),
        ("ks_bias_gelu_launch", N.BiasGeluConfig(128, 8, 1), N.BiasGeluArgs(None, None, None, 64 * 64, 64)),
        ("ks_reduction_launch", N.ReductionConfig(256, 4, 2),
         N.ReductionArgs(None, None, 64, 64, 0, 0, 0, None, 0, None)),
        ("ks_reduction_launch_noalloc", N.ReductionConfig(256, 4, 2),
         N.ReductionArgs(None, None, 64, 64, 0, 0, 0, None, 0, None)),
        ("ks_matmul_launch", N.MatmulConfig(128, 256, 64, 4, 2, 16), N.MatmulArgs(None, None, None, 64, 64, 64)),
        ("ks_flash_attention_launch", N.FlashAttentionConfig(256, 128, 2, 1),
         N.FlashAttentionArgs(None, None, None, None, 1, 1, 128, 128, 128, 0.0)),
    ]


def test_every_launch_rejects_null_pointers_and_null_structs(N):
    """Each family's launch checks its arguments before any CUDA call: null
    device pointers give invalid_args, and so do null config/args structs."""
    for fn, cfg, args in _launch_cases(N):
        f = getattr(N.lib, fn)
        assert f(C.byref(cfg), C.byref(args), None) == N.KS_ERR_INVALID_ARGS, fn
        assert f(None, C.byref(args), None) == N.KS_ERR_INVALID_ARGS, fn
        assert f(C.byref(cfg), None, None) == N.KS_ERR_INVALID_ARGS, fn


def test_negative_sizes_are_rejected(N):
    args = N.SoftmaxArgs(0x1000, 0x2000, -1, 64)
    assert N.lib.ks_softmax_launch(C.byref(N.SoftmaxConfig(256, 8, 0)), C.byref(args), None) == N.KS_ERR_INVALID_ARGS
    assert N.validate("matmul", N.MatmulConfig(128, 256, 64, 4, 2, 16), -1, 64, 64)[0] != N.KS_OK
