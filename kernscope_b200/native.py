"""ctypes binding of ``include/kernscope_b200.h`` (the sm_100a kernel library).

Loads ``kernscope_b200/lib/libkernscope_b200.so`` (built in-tree by
``python -m kernscope_b200.build``).  There is no fallback: if the library
is missing, importing this module raises, and every op raises on a non-zero
status.  Structures mirror the C structs field for field.
"""

from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "lib", "libkernscope_b200.so")

# status codes (ks_status)
KS_OK = 0
KS_ERR_INVALID_CONFIG = -20
KS_ERR_INVALID_ARGS = -21
KS_ERR_WORKSPACE = -22
KS_ERR_DEVICE_TIMEOUT = -23
KS_ERR_ARCH = -24

KS_BF16, KS_F32, KS_F64 = 0, 1, 2
KS_MODE_ONEPASS, KS_MODE_TWOPASS, KS_MODE_STRIDED, KS_MODE_TREE, KS_MODE_STAGED, KS_MODE_CLUSTER = 0, 1, 2, 3, 4, 5
KS_GELU_ERF, KS_GELU_TANH = 0, 1

MODE_NAMES = {"onepass": 0, "twopass": 1, "strided": 2, "tree": 3, "staged": 4}


class KsError(RuntimeError):
    """A non-zero ks_status returned by the C ABI."""

    def __init__(self, fn: str, status: int):
        self.status = status
        super().__init__(f"{fn} failed: {status} ({status_string(status)})")


class SoftmaxConfig(C.Structure):
    _fields_ = [("block", C.c_int), ("vec_width", C.c_int), ("mode", C.c_int)]


class SoftmaxArgs(C.Structure):
    _fields_ = [("x", C.c_void_p), ("out", C.c_void_p), ("rows", C.c_int64), ("cols", C.c_int64)]


class LayerNormConfig(C.Structure):
    _fields_ = [("block", C.c_int), ("vec_width", C.c_int), ("mode", C.c_int)]


class LayerNormArgs(C.Structure):
    _fields_ = [("x", C.c_void_p), ("gamma", C.c_void_p), ("beta", C.c_void_p), ("out", C.c_void_p),
                ("rows", C.c_int64), ("cols", C.c_int64), ("eps", C.c_float)]


class BiasGeluConfig(C.Structure):
    _fields_ = [("block", C.c_int), ("vec_width", C.c_int), ("gelu", C.c_int)]


class BiasGeluArgs(C.Structure):
    _fields_ = [("x", C.c_void_p), ("bias", C.c_void_p), ("out", C.c_void_p),
                ("total", C.c_int64), ("cols", C.c_int64)]


class ReductionConfig(C.Structure):
    _fields_ = [("block", C.c_int), ("vec_width", C.c_int), ("mode", C.c_int)]


class ReductionArgs(C.Structure):
    _fields_ = [("x", C.c_void_p), ("out", C.c_void_p), ("rows", C.c_int64), ("cols", C.c_int64),
                ("in_dtype", C.c_int), ("out_dtype", C.c_int), ("axis", C.c_int),
                ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t),
                ("partial_f64", C.c_void_p)]


class MatmulConfig(C.Structure):
    _fields_ = [("tile_m", C.c_int), ("tile_n", C.c_int), ("tile_k", C.c_int), ("stages", C.c_int),
                ("acc_stages", C.c_int), ("group_m", C.c_int), ("cta_group", C.c_int)]


class MatmulArgs(C.Structure):
    _fields_ = [("a", C.c_void_p), ("b", C.c_void_p), ("out", C.c_void_p),
                ("m", C.c_int64), ("n", C.c_int64), ("k", C.c_int64)]


class FlashAttentionConfig(C.Structure):
    _fields_ = [("tile_m", C.c_int), ("tile_n", C.c_int), ("stages", C.c_int), ("causal", C.c_int)]


class FlashAttentionArgs(C.Structure):
    _fields_ = [("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("out", C.c_void_p),
                ("batch", C.c_int64), ("heads", C.c_int64), ("nq", C.c_int64), ("nk", C.c_int64),
                ("d", C.c_int64), ("scale", C.c_float)]


CONFIG_TYPES = {
    "softmax": SoftmaxConfig, "layernorm": LayerNormConfig, "bias_gelu": BiasGeluConfig,
    "reduction": ReductionConfig, "matmul": MatmulConfig, "flash_attention": FlashAttentionConfig,
}

_P = C.POINTER
# name -> (restype, argtypes); every entry point declared in the header.
PROTOTYPES = {
    "ks_status_string": (C.c_char_p, [C.c_int]),
    "ks_abi_version": (C.c_int, []),
    "ks_build_info": (C.c_char_p, []),
    "ks_gpu_device_count": (C.c_int, [_P(C.c_int)]),
    "ks_gpu_set_device": (C.c_int, [C.c_int]),
    "ks_gpu_get_device": (C.c_int, [_P(C.c_int)]),
    "ks_gpu_arch": (C.c_int, [C.c_int, C.c_char_p, C.c_size_t]),
    "ks_gpu_sm_count": (C.c_int, [C.c_int, _P(C.c_int)]),
    "ks_gpu_l2_bytes": (C.c_int, [C.c_int, _P(C.c_size_t)]),
    "ks_gpu_malloc": (C.c_int, [_P(C.c_void_p), C.c_size_t]),
    "ks_gpu_free": (C.c_int, [C.c_void_p]),
    "ks_gpu_memset": (C.c_int, [C.c_void_p, C.c_int, C.c_size_t, C.c_void_p]),
    "ks_gpu_memcpy_htod": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ks_gpu_memcpy_dtoh": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ks_gpu_host_alloc": (C.c_int, [_P(C.c_void_p), C.c_size_t]),
    "ks_gpu_host_free": (C.c_int, [C.c_void_p]),
    "ks_gpu_stream_create": (C.c_int, [_P(C.c_void_p)]),
    "ks_gpu_stream_destroy": (C.c_int, [C.c_void_p]),
    "ks_gpu_stream_synchronize": (C.c_int, [C.c_void_p]),
    "ks_gpu_synchronize": (C.c_int, []),
    "ks_gpu_event_create": (C.c_int, [_P(C.c_void_p)]),
    "ks_gpu_event_destroy": (C.c_int, [C.c_void_p]),
    "ks_gpu_event_record": (C.c_int, [C.c_void_p, C.c_void_p]),
    "ks_gpu_event_synchronize": (C.c_int, [C.c_void_p]),
    "ks_gpu_event_elapsed_ms": (C.c_int, [C.c_void_p, C.c_void_p, _P(C.c_float)]),
    "ks_device_error_take": (C.c_int, [_P(C.c_int)]),
    "ks_selftest_bounded_wait": (C.c_int, [C.c_uint64, C.c_void_p]),
    "ks_set_wait_limit_ns": (C.c_int, [C.c_uint64]),
    "ks_softmax_validate": (C.c_int, [_P(SoftmaxConfig), C.c_int64, C.c_int64, C.c_char_p, C.c_size_t]),
    "ks_softmax_launch": (C.c_int, [_P(SoftmaxConfig), _P(SoftmaxArgs), C.c_void_p]),
    "ks_layernorm_validate": (C.c_int, [_P(LayerNormConfig), C.c_int64, C.c_int64, C.c_char_p, C.c_size_t]),
    "ks_layernorm_launch": (C.c_int, [_P(LayerNormConfig), _P(LayerNormArgs), C.c_void_p]),
    "ks_bias_gelu_validate": (C.c_int, [_P(BiasGeluConfig), C.c_int64, C.c_int64, C.c_char_p, C.c_size_t]),
    "ks_bias_gelu_launch": (C.c_int, [_P(BiasGeluConfig), _P(BiasGeluArgs), C.c_void_p]),
    "ks_reduction_validate": (C.c_int, [_P(ReductionConfig), _P(ReductionArgs), C.c_char_p, C.c_size_t]),
    "ks_reduction_workspace_bytes": (C.c_int, [_P(ReductionConfig), _P(ReductionArgs), _P(C.c_size_t)]),
    "ks_reduction_launch": (C.c_int, [_P(ReductionConfig), _P(ReductionArgs), C.c_void_p]),
    "ks_reduction_launch_noalloc": (C.c_int, [_P(ReductionConfig), _P(ReductionArgs), C.c_void_p]),
    "ks_matmul_validate": (C.c_int, [_P(MatmulConfig), C.c_int64, C.c_int64, C.c_int64, C.c_char_p, C.c_size_t]),
    "ks_matmul_launch": (C.c_int, [_P(MatmulConfig), _P(MatmulArgs), C.c_void_p]),
    "ks_flash_attention_validate": (C.c_int, [_P(FlashAttentionConfig), _P(FlashAttentionArgs), C.c_char_p,
                                              C.c_size_t]),
    "ks_flash_attention_launch": (C.c_int, [_P(FlashAttentionConfig), _P(FlashAttentionArgs), C.c_void_p]),
    "ks_peak_sink_words": (C.c_int, [_P(C.c_size_t)]),
    "ks_peak_copy": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ks_peak_read": (C.c_int, [C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p]),
    "ks_peak_mma_bf16": (C.c_int, [C.c_longlong, C.c_void_p, _P(C.c_double), C.c_void_p]),
    "ks_peak_ffma_f32": (C.c_int, [C.c_longlong, C.c_void_p, _P(C.c_double), C.c_void_p]),
    "ks_peak_smem": (C.c_int, [C.c_longlong, C.c_void_p, _P(C.c_double), C.c_void_p]),
    "ks_kernel_symbol": (C.c_int, [C.c_char_p, C.c_void_p, C.c_char_p, C.c_size_t]),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m kernscope_b200.build` "
            "(the kernels have no CPU fallback)")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def status_string(s: int) -> str:
    return lib.ks_status_string(int(s)).decode()


def check(fn: str, status: int) -> None:
    if status != KS_OK:
        raise KsError(fn, status)


def exported_symbols() -> list[str]:
    return sorted(PROTOTYPES)


def kernel_symbol(family: str, cfg) -> str:
    buf = C.create_string_buffer(256)
    check("ks_kernel_symbol", lib.ks_kernel_symbol(family.encode(), C.byref(cfg), buf, 256))
    return buf.value.decode()


def validate(family: str, cfg, *shape_or_args) -> tuple[int, str]:
    """Run ks_<family>_validate; returns (status, reason)."""
    buf = C.create_string_buffer(512)
    fn = getattr(lib, f"ks_{family}_validate")
    if family in ("reduction", "flash_attention"):
        st = fn(C.byref(cfg), C.byref(shape_or_args[0]), buf, 512)
    else:
        st = fn(C.byref(cfg), *[C.c_int64(v) for v in shape_or_args], buf, 512)
    return st, buf.value.decode()
