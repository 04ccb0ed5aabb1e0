"""Torch-tensor front end of the C ABI (device memory and streams from torch).

Each function validates dtype/layout, builds the family's config and args
structs, and calls ``ks_<family>_launch`` on the current torch stream.  Any
non-zero status raises ``KsError``; there is no CPU or library fallback.

Default configurations are the sm_100a picks for the benchmark shapes; the
tuner (``kernscope-tune``) searches the full config spaces.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import native as N


def _stream_ptr(stream=None) -> C.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _check_bf16_2d(name, t):
    if not (t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous()):
        raise ValueError(f"{name} must be a contiguous bf16 CUDA tensor")


def _pow2_block(cols: int, vec: int, per_thread: int) -> int:
    want = max(1, cols // (vec * per_thread))
    b = 128
    while b < want and b < 1024:
        b *= 2
    return b


def _cluster_default(family: str, make, rows, cols: int):
    """A few very long rows (at most 64 rows of 65536+ columns) leave most SMs
    idle one CTA per row; spreading each row over a cluster measured
    1590 -> 1987 GB/s (softmax) and 1310 -> 1778 GB/s (layernorm) at
    64 x 131072 on B200.  With more rows the per-row CTAs win."""
    if rows is None or rows > 64 or cols < 65536:
        return None
    for block in (512, 1024):
        cfg = make(block, 8, N.KS_MODE_CLUSTER)
        if N.validate(family, cfg, rows, cols)[0] == 0:
            return cfg
    return None


def default_softmax_config(cols: int, rows: int | None = None) -> N.SoftmaxConfig:
    c = _cluster_default("softmax", N.SoftmaxConfig, rows, cols)
    if c is not None:
        return c
    if rows is not None and rows >= 1024 and 16384 < cols <= 32768 and cols % 8 == 0:
        # 1024-thread STAGED CTAs keep three 64 KB rows in flight: 2048 x 32768
        # measured 3786 -> 4123 GB/s against ONEPASS on B200 (equal at 1024 rows)
        return N.SoftmaxConfig(1024, 8, N.KS_MODE_STAGED)
    vec = 8 if cols % 8 == 0 else 4 if cols % 4 == 0 else 2 if cols % 2 == 0 else 1
    block = _pow2_block(cols, vec, 4)
    mode = N.KS_MODE_ONEPASS if cols <= block * 32 else N.KS_MODE_TWOPASS
    return N.SoftmaxConfig(block, vec, mode)


def default_layernorm_config(cols: int, rows: int | None = None) -> N.LayerNormConfig:
    c = _cluster_default("layernorm", N.LayerNormConfig, rows, cols)
    if c is not None:
        return c
    if 8192 < cols <= 16384 and cols % 8 == 0:
        # a two-row bulk-copy ring per 512-thread CTA: 4096 x 16384 measured
        # 3787 -> 4295 GB/s against ONEPASS on B200 (2048 rows: 3627 -> 3771)
        return N.LayerNormConfig(512, 8, N.KS_MODE_STAGED)
    vec = 8 if cols % 8 == 0 else 4 if cols % 4 == 0 else 2 if cols % 2 == 0 else 1
    block = _pow2_block(cols, vec, 4)
    mode = N.KS_MODE_ONEPASS if cols <= block * 32 else N.KS_MODE_TWOPASS
    return N.LayerNormConfig(block, vec, mode)


def default_bias_gelu_config(cols: int, gelu: str = "tanh") -> N.BiasGeluConfig:
    vec = 8 if cols % 8 == 0 else 4 if cols % 4 == 0 else 2 if cols % 2 == 0 else 1
    if gelu != "tanh":
        # 8-wide erf: 1024 threads run the kernel that looks every bf16 code up
        # in a shared-memory table (one CTA per SM)
        return N.BiasGeluConfig(1024 if vec == 8 else 128, vec, N.KS_GELU_ERF)
    return N.BiasGeluConfig(128, vec, N.KS_GELU_TANH)


def default_reduction_config(cols: int, axis: int) -> N.ReductionConfig:
    if axis == -1:
        return N.ReductionConfig(512, 4, N.KS_MODE_STRIDED)
    vec = 8 if cols % 8 == 0 else 4 if cols % 4 == 0 else 2 if cols % 2 == 0 else 1
    return N.ReductionConfig(256, vec, N.KS_MODE_TREE)


def default_matmul_config(m: int, n: int, k: int) -> N.MatmulConfig:
    if n >= 256 and m * n >= 2048 * 2048:
        # 256x256 tiles on one CTA (two M=128 MMAs per B tile, cta_group 1),
        # bands of 8 N-tiles whose B panels stay in L2 (group_m -8)
        return N.MatmulConfig(256, 256, 64, 3, 1, -8, 1)
    return N.MatmulConfig(128, 128, 64, 6, 2, 8)


def default_flash_attention_config(causal: bool) -> N.FlashAttentionConfig:
    return N.FlashAttentionConfig(256, 128, 2, 1 if causal else 0)


def softmax(x: torch.Tensor, out=None, cfg=None, stream=None) -> torch.Tensor:
    _check_bf16_2d("x", x)
    rows, cols = x.shape
    out = torch.empty_like(x) if out is None else out
    cfg = cfg or default_softmax_config(cols, rows)
    args = N.SoftmaxArgs(x.data_ptr(), out.data_ptr(), rows, cols)
    N.check("ks_softmax_launch", N.lib.ks_softmax_launch(C.byref(cfg), C.byref(args), _stream_ptr(stream)))
    return out


def layernorm(x, gamma, beta, eps: float = 1e-5, out=None, cfg=None, stream=None) -> torch.Tensor:
    for nm, t in (("x", x), ("gamma", gamma), ("beta", beta)):
        _check_bf16_2d(nm, t)
    rows, cols = x.shape
    out = torch.empty_like(x) if out is None else out
    cfg = cfg or default_layernorm_config(cols, rows)
    args = N.LayerNormArgs(x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), out.data_ptr(), rows, cols, eps)
    N.check("ks_layernorm_launch", N.lib.ks_layernorm_launch(C.byref(cfg), C.byref(args), _stream_ptr(stream)))
    return out


def bias_gelu(x, bias, gelu: str = "tanh", out=None, cfg=None, stream=None) -> torch.Tensor:
    _check_bf16_2d("x", x)
    _check_bf16_2d("bias", bias)
    cols = bias.numel()
    out = torch.empty_like(x) if out is None else out
    cfg = cfg or default_bias_gelu_config(cols, gelu)
    args = N.BiasGeluArgs(x.data_ptr(), bias.data_ptr(), out.data_ptr(), x.numel(), cols)
    N.check("ks_bias_gelu_launch", N.lib.ks_bias_gelu_launch(C.byref(cfg), C.byref(args), _stream_ptr(stream)))
    return out


_DT = {torch.bfloat16: N.KS_BF16, torch.float32: N.KS_F32}


def reduction_args(x, out, axis: int, out_dtype, workspace=None, partial_f64=None) -> N.ReductionArgs:
    rows, cols = (x.shape[0], x.numel() // x.shape[0]) if x.dim() >= 1 else (1, 1)
    if x.dim() == 1:
        rows, cols = 1, x.numel()
    return N.ReductionArgs(x.data_ptr(), out.data_ptr(), rows, cols, _DT[x.dtype], _DT[out_dtype], axis,
                           workspace.data_ptr() if workspace is not None else None,
                           workspace.numel() if workspace is not None else 0,
                           partial_f64.data_ptr() if partial_f64 is not None else None)


def reduction_workspace(x, axis: int = 0, out_dtype=None, cfg=None) -> torch.Tensor:
    out_dtype = out_dtype or x.dtype
    cols = x.numel() // x.shape[0] if x.dim() > 1 else x.numel()
    cfg = cfg or default_reduction_config(cols, axis)
    dummy = torch.empty(1, dtype=out_dtype, device=x.device)
    args = reduction_args(x, dummy, axis, out_dtype)
    n = C.c_size_t(0)
    N.check("ks_reduction_workspace_bytes",
            N.lib.ks_reduction_workspace_bytes(C.byref(cfg), C.byref(args), C.byref(n)))
    return torch.empty(max(int(n.value), 256), dtype=torch.uint8, device=x.device)


def reduction(x, axis: int = 0, out_dtype=None, out=None, cfg=None, workspace=None, partial_f64=None,
              stream=None) -> torch.Tensor:
    """axis 0: y[j] = sum_i x[i, j]; axis -1: full sum of x (fp32 in/out)."""
    if not (x.is_cuda and x.is_contiguous() and x.dtype in _DT):
        raise ValueError("x must be a contiguous bf16/fp32 CUDA tensor")
    out_dtype = out_dtype or x.dtype
    cols = x.numel() // x.shape[0] if x.dim() > 1 else x.numel()
    if out is None:
        out = torch.empty(1 if axis == -1 else cols, dtype=out_dtype, device=x.device)
    cfg = cfg or default_reduction_config(cols, axis)
    if workspace is None:
        workspace = reduction_workspace(x, axis, out_dtype, cfg)
    args = reduction_args(x, out, axis, out_dtype, workspace, partial_f64)
    N.check("ks_reduction_launch", N.lib.ks_reduction_launch(C.byref(cfg), C.byref(args), _stream_ptr(stream)))
    return out


def matmul(a, b, out=None, cfg=None, stream=None) -> torch.Tensor:
    _check_bf16_2d("a", a)
    _check_bf16_2d("b", b)
    m, k = a.shape
    k2, n = b.shape
    if k != k2:
        raise ValueError("inner dimensions differ")
    out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device) if out is None else out
    cfg = cfg or default_matmul_config(m, n, k)
    args = N.MatmulArgs(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k)
    N.check("ks_matmul_launch", N.lib.ks_matmul_launch(C.byref(cfg), C.byref(args), _stream_ptr(stream)))
    return out


def flash_attention(q, k, v, causal: bool = True, scale: float = 0.0, out=None, cfg=None,
                    stream=None) -> torch.Tensor:
    """q [B,H,Nq,d], k/v [B,H,Nk,d] (or [Nq,d]/[Nk,d] single head)."""
    for nm, t in (("q", q), ("k", k), ("v", v)):
        _check_bf16_2d(nm, t)
    if q.dim() == 2:
        b, h, nq, d = 1, 1, q.shape[0], q.shape[1]
        nk = k.shape[0]
    else:
        b, h, nq, d = q.shape
        nk = k.shape[2]
    out = torch.empty_like(q) if out is None else out
    cfg = cfg or default_flash_attention_config(causal)
    cfg.causal = 1 if causal else 0
    args = N.FlashAttentionArgs(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), b, h, nq, nk, d, scale)
    N.check("ks_flash_attention_launch",
            N.lib.ks_flash_attention_launch(C.byref(cfg), C.byref(args), _stream_ptr(stream)))
    return out


def device_error_take() -> int:
    w = C.c_int(0)
    N.check("ks_device_error_take", N.lib.ks_device_error_take(C.byref(w)))
    return w.value


def _copy(dst: torch.Tensor, src: torch.Tensor, stream) -> None:
    """One async copy through the C ABI (pinned host <-> device, either way)."""
    n = src.numel() * src.element_size()
    sp = _stream_ptr(stream)
    if dst.is_cuda:
        N.check("ks_gpu_memcpy_htod", N.lib.ks_gpu_memcpy_htod(C.c_void_p(dst.data_ptr()),
                                                               C.c_void_p(src.data_ptr()), n, sp))
    else:
        N.check("ks_gpu_memcpy_dtoh", N.lib.ks_gpu_memcpy_dtoh(C.c_void_p(dst.data_ptr()),
                                                               C.c_void_p(src.data_ptr()), n, sp))


class HostRowPipeline:
    """Row-wise families on host-resident data: rows move in chunks through
    three streams -- host-to-device copy, kernel, device-to-host copy -- so the
    copy of one chunk's input, the kernel on the previous chunk and the copy
    of an earlier chunk's output overlap (PCIe moves both directions at once).

    ``step(host_in, dev_in, host_out, dev_out, launch)`` runs one pass over all
    rows: ``host_in`` / ``dev_in`` are matching [rows, ...] tensors (pinned
    host, device), ``launch(r0, r1, stream)`` enqueues the family on rows
    [r0, r1) of the device tensors, and the result lands in ``host_out``.
    Consecutive steps pipeline as well; a chunk's device buffers are reused
    only after the previous step's kernel and output copy are done with them.
    Returns an event that completes when this step's output is on the host.

    The default is two chunks per step: because consecutive steps pipeline,
    larger chunks lose nothing to filling the pipeline and pay the per-copy
    cost less often (measured on B200 for softmax 4096x8192 over 20 steps:
    95.1 GB/s with 2 chunks, 92.7 with 4, 87.4 with 8, 79.6 with 16, against
    98 GB/s of bidirectional PCIe copy).
    """

    def __init__(self, rows: int, chunk_rows: int | None = None):
        if chunk_rows is None:
            chunk_rows = (rows + 1) // 2
        self.chunks = [(r, min(rows, r + chunk_rows)) for r in range(0, rows, max(1, chunk_rows))]
        self.s_in, self.s_k, self.s_out = (torch.cuda.Stream() for _ in range(3))
        self.ev_k = [None] * len(self.chunks)
        self.ev_out = [None] * len(self.chunks)

    def step(self, host_in, dev_in, host_out, dev_out, launch):
        for i, (r0, r1) in enumerate(self.chunks):
            if self.ev_k[i] is not None:
                self.s_in.wait_event(self.ev_k[i])  # the last step's kernel has read this chunk
            for h, d in zip(host_in, dev_in):
                _copy(d[r0:r1], h[r0:r1], self.s_in)
            e_in = torch.cuda.Event()
            e_in.record(self.s_in)
            self.s_k.wait_event(e_in)
            if self.ev_out[i] is not None:
                self.s_k.wait_event(self.ev_out[i])  # the last step's output copy has read this chunk
            launch(r0, r1, self.s_k)
            self.ev_k[i] = torch.cuda.Event()
            self.ev_k[i].record(self.s_k)
            self.s_out.wait_event(self.ev_k[i])
            _copy(host_out[r0:r1], dev_out[r0:r1], self.s_out)
            self.ev_out[i] = torch.cuda.Event()
            self.ev_out[i].record(self.s_out)
        return self.ev_out[-1]

    def join(self, stream=None) -> None:
        """Make `stream` (default: current) wait for everything enqueued."""
        s = stream if stream is not None else torch.cuda.current_stream()
        for st in (self.s_in, self.s_k, self.s_out):
            s.wait_stream(st)
