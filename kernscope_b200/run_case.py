"""Run one family's kernel a fixed number of times at one shape (for profilers).

    python -m kernscope_b200.run_case --family softmax --shape 4096,8192 --launches 4
    python -m kernscope_b200.run_case --family flash_attention --shape 1,32,8192,128 --causal

Inputs are seeded device tensors with the benchmark distributions; each
launch goes through the C ABI with the family's default sm_100a config (or
--config as JSON with the config struct's fields).  Exits 0 after a device
synchronize, so a profiler can capture e.g. the last launch with
``-s <launches-1> -c 1``.
"""

from __future__ import annotations

import argparse
import json
import math
import sys


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--family", required=True,
                    choices=("softmax", "layernorm", "bias_gelu", "reduction", "matmul", "flash_attention"))
    ap.add_argument("--shape", required=True, help="softmax/layernorm/bias_gelu R,C; reduction N (full sum) or "
                    "R,C (axis 0); matmul M,N,K; flash_attention B,H,N,d")
    ap.add_argument("--launches", type=int, default=4)
    ap.add_argument("--causal", action="store_true")
    ap.add_argument("--gelu", default="tanh", choices=("erf", "tanh"))
    ap.add_argument("--config", default=None, help="config struct fields as JSON")
    a = ap.parse_args(argv)
    shape = [int(v) for v in a.shape.split(",")]

    import torch

    from . import native as N
    from . import ops

    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    rn = lambda *s: torch.randn(*s, generator=g, device="cuda")  # noqa: E731
    cfg_fields = json.loads(a.config) if a.config else None

    def mk(cls):
        return cls(**cfg_fields) if cfg_fields else None

    f = a.family
    if f == "softmax":
        x = (rn(*shape) * 2).bfloat16()
        y = torch.empty_like(x)
        run = lambda: ops.softmax(x, out=y, cfg=mk(N.SoftmaxConfig))  # noqa: E731
    elif f == "layernorm":
        x = rn(*shape).bfloat16()
        gm, bt = (1 + 0.1 * rn(shape[1])).bfloat16(), (0.1 * rn(shape[1])).bfloat16()
        y = torch.empty_like(x)
        run = lambda: ops.layernorm(x, gm, bt, out=y, cfg=mk(N.LayerNormConfig))  # noqa: E731
    elif f == "bias_gelu":
        x = rn(*shape).bfloat16()
        b = (0.1 * rn(shape[1])).bfloat16()
        y = torch.empty_like(x)
        run = lambda: ops.bias_gelu(x, b, gelu=a.gelu, out=y, cfg=mk(N.BiasGeluConfig))  # noqa: E731
    elif f == "reduction":
        if len(shape) == 1:
            x = torch.rand(shape[0], generator=g, device="cuda")
            axis = -1
        else:
            x = rn(*shape).bfloat16()
            axis = 0
        cfg = mk(N.ReductionConfig)
        ws = ops.reduction_workspace(x, axis=axis, cfg=cfg)
        run = lambda: ops.reduction(x, axis=axis, cfg=cfg, workspace=ws)  # noqa: E731
    elif f == "matmul":
        m, n, k = shape
        s = 1.0 / math.sqrt(k)
        am, bm = (rn(m, k) * s).bfloat16(), (rn(k, n) * s).bfloat16()
        c = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
        run = lambda: ops.matmul(am, bm, out=c, cfg=mk(N.MatmulConfig))  # noqa: E731
    else:
        q, k, v = (rn(*shape).bfloat16() for _ in range(3))
        o = torch.empty_like(q)
        run = lambda: ops.flash_attention(q, k, v, causal=a.causal, out=o, cfg=mk(N.FlashAttentionConfig))  # noqa: E731
    for _ in range(a.launches):
        run()
    torch.cuda.synchronize()
    print(f"ok {f} {a.shape} x{a.launches}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
