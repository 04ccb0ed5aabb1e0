"""Run one family's kernel a fixed number of times at one shape (for profilers).

    python -m kernscope_b200.run_case --family softmax --shape 4096,8192 --launches 4
    python -m kernscope_b200.run_case --family flash_attention --shape 1,32,8192,128 --causal

Inputs are seeded device tensors with the benchmark distributions; each
launch goes through the C ABI with the family's default sm_100a config (or
--config as JSON with the config struct's fields).  ``--rotate R`` cycles the
launches through R input/output sets, as the benchmark does, so that a
launch neither finds its inputs in L2 nor overwrites its own dirty outputs
there: the DRAM bytes of a later launch then include the write-back of the
earlier launches' outputs, the steady state of a loop.  Exits 0 after a
device synchronize, so a profiler can capture e.g. the last launch with
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
    ap.add_argument("--rotate", type=int, default=1, help="input/output sets the launches cycle through")
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
    R = max(1, a.rotate)
    if f == "softmax":
        xs = [(rn(*shape) * 2).bfloat16() for _ in range(R)]
        ys = [torch.empty_like(xs[0]) for _ in range(R)]
        run = lambda i: ops.softmax(xs[i % R], out=ys[i % R], cfg=mk(N.SoftmaxConfig))  # noqa: E731
    elif f == "layernorm":
        xs = [rn(*shape).bfloat16() for _ in range(R)]
        gm, bt = (1 + 0.1 * rn(shape[1])).bfloat16(), (0.1 * rn(shape[1])).bfloat16()
        ys = [torch.empty_like(xs[0]) for _ in range(R)]
        run = lambda i: ops.layernorm(xs[i % R], gm, bt, out=ys[i % R], cfg=mk(N.LayerNormConfig))  # noqa: E731
    elif f == "bias_gelu":
        xs = [rn(*shape).bfloat16() for _ in range(R)]
        b = (0.1 * rn(shape[1])).bfloat16()
        ys = [torch.empty_like(xs[0]) for _ in range(R)]
        run = lambda i: ops.bias_gelu(xs[i % R], b, gelu=a.gelu, out=ys[i % R],  # noqa: E731
                                      cfg=mk(N.BiasGeluConfig))
    elif f == "reduction":
        if len(shape) == 1:
            xs = [torch.rand(shape[0], generator=g, device="cuda") for _ in range(R)]
            axis = -1
        else:
            xs = [rn(*shape).bfloat16() for _ in range(R)]
            axis = 0
        cfg = mk(N.ReductionConfig)
        ws = ops.reduction_workspace(xs[0], axis=axis, cfg=cfg)
        run = lambda i: ops.reduction(xs[i % R], axis=axis, cfg=cfg, workspace=ws)  # noqa: E731
    elif f == "matmul":
        m, n, k = shape
        s = 1.0 / math.sqrt(k)
        am, bm = (rn(m, k) * s).bfloat16(), (rn(k, n) * s).bfloat16()
        c = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
        run = lambda i: ops.matmul(am, bm, out=c, cfg=mk(N.MatmulConfig))  # noqa: E731
    else:
        q, k, v = (rn(*shape).bfloat16() for _ in range(3))
        o = torch.empty_like(q)
        run = lambda i: ops.flash_attention(q, k, v, causal=a.causal, out=o,  # noqa: E731
                                            cfg=mk(N.FlashAttentionConfig))
    for i in range(a.launches):
        run(i)
    torch.cuda.synchronize()
    print(f"ok {f} {a.shape} x{a.launches}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
