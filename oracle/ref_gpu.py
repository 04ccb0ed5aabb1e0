"""The reference generator's own kernels on this GPU (test infrastructure only).

``oracle/ref_tune/build_ref_kernels.py`` builds, for every config of the
reference tuner's bounded "auto" grid at the benchmark shapes, one shared
library holding the generated kernel and a launcher (``ks_ref_launch``). This
module launches them the way the reference's gate runner does
(``kernels/templates/tools/hip_template_runner.cpp``: the kernel's own
argument order, the grid and block from the generator's
``launch_geometry``), checks each config's output against the oracle on
sampled rows (the reference tuner discards configs that fail its gate), and
times the survivors with CUDA events after an L2 flush, median of the
repetitions (the reference's libs/bench methodology).

Only ``bench.py --impl reference`` and the GPU tests use it; nothing of the
product path does.
"""

from __future__ import annotations

import ctypes
import json
import os
import statistics

import numpy as np

from oracle import metrics as om
from oracle import refs as orf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "oracle", "_ref")
INDEX = os.path.join(REF_DIR, "kernels", "index.json")

FAMILIES = ("softmax", "layernorm", "bias_gelu", "matmul", "flash_attention")


def index() -> list | None:
    if not os.path.exists(INDEX):
        return None
    with open(INDEX) as f:
        return json.load(f)


class RefKernel:
    """One generated kernel: ``launch(args)`` with args in the kernel's order
    (device pointers as ints, then the int32 scalars)."""

    def __init__(self, entry: dict):
        self.entry = entry
        self.lib = ctypes.CDLL(os.path.join(REF_DIR, entry["lib"]), mode=os.RTLD_LOCAL)
        self.fn = self.lib.ks_ref_launch
        self.fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        self.fn.restype = ctypes.c_int

    def launch(self, ptrs: list[int], ints: list[int], stream: int = 0) -> None:
        vals = [ctypes.c_void_p(p) for p in ptrs] + [ctypes.c_int(v) for v in ints]
        arr = (ctypes.c_void_p * len(vals))(*[ctypes.cast(ctypes.pointer(v), ctypes.c_void_p) for v in vals])
        gx, gy = (int(v) for v in self.entry["grid"])  # the index's JSON numbers may be written as floats
        bx, by = (int(v) for v in self.entry["block"])
        rc = self.fn(arr, gx, gy, bx, by, ctypes.c_void_p(stream))
        if rc != 0:
            raise RuntimeError(f"reference kernel launch failed ({rc}) for {self.entry['config']}")


def _inputs(family: str, shape, dev):
    """Seeded device inputs with the benchmark's distributions, and the
    kernel's (pointers, ints, output)."""
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(7)

    def normal(*s, std=1.0, mean=0.0):
        return (torch.randn(*s, generator=g, device=dev) * std + mean).to(torch.bfloat16)

    if family == "softmax":
        r, c = shape
        x = normal(r, c, std=2.0)
        out = torch.empty_like(x)
        return dict(x=x), [x.data_ptr(), out.data_ptr()], [r, c], out
    if family == "layernorm":
        r, c = shape
        x, gm, bt = normal(r, c), normal(c, std=0.1, mean=1.0), normal(c, std=0.1)
        out = torch.empty_like(x)
        return dict(x=x, gamma=gm, beta=bt), [x.data_ptr(), gm.data_ptr(), bt.data_ptr(), out.data_ptr()], [r, c], out
    if family == "bias_gelu":
        r, c = shape
        x, b = normal(r, c), normal(c, std=0.1)
        out = torch.empty_like(x)
        return dict(x=x, bias=b), [x.data_ptr(), b.data_ptr(), out.data_ptr()], [r * c, c], out
    if family == "matmul":
        m, n, k = shape
        a, b = normal(m, k, std=k ** -0.5), normal(k, n, std=k ** -0.5)
        out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        return dict(a=a, b=b), [a.data_ptr(), b.data_ptr(), out.data_ptr()], [m, n, k], out
    raise KeyError(family)


def _expected(family: str, t: dict, rows) -> np.ndarray:
    """The oracle's output for the sampled rows."""
    f = lambda z: z.float().cpu().numpy()  # noqa: E731  (bf16 values, exactly in fp32)
    if family == "softmax":
        exp = orf.softmax(f(t["x"][rows]))
    elif family == "layernorm":
        exp = orf.layernorm(f(t["x"][rows]), f(t["gamma"]), f(t["beta"]))
    elif family == "bias_gelu":
        exp = orf.bias_gelu(f(t["x"][rows]), f(t["bias"]))  # the reference's exact-erf GELU
    else:
        exp = orf.matmul(f(t["a"][rows]), f(t["b"]))
    return np.asarray(exp, dtype=np.float32)


def run_family(family: str, reps: int = 3, dev: str = "cuda:0") -> dict:
    """Check and time every built config of one family at its benchmark
    shape; the best passing config's throughput is the family's figure."""
    import torch

    entries = [e for e in (index() or []) if e["family"] == family]
    if not entries:
        return {"unavailable": "reference kernels not built (oracle/ref_tune/build_ref_kernels.py)"}
    if not any("lib" in e for e in entries):
        reasons = sorted({e.get("rejected", "")[:60] for e in entries})
        return {"unavailable": f"none of the {len(entries)} auto-grid configs builds for CUDA", "reasons": reasons}
    shape = entries[0]["shape"]
    t, ptrs, ints, out = _inputs(family, shape, dev)
    lead = shape[0]
    rows = sorted({0, 1, lead // 3, lead // 2, lead - 1})
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > L2
    if family == "matmul":
        m, n, k = shape
        work, unit = 2.0 * m * n * k / 1e12, "TFLOP/s"
    else:
        nbytes = {"softmax": 4, "layernorm": 4, "bias_gelu": 4}[family] * shape[0] * shape[1]
        work, unit = nbytes / 1e9, "GB/s"
    exp = _expected(family, t, rows)
    results = []
    for e in entries:
        if "lib" not in e:
            results.append({"config": e["config"], "rejected": e.get("rejected", "not built")})
            continue
        kern = RefKernel(e)
        out.zero_()
        kern.launch(ptrs, ints)
        torch.cuda.synchronize()
        err = om.floor_rel_err(out[rows].float().cpu().numpy(), exp)
        if not (err["norm"] <= 1e-2):
            results.append({"config": e["config"], "gate_failed": err})
            continue
        ms = []
        for _ in range(reps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            kern.launch(ptrs, ints)
            e1.record()
            e1.synchronize()
            ms.append(e0.elapsed_time(e1))
        med = statistics.median(ms)
        results.append({"config": e["config"], "median_ms": round(med, 4), "value": round(work / (med / 1e3), 2)})
    timed = [r for r in results if "value" in r]
    if not timed:
        worst = min((r["gate_failed"]["norm"] for r in results if "gate_failed" in r), default=None)
        return {"unavailable": "no reference config passed the gate", "configs_built": len(results),
                "best_norm_err": worst}
    best = max(timed, key=lambda r: r["value"])
    return {"value": best["value"], "unit": unit, "shape": shape, "best_config": best["config"],
            "median_ms": best["median_ms"], "configs_timed": len(timed),
            "configs_rejected": len(results) - len(timed),
            "rejections": sorted({r.get("rejected", "gate failed")[:80] for r in results if "value" not in r})}
