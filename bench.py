"""Benchmark of the kernscope-tune hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                    [--impl kernscope|reference] [--no-families]

Metric: "bf16 TFLOP/s & HBM GB/s per kernel family as % of
B200 roofline, 1/2/4/8 GPU".  The headline workload is configuration C2,
row softmax of 4096 x 8192 bf16 (HBM GB/s of algorithmic bytes: 2 B read +
2 B written per element); the JSON line also carries, under "families", the
same measurement for every other family at its benchmark configuration.

A step is one launch of the family's kernel over one batch, through the C ABI
(``ks_<family>_launch``).  ``value`` is whole-job throughput with inputs
resident in HBM; ``e2e`` is the same metric through the same C ABI with the
inputs copied from pinned host memory and the outputs copied back inside the
timed region.  Multi-GPU (torchrun): the headline is weak scaling by default
(every rank runs one full batch of the configuration on its own GPU: rows /
M-panels / heads / elements of a G-times larger job), and every family also
reports strong scaling under "strong": the one configuration sharded over
the G GPUs (rows, elements, M-panels with B replicated, batch x head pairs),
with efficiency t1 / (G * t_G) against the whole configuration's time on
one GPU in the same run.  ``--scaling strong`` makes the sharded
configuration the headline.  The reduction adds its one cross-GPU combine
(an NCCL all-reduce of the fp64 partials, one call per eight consecutive
jobs) to every job.  Time = max over
ranks of CUDA-event time, barrier + synchronize on both sides, after an
untimed pre-roll that brings the clocks back up after the barrier.

Inputs are synthetic (seeded torch RNG on the device) with the
configurations' shapes and distributions.  Between timed steps the input
buffers rotate through enough copies that the working set is >= 4x the L2,
so no step reads its inputs from L2.
"""

from __future__ import annotations

import argparse
import ctypes as C
import json
import math
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def _traffic_table():
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as fh:
            return json.load(fh)
    return {}


# ---------------------------------------------------------------------------
# Workloads: per-rank shapes of the benchmark configurations
# ---------------------------------------------------------------------------
WORKLOADS = {
    "softmax": {"config": "C2", "shape": (4096, 8192), "bound": "hbm", "dtype": "bf16",
                "desc": "row softmax 4096x8192 bf16, x~N(0,2^2)"},
    "layernorm": {"config": "C3a", "shape": (16384, 4096), "bound": "hbm", "dtype": "bf16",
                  "desc": "layernorm 16384x4096 bf16, gamma~N(1,0.1), beta~N(0,0.1), eps 1e-5"},
    "bias_gelu": {"config": "C3b", "shape": (16384, 16384), "bound": "hbm", "dtype": "bf16",
                  "desc": "bias_gelu (tanh) 16384x16384 bf16, bias[16384]"},
    "bias_gelu_erf": {"config": "C3b", "shape": (16384, 16384), "bound": "hbm", "dtype": "bf16",
                      "desc": "bias_gelu (exact erf, the reference's GELU) 16384x16384 bf16, bias[16384]"},
    "reduction": {"config": "C3c", "shape": (1 << 28,), "bound": "hbm", "dtype": "f32",
                  "desc": "full fp32 sum of 2^28 uniform[0,1) (fp64 partials, NCCL combine for N>1)"},
    "matmul": {"config": "C4", "shape": (8192, 8192, 8192), "bound": "tensor", "dtype": "bf16",
               "desc": "GEMM 8192^3 bf16, fp32 accumulate, A,B~N(0,1/sqrt(K))"},
    "matmul_65536": {"config": "C4", "shape": (65536, 8192, 8192), "bound": "tensor", "dtype": "bf16",
                     "desc": "GEMM 65536x8192x8192 bf16"},
    "flash_attention": {"config": "C5", "shape": (8, 32, 8192, 128), "bound": "tensor", "dtype": "bf16",
                        "desc": "flash attention fwd causal B8 H32 N8192 d128 bf16"},
}


# the row-wise families: rows shard, and the end-to-end leg pipelines row chunks
ROW_FAMILIES = ("softmax", "layernorm", "bias_gelu", "bias_gelu_erf")


class Workload:
    """Device buffers + launch closure for one family at one per-rank shape."""

    def __init__(self, name, shape, rank, world, seed_base=0):
        import torch

        from kernscope_b200 import native as N
        from kernscope_b200 import ops

        self.name, self.shape, self.N, self.ops = name, shape, N, ops
        self.torch = torch
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev)
        g.manual_seed(1000 * rank + seed_base + 17)
        self.gen, self.dev = g, dev
        self.extra = {}
        if name == "softmax":
            r, c = shape
            self.in_bytes, self.out_bytes = r * c * 2, r * c * 2
            self.alg_bytes, self.flops = r * c * 4, 0
            self.make = lambda: [(torch.randn((r, c), generator=g, device=dev) * 2.0).to(torch.bfloat16)]
            self.outs = lambda: [torch.empty((r, c), dtype=torch.bfloat16, device=dev)]
            self.cfg = ops.default_softmax_config(c)
        elif name == "layernorm":
            r, c = shape
            self.in_bytes, self.out_bytes = r * c * 2 + 2 * c * 2, r * c * 2
            self.alg_bytes, self.flops = r * c * 4 + 2 * c * 2, 0
            gamma = (1.0 + 0.1 * torch.randn(c, generator=g, device=dev)).to(torch.bfloat16)
            beta = (0.1 * torch.randn(c, generator=g, device=dev)).to(torch.bfloat16)
            self.make = lambda: [torch.randn((r, c), generator=g, device=dev).to(torch.bfloat16), gamma, beta]
            self.outs = lambda: [torch.empty((r, c), dtype=torch.bfloat16, device=dev)]
            self.cfg = ops.default_layernorm_config(c)
        elif name in ("bias_gelu", "bias_gelu_erf"):
            r, c = shape
            self.gelu = "erf" if name == "bias_gelu_erf" else "tanh"
            self.in_bytes, self.out_bytes = r * c * 2 + c * 2, r * c * 2
            self.alg_bytes, self.flops = r * c * 4 + c * 2, 0
            bias = (0.1 * torch.randn(c, generator=g, device=dev)).to(torch.bfloat16)
            self.make = lambda: [torch.randn((r, c), generator=g, device=dev).to(torch.bfloat16), bias]
            self.outs = lambda: [torch.empty((r, c), dtype=torch.bfloat16, device=dev)]
            self.cfg = ops.default_bias_gelu_config(c, self.gelu)
            self.extra["reference_model_bytes"] = r * c * 2 * 3
        elif name == "reduction":
            (n,) = shape
            self.in_bytes, self.out_bytes = n * 4, 4
            self.alg_bytes, self.flops = n * 4 + 4, 0
            self.make = lambda: [torch.rand(n, generator=g, device=dev)]
            self.outs = lambda: [torch.empty(1, dtype=torch.float32, device=dev),
                                 torch.empty(1, dtype=torch.float64, device=dev)]
            self.cfg = ops.default_reduction_config(n, -1)
        elif name.startswith("matmul"):
            m, n, k = shape
            self.in_bytes, self.out_bytes = (m * k + k * n) * 2, m * n * 2
            self.alg_bytes, self.flops = (m * k + k * n + m * n) * 2, 2 * m * n * k
            sig = 1.0 / math.sqrt(k)
            bmat = (torch.randn((k, n), generator=g, device=dev) * sig).to(torch.bfloat16)
            self.make = lambda: [(torch.randn((m, k), generator=g, device=dev) * sig).to(torch.bfloat16), bmat]
            self.outs = lambda: [torch.empty((m, n), dtype=torch.bfloat16, device=dev)]
            self.cfg = ops.default_matmul_config(m, n, k)
        elif name == "flash_attention":
            b, h, s, d = shape
            self.in_bytes, self.out_bytes = 3 * b * h * s * d * 2, b * h * s * d * 2
            self.alg_bytes = 4 * b * h * s * d * 2
            self.flops = 4 * d * b * h * s * (s + 1) // 2  # causal count
            self.make = lambda: [torch.randn((b, h, s, d), generator=g, device=dev).to(torch.bfloat16)
                                 for _ in range(3)]
            self.outs = lambda: [torch.empty((b, h, s, d), dtype=torch.bfloat16, device=dev)]
            self.cfg = ops.default_flash_attention_config(True)
        else:
            raise KeyError(name)
        footprint = self.in_bytes + self.out_bytes
        self.rotate = 1 if footprint >= 4 * L2_BYTES else int(math.ceil(4 * L2_BYTES / footprint))
        self.sets = [(self.make(), self.outs()) for _ in range(self.rotate)]
        self.ws = None
        if name == "reduction":
            self.ws = ops.reduction_workspace(self.sets[0][0][0], axis=-1, cfg=self.cfg)
            # fp64 partials in two rows of COMBINE_BATCH steps: at N > 1 one
            # all-reduce combines a row (the cross-GPU sums of that many
            # consecutive jobs) while the next row's kernels run
            self.partials = torch.empty((2, COMBINE_BATCH), dtype=torch.float64, device=dev)

    def launch(self, i, stream=None, slot=None):
        ins, outs = self.sets[i % self.rotate]
        ops = self.ops
        if self.name == "softmax":
            ops.softmax(ins[0], out=outs[0], cfg=self.cfg, stream=stream)
        elif self.name == "layernorm":
            ops.layernorm(ins[0], ins[1], ins[2], out=outs[0], cfg=self.cfg, stream=stream)
        elif self.name.startswith("bias_gelu"):
            ops.bias_gelu(ins[0], ins[1], gelu=self.gelu, out=outs[0], cfg=self.cfg, stream=stream)
        elif self.name == "reduction":
            ops.reduction(ins[0], axis=-1, out=outs[0], cfg=self.cfg, workspace=self.ws,
                          partial_f64=self.partials.view(-1)[slot if slot is not None else 0],
                          stream=stream)
        elif self.name.startswith("matmul"):
            ops.matmul(ins[0], ins[1], out=outs[0], cfg=self.cfg, stream=stream)
        else:
            ops.flash_attention(ins[0], ins[1], ins[2], causal=True, out=outs[0], cfg=self.cfg, stream=stream)

    def config_name(self):
        return self.N.kernel_symbol("flash_attention" if self.name == "flash_attention" else
                                    "matmul" if self.name.startswith("matmul") else
                                    "bias_gelu" if self.name.startswith("bias_gelu") else self.name, self.cfg)


# ---------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() in ("active", "1"):
                    reasons.add(nm)
        sm.sort()
        med = sm[len(sm) // 2] if sm else None
        return {"sm_mhz": med, "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
def _dist_setup(args):
    import torch

    from kernscope_b200 import dist

    rank, world, local = dist.setup(backend="nccl", timeout_s=120)
    if world == 1:
        torch.cuda.set_device(0)
    return rank, world, local


def _barrier(world):
    from kernscope_b200 import dist

    dist.barrier(world)


def _max_over_ranks(v, world):
    from kernscope_b200 import dist

    return dist.max_over_ranks(v, world, device="cuda")


def _combine(w, world):
    """The reduction's cross-GPU combine of one job: all-reduce of its fp64
    partial (slot 0, where ``launch`` writes it by default)."""
    if world > 1 and w.name == "reduction":
        from kernscope_b200 import dist

        dist.combine_partials(w.partials[0, :1], world)


# Consecutive full-sum jobs whose fp64 partials one all-reduce combines at
# N > 1.  An all-reduce of a few bytes costs tens of microseconds of NCCL
# latency on eight GPUs, more than one 2^25-element shard's kernel; one call
# per COMBINE_BATCH jobs (a vector of that many partials) keeps that latency
# behind the kernels.  Every job still gets its own cross-GPU sum.
COMBINE_BATCH = 8


def _reduction_steps(w, steps, world, stream, first=0):
    """Steps first..first+steps-1 of the multi-GPU reduction.  Step j writes
    its fp64 partial into row (j // B) % 2, column j % B of ``w.partials``
    (B = COMBINE_BATCH); after the last step of each row one NCCL all-reduce
    of that row (the cross-GPU sums of its B jobs) runs on a side stream,
    overlapping the next row's kernels, and the row is rewritten only after
    that combine.  The caller's stream waits for every combine.  Used
    eagerly and inside a CUDA-graph capture alike; every rank issues the same
    collectives in the same order."""
    import torch

    from kernscope_b200 import dist

    side = getattr(w, "_side", None) or torch.cuda.Stream()
    w._side = side
    B = COMBINE_BATCH
    done = {}
    for j in range(steps):
        b, col = divmod(j, B)
        row = b % 2
        if col == 0 and b >= 2:
            stream.wait_event(done[b - 2])
        w.launch(first + j, stream=stream, slot=row * B + col)
        if col == B - 1 or j == steps - 1:
            k = torch.cuda.Event()
            k.record(stream)
            side.wait_event(k)
            with torch.cuda.stream(side):
                dist.combine_partials(w.partials[row, :col + 1], world, to_f32=False)
            c = torch.cuda.Event()
            c.record(side)
            done[b] = c
    for b in sorted(done)[-2:]:
        stream.wait_event(done[b])


def _enqueue(w, first, count, world, stream):
    """Launches first..first+count-1 (rotating buffer sets) on `stream`; the
    multi-GPU reduction with its overlapped, batched combines."""
    if world > 1 and w.name == "reduction":
        _reduction_steps(w, count, world, stream, first)
    else:
        for i in range(first, first + count):
            w.launch(i, stream=stream)


def measure_device(w, steps, warmup, world, graph=True, preroll_ms=3.0):
    """Timed region: `steps` launches on rotating buffers, CUDA events on the
    launching stream, max over ranks.

    The timed launches are captured in one CUDA graph (the multi-GPU
    reduction's graph holds its NCCL combines too), so host overhead never
    paces the GPU.  The barrier before the timed region idles the GPU, so a
    pre-roll graph of untimed launches (about `preroll_ms` of work, at least
    3) is replayed right after the barrier with no host sync before the
    start event: the clocks are back up when timing starts.  Every rank
    takes the same collective steps: the pre-roll length and the capture's
    success are agreed over ranks before any replay.  Returns
    (max-over-ranks ms, this rank's ms, timing label)."""
    import torch

    from kernscope_b200 import dist

    stream = torch.cuda.current_stream()
    cap = torch.cuda.Stream()
    # untimed warm-up, eager; its event time sizes the pre-roll
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    _enqueue(w, 0, warmup, world, stream)
    t1.record(stream)
    torch.cuda.synchronize()
    est = max(t0.elapsed_time(t1) / max(1, warmup), 1e-3)
    npre = int(_max_over_ranks(min(max(3, math.ceil(preroll_ms / est)), max(3, 4 * steps)), world))
    g = gp = None
    ok = 1.0
    if graph:
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                _enqueue(w, 0, steps, world, cap)
            gp = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gp, stream=cap):
                _enqueue(w, steps, npre, world, cap)
        except Exception:  # noqa: BLE001 - capture refused: every rank times eager launches instead
            ok = 0.0
        torch.cuda.synchronize()
        ok = -_max_over_ranks(-ok, world)  # min over ranks
        if ok < 1.0:
            g = gp = None
    label = "graph" if g is not None else "eager"
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier(world)
    if g is not None:
        gp.replay()
        e0.record(stream)
        g.replay()
    else:
        _enqueue(w, steps, npre, world, stream)
        e0.record(stream)
        _enqueue(w, 0, steps, world, stream)
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    _barrier(world)
    del g, gp
    dist.barrier(world)
    return _max_over_ranks(ms, world), ms, label


def _rank_spread(ms, world):
    """Per-rank timed-region ms of every rank (gathered), for the line's spread."""
    from kernscope_b200 import dist

    return dist.gather_values(ms, world, device="cuda")


def measure_e2e(w, steps, world):
    """Same metric through the public API with host buffers: every step
    copies its inputs from pinned host memory to the device, runs the family
    and copies the result back, all inside the timed region.  Row-wise
    families go through ``ops.HostRowPipeline`` (row chunks on three streams,
    so input and output copies overlap each other and the kernel); the rest
    copy, launch and copy back on one stream."""
    import torch

    from kernscope_b200 import ops

    ins, outs = w.sets[0]
    host_in = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in ins]
    for h, t in zip(host_in, ins):
        h.copy_(t)
    host_out = torch.empty(outs[0].shape, dtype=outs[0].dtype, pin_memory=True)
    stream = torch.cuda.current_stream()
    h2d = sum(t.numel() * t.element_size() for t in ins)
    d2h = outs[0].numel() * outs[0].element_size()

    if w.name in ROW_FAMILIES:
        rows = ins[0].shape[0]
        pipe = ops.HostRowPipeline(rows)
        row_in = [0]  # x is row-sharded; gamma/beta/bias stay whole
        h2d_whole = [(h, t) for k, (h, t) in enumerate(zip(host_in, ins)) if k not in row_in]

        def launch(r0, r1, st):
            x, y = ins[0][r0:r1], outs[0][r0:r1]
            if w.name == "softmax":
                ops.softmax(x, out=y, cfg=w.cfg, stream=st)
            elif w.name == "layernorm":
                ops.layernorm(x, ins[1], ins[2], out=y, cfg=w.cfg, stream=st)
            else:
                ops.bias_gelu(x, ins[1], gelu=w.gelu, out=y, cfg=w.cfg, stream=st)

        def step():
            if h2d_whole and pipe.ev_k[-1] is not None:
                pipe.s_in.wait_event(pipe.ev_k[-1])  # the last step's kernels are done with them
            for h, t in h2d_whole:  # the per-column vectors, once per step
                ops._copy(t, h, pipe.s_in)
            pipe.step([host_in[0]], [ins[0]], host_out, outs[0], launch)

        def finish():
            pipe.join(stream)
    else:
        def step():
            for h, t in zip(host_in, ins):
                ops._copy(t, h, stream)
            w.launch(0)
            _combine(w, world)
            ops._copy(host_out, outs[0], stream)

        def finish():
            pass

    step()
    finish()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier(world)
    e0.record(stream)
    if w.name in ROW_FAMILIES:
        pipe.s_in.wait_stream(stream)  # the copies start after the start event
    for _ in range(steps):
        step()
    finish()
    e1.record(stream)
    e1.synchronize()
    ms = _max_over_ranks(e0.elapsed_time(e1), world)
    _barrier(world)
    return ms, h2d, d2h


def _units(w, bound):
    return (w.flops / 1e12, "TFLOP/s") if bound == "tensor" else (w.alg_bytes / 1e9, "GB/s")


def cpu_baseline(name, shape, budget_s=10.0):
    """The CPU oracle (numpy port of the reference's refs.py) on one core, on
    a bounded sample of the workload; returns the metric in its unit."""
    import numpy as np

    from oracle import inputs as oin
    from oracle import refs as orf

    t_total, units, sample = 0.0, 0.0, ""
    rows = 1
    while t_total < budget_s:
        if name == "softmax":
            r, c = shape
            x = oin.baseline_inputs("softmax", shape, seed=1, row0=0, nrows=min(rows, r))["x"]
            t0 = time.perf_counter(); orf.softmax(x); dt = time.perf_counter() - t0
            u = x.shape[0] * c * 4 / 1e9; sample = f"{x.shape[0]} of {r} rows"
        elif name == "layernorm":
            r, c = shape
            d = oin.baseline_inputs("layernorm", shape, seed=2, row0=0, nrows=min(rows, r))
            t0 = time.perf_counter(); orf.layernorm(d["x"], d["gamma"], d["beta"]); dt = time.perf_counter() - t0
            u = d["x"].shape[0] * c * 4 / 1e9; sample = f"{d['x'].shape[0]} of {r} rows"
        elif name.startswith("bias_gelu"):
            r, c = shape
            d = oin.baseline_inputs("bias_gelu", shape, seed=2, row0=0, nrows=min(rows, r))
            fn = orf.bias_gelu if name == "bias_gelu_erf" else orf.bias_gelu_tanh
            t0 = time.perf_counter(); fn(d["x"], d["bias"]); dt = time.perf_counter() - t0
            u = d["x"].shape[0] * c * 4 / 1e9; sample = f"{d['x'].shape[0]} of {r} rows"
        elif name == "reduction":
            (n,) = shape
            cnt = min(rows * 65536, n)
            x = oin.baseline_inputs("reduction_full", shape, seed=2, row0=0, nrows=cnt)["x"]
            t0 = time.perf_counter(); orf.sum_full_f64(x); dt = time.perf_counter() - t0
            u = cnt * 4 / 1e9; sample = f"{cnt} of {n} elements"
        elif name.startswith("matmul"):
            m, n, k = shape
            d = oin.baseline_inputs("matmul", (m, n, k), seed=3, row0=0, nrows=min(rows * 8, m))
            t0 = time.perf_counter(); orf.matmul(d["a"], d["b"]); dt = time.perf_counter() - t0
            u = 2 * d["a"].shape[0] * n * k / 1e12; sample = f"{d['a'].shape[0]} of {m} rows (BLAS threads: numpy default)"
        else:
            b, h, s, dd = shape
            nq = min(rows * 64, s)
            d = oin.baseline_inputs("attention", (b, h, s, s, dd), seed=4, row0=0, nrows=1)
            t0 = time.perf_counter(); orf.attention(d["q"][0, s - nq:], d["k"][0], d["v"][0], causal=False)
            dt = time.perf_counter() - t0
            # the last nq query rows attend to (almost) every key under the causal mask
            u = 4 * dd * nq * s / 1e12; sample = f"last {nq} query rows of 1 of {b*h} heads"
        t_total += dt
        units += u
        rows *= 2
    return units / t_total, sample


def measure_strong(nm, args, rank, world, t1_ms):
    """Strong scaling of one fixed configuration: every rank takes its shard
    of the one job (``dist.strong_shard``: rows, elements, M-panels with B
    replicated, or batch x head pairs) and the job's time is the slowest
    rank's.  `t1_ms` is the per-step time of the whole configuration on one
    GPU, measured in the same run (the weak measurement, max over ranks), so
    efficiency = t1 / (G * t_G).  The step count keeps the timed region near
    2 ms or more."""
    import torch

    from kernscope_b200 import dist

    spec = WORKLOADS[nm]
    shard, desc = dist.strong_shard(nm, spec["shape"], rank, world)
    w = Workload(nm, shard, rank, world, seed_base=7)
    steps = int(min(4000, max(int(args.family_steps), math.ceil(2.0 / max(t1_ms / world, 1e-3)))))
    steps = int(_max_over_ranks(steps, world))
    ms, my_ms, label = measure_device(w, steps, 3, world)
    per = ms / steps
    u_full = _job_units(nm, spec["shape"], spec["bound"])
    out = {"shape_per_gpu": list(shard), "shard": desc, "steps": steps, "ms_per_step": round(per, 5),
           "value": round(u_full / (per / 1e3), 2), "t1_ms_per_step": round(t1_ms, 5),
           "efficiency": round(t1_ms / (world * per), 4),
           "rank_ms_per_step": [round(v / steps, 5) for v in _rank_spread(my_ms, world)], "timing": label}
    del w
    torch.cuda.empty_cache()
    return out


def _job_units(nm, shape, bound):
    """Work units (TFLOP or GB of algorithmic traffic) of one step of the
    configuration at `shape`."""
    if nm in ("softmax",):
        r, c = shape
        b = r * c * 4
    elif nm == "layernorm":
        r, c = shape
        b = r * c * 4 + 2 * c * 2
    elif nm.startswith("bias_gelu"):
        r, c = shape
        b = r * c * 4 + c * 2
    elif nm == "reduction":
        b = shape[0] * 4 + 4
    elif nm.startswith("matmul"):
        m, n, k = shape
        return 2 * m * n * k / 1e12
    else:
        bb, h, s, d = shape
        return 4 * d * bb * h * s * (s + 1) // 2 / 1e12
    return b / 1e9


def run_families(names, args, rank, world):
    out = {}
    peaks = _peaks()
    traffic = _traffic_table()
    for nm in names:
        spec = WORKLOADS[nm]
        try:
            w = Workload(nm, spec["shape"], rank, world)
        except Exception as exc:  # noqa: BLE001 - report, keep the other families
            out[nm] = {"error": str(exc)[:200]}
            continue
        try:
            w.launch(0)
        except Exception as exc:  # noqa: BLE001
            out[nm] = {"error": str(exc)[:200]}
            del w
            continue
        steps = max(3, int(args.family_steps))
        ms, my_ms, label = measure_device(w, steps, 3, world)
        per = ms / steps
        u, unit = _units(w, spec["bound"])
        val = u * world / (per / 1e3)
        peak = peaks["hbm_gbs"] if spec["bound"] == "hbm" else peaks["bf16_tflops"]
        ach = u / (per / 1e3)
        out[nm] = {"config": spec["config"], "workload": spec["desc"], "kernel": w.config_name(),
                   "value": round(val, 2), "unit": unit, "ms_per_step": round(per, 5), "timing": label,
                   "roofline": {"bound": spec["bound"], "achieved": round(ach, 2), "peak": peak, "unit": unit,
                                "frac": round(ach / peak, 4), "traffic": traffic.get(nm)}}
        if spec["bound"] == "tensor":
            # the timed region is steps x ms_per_step of back-to-back launches under the
            # power cap: the sustained cuBLAS figure is the like-for-like denominator
            out[nm]["roofline"]["peak_sustained"] = peaks["bf16_tflops_sustained"]
            out[nm]["roofline"]["frac_sustained"] = round(ach / peaks["bf16_tflops_sustained"], 4)
        if world > 1:
            out[nm]["rank_ms_per_step"] = [round(v / steps, 5) for v in _rank_spread(my_ms, world)]
        del w
        import torch

        torch.cuda.empty_cache()
        if world > 1 and not args.no_strong:
            try:
                out[nm]["strong"] = measure_strong(nm, args, rank, world, per)
            except Exception as exc:  # noqa: BLE001
                out[nm]["strong"] = {"error": str(exc)[:200]}
    return out


def _ref_worker_init():
    # one BLAS thread per process: the pool itself uses every core
    for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[var] = "1"


# Rows (matmul: A rows; attention: query rows; reduction: 64K-element blocks)
# per worker per step, sized to ~0.1-0.5 s of numpy work on one core.
REF_CHUNK = {"softmax": 256, "layernorm": 512, "bias_gelu": 64, "bias_gelu_erf": 64, "reduction": 512, "matmul": 256,
             "matmul_65536": 256, "flash_attention": 256}


def main_reference(args):
    """--impl reference: the reference's CPU path (the numpy port of the
    reference's refs.py) on every host core, rank 0 only.  A step is one
    bounded sample of the workload: each of the `cores` worker processes
    computes its own row chunk; the inputs are generated outside the timed
    part, and the step's time is the slowest worker's compute time."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import multiprocessing as mp

    spec = WORKLOADS[args.workload]
    cores = os.cpu_count() or 1
    ctx = mp.get_context("spawn")
    chunk = REF_CHUNK[args.workload]
    with ctx.Pool(cores, initializer=_ref_worker_init) as pool:
        def one_step(step):
            jobs = [(args.workload, (step * cores + i) * chunk, chunk) for i in range(cores)]
            res = pool.map(_ref_chunk, jobs)
            return max(r[1] for r in res), sum(r[0] for r in res)
        for i in range(args.warmup):
            one_step(i)
        tt, uu = 0.0, 0.0
        for i in range(args.steps):
            dt, u = one_step(args.warmup + i)
            tt += dt
            uu += u
    val = uu / tt
    unit = "TFLOP/s" if spec["bound"] == "tensor" else "GB/s"
    line = {"metric": "bf16 TFLOP/s & HBM GB/s per kernel family as % of B200 roofline",
            "impl": "reference", "value": round(val, 6), "unit": unit, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(tt / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": args.scaling, "vs_baseline": None, "dtype": spec["dtype"], "data": "synthetic",
            "config": {"workload": spec["desc"], "baseline_config": spec["config"]},
            "cpu_baseline": {"value": round(val, 6), "unit": unit, "cores": cores, "kind": "port",
                             "sample": f"{cores} worker processes x {chunk}-row chunks per step, compute only "
                                       "(numpy restatement of tests/golden/kernscope_golden/refs.py, 1 BLAS "
                                       "thread per process)"},
            "e2e": {"value": round(val, 6), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    gk = _reference_gpu_kernels()
    if gk is not None:
        line["reference_gpu_kernels"] = gk
    print(json.dumps(line))
    return 0


def _reference_gpu_kernels():
    """The reference generator's own kernels (its tuner's auto grid, built by
    oracle/ref_tune/build_ref_kernels.py) timed on this GPU at the benchmark
    shapes, best gate-passing config per family; None without a GPU or
    without the built kernels.  Informational: the arm's value stays the
    reference's CPU path."""
    try:
        import torch

        if not torch.cuda.is_available():
            return None
        from oracle import ref_gpu

        if ref_gpu.index() is None:
            return None
        torch.cuda.set_device(0)
        out = {}
        for fam in ref_gpu.FAMILIES:
            try:
                out[fam] = ref_gpu.run_family(fam)
            except Exception as exc:  # noqa: BLE001 - one family's failure is reported, not fatal
                out[fam] = {"unavailable": str(exc)[:200]}
            torch.cuda.empty_cache()
        return out
    except Exception as exc:  # noqa: BLE001
        return {"unavailable": str(exc)[:200]}


def _ref_chunk(job):
    """(units, seconds) of the reference computation for one row chunk."""
    name, row0, nrows = job
    from oracle import inputs as oin
    from oracle import refs as orf

    shape = WORKLOADS[name]["shape"]
    if name in ROW_FAMILIES:
        rows = shape[0]
        row0 %= rows
        nrows = min(nrows, rows - row0)
    if name == "softmax":
        x = oin.baseline_inputs("softmax", shape, seed=1, row0=row0, nrows=nrows)["x"]
        t0 = time.perf_counter(); orf.softmax(x); dt = time.perf_counter() - t0
        return x.size * 4 / 1e9, dt
    if name == "layernorm":
        d = oin.baseline_inputs("layernorm", shape, seed=2, row0=row0, nrows=nrows)
        t0 = time.perf_counter(); orf.layernorm(d["x"], d["gamma"], d["beta"]); dt = time.perf_counter() - t0
        return d["x"].size * 4 / 1e9, dt
    if name.startswith("bias_gelu"):
        d = oin.baseline_inputs("bias_gelu", shape, seed=2, row0=row0, nrows=nrows)
        fn = orf.bias_gelu if name == "bias_gelu_erf" else orf.bias_gelu_tanh
        t0 = time.perf_counter(); fn(d["x"], d["bias"]); dt = time.perf_counter() - t0
        return d["x"].size * 4 / 1e9, dt
    if name == "reduction":
        (n,) = shape
        cnt = nrows * 65536
        i0 = (row0 * 65536) % (n - cnt)
        x = oin.baseline_inputs("reduction_full", shape, seed=2, row0=i0, nrows=cnt)["x"]
        t0 = time.perf_counter(); orf.sum_full_f64(x); dt = time.perf_counter() - t0
        return cnt * 4 / 1e9, dt
    if name.startswith("matmul"):
        m, n, k = shape
        r0 = row0 % m
        d = oin.baseline_inputs("matmul", shape, seed=3, row0=r0, nrows=min(nrows, m - r0))
        t0 = time.perf_counter(); orf.matmul(d["a"], d["b"]); dt = time.perf_counter() - t0
        return 2 * d["a"].shape[0] * n * k / 1e12, dt
    b, h, s, dd = shape
    head = (row0 // s) % (b * h)
    d = oin.baseline_inputs("attention", (b, h, s, s, dd), seed=4, row0=head, nrows=1)
    q = d["q"][0, s - nrows:]  # the last rows: each attends to (almost) all keys under the causal mask
    t0 = time.perf_counter(); orf.attention(q, d["k"][0], d["v"][0]); dt = time.perf_counter() - t0
    return 4 * dd * q.shape[0] * s / 1e12, dt


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="kernscope", choices=("kernscope", "reference"))
    ap.add_argument("--workload", default="softmax", choices=sorted(WORKLOADS))
    ap.add_argument("--no-families", action="store_true", help="skip the per-family summary")
    ap.add_argument("--scaling", default="weak", choices=("weak", "strong"),
                    help="headline at N>1: weak (one full configuration per GPU) or strong (the configuration "
                         "sharded over the GPUs); every family reports both at N>1 unless --no-strong")
    ap.add_argument("--no-strong", action="store_true", help="skip the strong-scaling measurements at N>1")
    ap.add_argument("--family-steps", type=int, default=20)
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--clock-window", type=float, default=0.9,
                    help="seconds of extra launches around the timed region for the nvidia-smi clock samples "
                         "(0 when the run is profiled, where every launch is replayed)")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = 200
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        return main_reference(args)

    import torch

    rank, world, local = _dist_setup(args)
    spec = WORKLOADS[args.workload]
    peaks = _peaks()
    w = Workload(args.workload, spec["shape"], rank, world)
    # clocks: sample through a window that contains the timed region
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    t_window = time.time()
    while time.time() - t_window < args.clock_window * 2 / 3:  # ramp the clocks before timing
        for i in range(16):
            w.launch(i)
        torch.cuda.synchronize()
    ms, my_ms, timing = measure_device(w, args.steps, args.warmup, world)
    rank_ms = _rank_spread(my_ms, world) if world > 1 else None
    extra_t = time.time()
    while time.time() - extra_t < args.clock_window / 3:
        for i in range(16):
            w.launch(i)
        torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    per = ms / args.steps
    u, unit = _units(w, spec["bound"])
    value = u * world / (per / 1e3)
    achieved = u / (per / 1e3)
    peak = peaks["hbm_gbs"] if spec["bound"] == "hbm" else peaks["bf16_tflops"]
    traffic = _traffic_table().get(args.workload)
    e2e_ms, h2d, d2h = measure_e2e(w, args.e2e_steps, world)
    e2e_val = u * world / (e2e_ms / args.e2e_steps / 1e3)
    kernel = w.config_name()
    del w
    torch.cuda.empty_cache()
    strong = None
    if world > 1 and (args.scaling == "strong" or not args.no_strong):
        strong = measure_strong(args.workload, args, rank, world, per)
    fams = None
    if not args.no_families:
        # the heaviest (power-capped) workload last, so it does not heat the GPU
        # for the others
        order = ["layernorm", "bias_gelu", "bias_gelu_erf", "reduction", "softmax", "flash_attention", "matmul",
                 "matmul_65536"]
        names = [n for n in order if n != args.workload]
        fams = run_families(names, args, rank, world)
    cpu = None
    if rank == 0 and world == 1:
        cv, sample = cpu_baseline(args.workload, spec["shape"], args.cpu_budget)
        cpu = {"value": round(cv, 4), "unit": unit, "cores": 1, "kind": "port",
               "sample": sample + " (numpy restatement of tests/golden/kernscope_golden/refs.py, 1 process)"}
    if rank == 0:
        steps_line, shape_line, par = args.steps, list(spec["shape"]), f"dp{world} (weak: one batch per GPU)"
        if args.scaling == "strong" and strong is not None:
            # headline = the one configuration sharded over the GPUs
            per, value, steps_line = strong["ms_per_step"], strong["value"], strong["steps"]
            shape_line, par = strong["shape_per_gpu"], f"dp{world} (strong: {strong['shard']} on rank 0)"
            achieved = _job_units(args.workload, strong["shape_per_gpu"], spec["bound"]) / (per / 1e3)
        line = {
            "metric": "bf16 TFLOP/s & HBM GB/s per kernel family as % of B200 roofline",
            "value": round(value, 2), "unit": unit, "n_gpus": world, "steps": steps_line,
            "warmup": args.warmup, "ms_per_step": round(per, 5), "higher_is_better": True,
            "scaling": args.scaling if world > 1 else "weak", "vs_baseline": None, "dtype": spec["dtype"],
            "data": "synthetic (seeded torch RNG on device, configuration distributions)",
            "config": {"workload": spec["desc"], "baseline_config": spec["config"],
                       "shape_per_gpu": shape_line, "kernel": kernel,
                       "parallelism": par,
                       "l2": "rotating input/output sets, working set >= 4x L2 (no step reads inputs from L2)",
                       "timing": f"CUDA events on the launching stream, {timing}-replayed launch loop after an "
                                 "untimed pre-roll that follows the barrier (multi-GPU reduction: one NCCL "
                                 "all-reduce per 8 jobs' fp64 partials on a side stream overlapping the next "
                                 "jobs), max over ranks"},
            "roofline": {"bound": spec["bound"], "achieved": round(achieved, 2), "peak": peak, "unit": unit,
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "peak_source": peaks["source"]},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_val, 3), "unit": unit, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": args.steps,
            "clocks": clocks,
        }
        if rank_ms is not None:
            line["rank_ms_per_step"] = [round(v / args.steps, 5) for v in rank_ms]
        if strong is not None:
            line["strong"] = strong
        if fams is not None:
            line["families"] = fams
        print(json.dumps(line))
    from kernscope_b200 import dist

    dist.teardown(world)
    return 0


if __name__ == "__main__":
    sys.exit(main())
