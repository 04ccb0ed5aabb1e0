"""Multi-GPU plumbing of the benchmark: one process per GPU, torch.distributed.

The work shards with no data-path collective (rows, M-panels, heads are
independent); the only exchange is the reduction family's final combine, an
all-reduce of each GPU's fp64 partial sum (NCCL over NVLink on the GPU box,
gloo in the CPU tests).  Job time is the slowest rank's device time.
"""

from __future__ import annotations

import datetime
import os


def setup(backend: str | None = None, timeout_s: int = 120):
    """Init the process group from RANK/WORLD_SIZE/LOCAL_RANK (torchrun env);
    returns (rank, world, local_rank).  Single process: no group."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
        kw = {}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return rank, world, local


def barrier(world: int) -> None:
    import torch

    if torch.cuda.is_available():
        torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    if torch.cuda.is_available():
        torch.cuda.synchronize()


def max_over_ranks(value: float, world: int, device=None) -> float:
    """The job's time: maximum of a per-rank value."""
    if world == 1:
        return float(value)
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_values(value: float, world: int, device=None) -> list[float]:
    """Every rank's value of a per-rank scalar, in rank order."""
    if world == 1:
        return [float(value)]
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(x.item()) for x in out]


def combine_partials(partial_f64, world: int, to_f32: bool = True):
    """The reduction family's cross-GPU combine: sum the per-GPU fp64 partial
    sums in place (count 1); returns the fp32 total (or, with to_f32 False,
    the fp64 partial itself, so that no conversion kernel follows)."""
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(partial_f64, op=dist.ReduceOp.SUM)
    return partial_f64.to(dtype=__import__("torch").float32) if to_f32 else partial_f64


def strong_shard(family: str, shape, rank: int, world: int):
    """This rank's part of a fixed job (strong scaling): rows of the row-wise
    families, elements of the full sum, M-panels of the GEMM (B replicated),
    batch x head pairs of attention.  Returns (shard shape, description)."""
    shape = tuple(int(v) for v in shape)
    if family in ("softmax", "layernorm", "bias_gelu", "bias_gelu_erf"):
        r0, r1 = shard_rows(shape[0], rank, world)
        return (r1 - r0, shape[1]), f"rows [{r0}, {r1}) of {shape[0]}"
    if family == "reduction":
        e0, e1 = shard_rows(shape[0], rank, world)
        return (e1 - e0,), f"elements [{e0}, {e1}) of {shape[0]}"
    if family.startswith("matmul"):
        m0, m1 = shard_rows(shape[0], rank, world)
        return (m1 - m0, shape[1], shape[2]), f"A/C rows [{m0}, {m1}) of {shape[0]}, B replicated"
    if family == "flash_attention":
        b, h, s, d = shape
        p0, p1 = shard_rows(b * h, rank, world)
        n = p1 - p0
        sh = (n // h, h, s, d) if n % h == 0 else (1, n, s, d)
        return sh, f"(batch, head) pairs [{p0}, {p1}) of {b * h}"
    raise KeyError(family)


def shard_rows(rows: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous row range [r0, r1) of `rows` for `rank` (remainder spread
    over the first ranks) -- the strong-scaling split of a fixed job."""
    base, extra = divmod(rows, world)
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


def teardown(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        if dist.is_initialized():
            dist.destroy_process_group()
