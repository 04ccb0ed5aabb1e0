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


def combine_partials(partial_f64, world: int):
    """The reduction family's cross-GPU combine: sum the per-GPU fp64 partial
    sums in place (count 1); returns the fp32 total."""
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(partial_f64, op=dist.ReduceOp.SUM)
    return partial_f64.to(dtype=__import__("torch").float32)


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
