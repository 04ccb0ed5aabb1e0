"""CPU, world_size 2 gloo ranks: the multi-GPU host logic of the benchmark.

Each rank sums its shard of the full-sum workload in fp64 (the GPU kernel's
partial), the ranks combine with one all-reduce (the reduction family's only
collective), and the job time is the maximum over ranks.  Also: a rank that
raises before the collective makes the other rank's collective fail within
the process-group timeout instead of hanging (failure on the host, no GPU).
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n, q, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch

    from kernscope_b200 import dist
    from oracle import inputs as oin

    r, w, _ = dist.setup(backend="gloo", timeout_s=10)
    try:
        if rank == fail_rank:
            raise RuntimeError("injected rank failure")
        r0, r1 = dist.shard_rows(n, r, w)
        x = oin.baseline_inputs("reduction_full", (n,), seed=2, row0=r0, nrows=r1 - r0)["x"]
        mine = float(np.sum(x, dtype=np.float64))
        part = torch.tensor([mine], dtype=torch.float64)
        total = dist.combine_partials(part, w)  # in place: part now holds the job's sum
        t = dist.max_over_ranks(1.0 + rank, w)
        assert dist.gather_values(0.5 + rank, w) == [0.5 + k for k in range(w)]  # per-rank spread, rank order
        q.put((rank, float(total.item()), mine, t, None))
    except Exception as exc:  # noqa: BLE001 - report to the parent
        q.put((rank, None, None, None, type(exc).__name__ + ": " + str(exc)[:120]))
    finally:
        dist.teardown(w)


def _run(world, n, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    return sorted(out)


def test_two_rank_sum_combine_and_max_time():
    n = 3_000_001
    out = _run(2, n)
    from oracle import inputs as oin

    ref = float(np.sum(oin.baseline_inputs("reduction_full", (n,), seed=2)["x"], dtype=np.float64))
    for rank, total, part, t, err in out:
        assert err is None
        assert abs(total - ref) <= 1e-5 * ref
        assert t == 2.0  # max over ranks of 1 + rank
    assert abs(out[0][2] + out[1][2] - ref) <= 1e-9 * ref


def test_shard_rows_cover():
    from kernscope_b200 import dist

    for rows, world in ((4096, 8), (10, 3), (1, 2)):
        spans = [dist.shard_rows(rows, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == rows
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


@pytest.mark.timeout(180)
def test_failed_rank_ends_collective_with_error():
    out = _run(2, 1000, fail_rank=1)
    errs = {rank: err for rank, _, _, _, err in out}
    assert "injected rank failure" in errs[1]
    assert errs[0] is not None  # the surviving rank's all-reduce errored out instead of hanging


@pytest.mark.parametrize("family", ["softmax", "layernorm", "bias_gelu", "bias_gelu_erf", "reduction", "matmul",
                                    "matmul_65536", "flash_attention"])
def test_strong_shards_partition_the_job(family):
    """Strong scaling: the G shards of a benchmark configuration cover the
    whole job exactly (rows, elements, M-panels, batch x head pairs), so the
    sharded job does the same algorithmic work as one GPU does alone."""
    import importlib.util

    from kernscope_b200 import dist

    spec = importlib.util.spec_from_file_location("bench", os.path.join(os.path.dirname(__file__), "..", "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    wl = bench.WORKLOADS[family]
    full = bench._job_units(family, wl["shape"], wl["bound"])
    for world in (1, 2, 4, 8):
        shards = [dist.strong_shard(family, wl["shape"], r, world)[0] for r in range(world)]
        parts = [bench._job_units(family, sh, wl["bound"]) for sh in shards]
        if family in ("layernorm", "bias_gelu", "bias_gelu_erf"):  # gamma/beta/bias are read by every shard
            extra = (world - 1) * (2 * wl["shape"][1] * 2 if family == "layernorm" else wl["shape"][1] * 2) / 1e9
            assert abs(sum(parts) - extra - full) <= 1e-9 * full
        elif family == "reduction":  # every shard writes its own 4-byte result
            assert abs(sum(parts) - (world - 1) * 4e-9 - full) <= 1e-9 * full
        else:
            assert abs(sum(parts) - full) <= 1e-9 * full, (world, shards)
        if family.startswith("matmul"):
            assert all(sh[1:] == tuple(wl["shape"][1:]) for sh in shards)  # B replicated, K and N whole


def _shard_status(N, ops, family, shape):
    """(status, reason) of the family's validator for one shard, with the
    config the benchmark launches for that shard (pointers are placeholders:
    the validators read shapes and configs only)."""
    p = 256
    if family == "softmax":
        return N.validate("softmax", ops.default_softmax_config(shape[1]), *shape)
    if family == "layernorm":
        return N.validate("layernorm", ops.default_layernorm_config(shape[1]), *shape)
    if family in ("bias_gelu", "bias_gelu_erf"):
        cfg = ops.default_bias_gelu_config(shape[1], "erf" if family == "bias_gelu_erf" else "tanh")
        return N.validate("bias_gelu", cfg, shape[0] * shape[1], shape[1])
    if family == "reduction":
        a = N.ReductionArgs(p, p, shape[0], 1, N.KS_F32, N.KS_F32, -1, None, 0, None)
        return N.validate("reduction", ops.default_reduction_config(shape[0], -1), a)
    if family.startswith("matmul"):
        return N.validate("matmul", ops.default_matmul_config(*shape), *shape)
    b, h, s, d = shape
    a = N.FlashAttentionArgs(p, p, p, p, b, h, s, s, d, d ** -0.5)
    return N.validate("flash_attention", ops.default_flash_attention_config(True), a)


@pytest.mark.parametrize("family", ["softmax", "layernorm", "bias_gelu", "bias_gelu_erf", "reduction", "matmul",
                                    "matmul_65536", "flash_attention"])
def test_strong_shards_pass_the_validators(family):
    """Every rank's shard of a benchmark configuration at 1, 2, 4 and 8 GPUs
    (the strong-scaling runs) is a shape the family's validator accepts with
    the config the benchmark launches for it."""
    import importlib.util

    from kernscope_b200 import dist, native as N, ops

    spec = importlib.util.spec_from_file_location("bench", os.path.join(os.path.dirname(__file__), "..", "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    shape = bench.WORKLOADS[family]["shape"]
    for world in (1, 2, 4, 8):
        for r in range(world):
            sh, _ = dist.strong_shard(family, shape, r, world)
            st, why = _shard_status(N, ops, family, sh)
            assert st == 0, (family, world, r, sh, why)
