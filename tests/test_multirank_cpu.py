"""
The multi-GPU path of bench.py on CPU: two ``gloo`` ranks run the replica
bench's cross-rank steps (the only data the replicas exchange): the job's
elapsed time is the slowest rank's (all-reduce MAX), rates add up (all-reduce
SUM), every rank's GPU id is gathered in rank order for the clock sampler, and
the whole-job tok/s counts every rank's sequences over the slowest rank's
time. Each rank also derives its own workload seed (replicas decode different
sequences). And a rank that leaves between steps makes the survivor's next
reduction end with an error within the group's short timeout, not hang.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _worker(rank: int, ws: int, port: int, q) -> None:
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(ws),
                      LOCAL_RANK=str(rank))
    import bench
    dist.init_process_group("gloo", rank=rank, world_size=ws,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        env = bench.dist_env()
        ms = [120.0, 135.5][rank]  # rank 1 is the slow one
        mx = bench.max_over_ranks(dist, ms, torch.device("cpu"))
        sums = bench.sum_over_ranks(dist, [1000.0 * (rank + 1), 1.5], torch.device("cpu"))
        ids = bench.job_gpu_ids(dist, f"GPU-{rank}")
        val = bench.replica_value(bench.N_SEQ, ws, 100, mx)
        rs = __import__("numpy").random.RandomState(2026 + 1000 * rank)
        ctx = bench.contexts(rs)
        q.put((rank, env, mx, sums, ids, val, int(ctx.sum())))
    finally:
        dist.destroy_process_group()


def test_replica_reductions_over_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    out.sort()
    for rank, env, mx, sums, ids, val, ctx_sum in out:
        assert env == (2, rank, rank)
        assert mx == 135.5                       # the slowest rank's time, on every rank
        assert sums == [3000.0, 3.0]             # rates add up
        assert ids == "GPU-0,GPU-1"              # rank order
        assert val == pytest.approx(256 * 2 * 100 / 0.1355)
    assert out[0][6] != out[1][6]                # each replica decodes its own sequences


def test_single_process_reductions_are_identity():
    sys.path.insert(0, str(ROOT))
    import bench
    assert not dist.is_initialized()
    assert bench.max_over_ranks(dist, 7.0, torch.device("cpu")) == 7.0
    assert bench.sum_over_ranks(dist, [1.0, 2.0], torch.device("cpu")) == [1.0, 2.0]
    assert bench.job_gpu_ids(dist, "GPU-x") == "GPU-x"


def _dying_worker(rank: int, ws: int, port: int, q) -> None:
    """Rank 1 leaves between steps (after a first reduction, before the next,
    with nothing in flight); rank 0 then enters the next reduction, which must
    end with an error within the group's short timeout instead of waiting."""
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(ws),
                      LOCAL_RANK=str(rank))
    import time

    import bench
    dist.init_process_group("gloo", rank=rank, world_size=ws,
                            timeout=__import__("datetime").timedelta(seconds=5))
    first = bench.max_over_ranks(dist, [10.0, 20.0][rank], torch.device("cpu"))
    if rank == 1:
        q.put((rank, first, "left", 0.0))
        q.close()
        q.join_thread()  # the result is sent before the process goes
        os._exit(0)  # gone without a goodbye: no destroy_process_group, no further collective
    time.sleep(0.5)
    t0 = time.perf_counter()
    try:
        bench.max_over_ranks(dist, 30.0, torch.device("cpu"))
        outcome = "returned"
    except Exception as e:  # noqa: BLE001 — the failure is the expected outcome
        outcome = type(e).__name__
    q.put((rank, first, outcome, time.perf_counter() - t0))
    q.close()
    q.join_thread()
    os._exit(0)


def test_a_rank_that_leaves_makes_the_next_reduction_fail_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29800 + os.getpid() % 150
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    (r0, first0, outcome0, waited0), (r1, first1, outcome1, _) = out
    assert first0 == first1 == 20.0       # the step both ranks took
    assert outcome1 == "left"
    assert outcome0 != "returned", "the survivor's reduction must fail, not return"
    assert waited0 < 60.0                 # ended by the peer's exit or the 5 s group timeout
