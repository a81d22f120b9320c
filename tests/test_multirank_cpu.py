"""
The multi-GPU path of bench.py on CPU: two ``gloo`` ranks run the replica
bench's cross-rank steps (the only data the replicas exchange): the job's
elapsed time is the slowest rank's (all-reduce MAX), rates add up (all-reduce
SUM), every rank's GPU id is gathered in rank order for the clock sampler, and
the whole-job tok/s counts every rank's sequences over the slowest rank's
time. Each rank also derives its own workload seed (replicas decode different
sequences).
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
