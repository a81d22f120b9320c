"""
Failure detection without a GPU fault: every wait in the kernels is bounded
(about a second of %globaltimer) and reports PKV_DEV_WAIT_TIMEOUT in the status
word instead of hanging. ``pkv_wait_probe`` makes an mbarrier wait and a
device-word wait run out on purpose (nothing arrives, nothing sets the word);
the host then reads the error through ``check_status`` and the same context
keeps working (a decode step afterwards matches the oracle).
"""

from __future__ import annotations

import time

import numpy as np
import pytest
import torch

from llm_serving_layer_b200 import B200PagedBackend, build_meta
from llm_serving_layer_b200 import _native as N
from llm_serving_layer_b200._native import PkvError
from oracle import OraclePool, attend_exact  # the checker

pytestmark = pytest.mark.gpu


def test_bounded_waits_give_up_report_and_leave_the_context_usable():
    dev = torch.device("cuda:0")
    bk = B200PagedBackend(1, 32, 16, 8, 32, 64, device=dev, dtype=torch.float16)
    never = torch.zeros(1, dtype=torch.int32, device=dev)
    result = torch.full((1,), -1, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    N.check(N.lib().pkv_wait_probe(never.data_ptr(), bk._status.data_ptr(), result.data_ptr(),
                                   N.raw_stream(0)), "wait_probe")
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert int(result.item()) == 0, "neither wait may have been satisfied"
    assert 1.5 < dt < 30, f"two bounded waits of ~1 s each took {dt:.2f} s"
    with pytest.raises(PkvError, match="(?i)wait"):
        bk.check_status()
    bk.check_status()  # the error was reported once and cleared

    # the context still runs the hot path correctly
    rs = np.random.RandomState(0)
    host = OraclePool(1, 32, 16, 8, 64, dtype=np.float16)
    tables, ctx = [[3, 9], [17]], [20, 5]
    hist = build_meta(tables, ctx, ctx, 16, device=dev)
    k = (rs.standard_normal((25, 8, 64)) * 0.7).astype(np.float16)
    v = (rs.standard_normal((25, 8, 64)) * 0.7).astype(np.float16)
    bk.append_kv(0, torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev), hist)
    host.append_kv(0, k, v, hist.slot_mapping.cpu().numpy())
    step = build_meta(tables, ctx, [1, 1], 16, device=dev)
    q = rs.standard_normal((2, 32, 64)).astype(np.float16)
    out = bk.attend(torch.from_numpy(q).to(dev), 0, 0.125, step)
    torch.cuda.synchronize()
    bk.check_status()
    err = np.abs(out.float().cpu().numpy() - attend_exact(q, host.k[0], host.v[0], 0.125, step)).max()
    assert err <= 2e-3
