"""
The CPU oracle replays the reference scheduler's recorded backend calls
(``tests/golden/scheduler_trace.npz``, made by ``tests/golden/make_trace.py``
from the reference's own ``Scheduler``, ``RadixCache`` and ``KVSwapSpace`` on
its ``PagedTorchBackend``): after every scheduler step its pools hash to the
reference's, the swapped-out host buffers are the reference's bit for bit, and
every attention output is the reference's to one fp16 ulp. This pins the trace
and the oracle together; ``test_gpu_trace.py`` replays the same calls on the
B200 backend.
"""

from __future__ import annotations

import numpy as np

from oracle import OraclePool, attend_reference  # the checker
from sched_trace import load, pool_sha


def test_trace_covers_the_reference_callers():
    t = load()
    s = t.stats
    assert s["copy_block"] == 1 and s["cow_copies"] == 1
    assert s["swap_out"] >= 1 and s["swap_in"] >= 1 and s["preemptions"] >= 1
    assert s["blocks_reused"] > 0
    assert s["decode_steps"] > 0 and s["mixed_steps"] > 0
    assert (t.num_layers, t.n_kv_heads, t.n_heads, t.head_dim, t.block_size) == (2, 8, 32, 64, 16)


def test_oracle_replays_the_reference_scheduler_trace():
    t = load()
    pool = OraclePool(t.num_layers, t.num_blocks, t.block_size, t.n_kv_heads, t.head_dim, dtype=np.float16)
    metas = [t.meta(i) for i in range(t.n_metas)]
    swapped = {}
    counts = dict.fromkeys(("append", "attend", "copy", "swap_out", "swap_in", "release", "step"), 0)
    for ev in t.events():
        kind = ev[0]
        counts[kind] += 1
        if kind == "append":
            _, _, layer, mi, k, v = ev
            pool.append_kv(layer, k, v, metas[mi]["slot_mapping"])
        elif kind == "attend":
            _, _, layer, mi, q, out = ev
            got = attend_reference(q, pool.k[layer], pool.v[layer], t.scale, metas[mi]).astype(np.float64)
            want = out.astype(np.float64)
            tol = np.spacing(np.abs(out)).astype(np.float64) + 5e-4
            assert np.all(np.abs(got - want) <= tol), f"attention differs at step {ev[1]} layer {layer}"
        elif kind == "copy":
            pool.copy_block(ev[2], ev[3])
        elif kind == "swap_out":
            _, _, hid, ids, ntok, kh, vh = ev
            k, v = pool.swap_out(ids)
            assert np.array_equal(k, kh) and np.array_equal(v, vh), f"swap-out {hid} differs"
            swapped[hid] = (k, v)
        elif kind == "swap_in":
            _, _, hid, ids = ev
            pool.swap_in(*swapped[hid], ids)
        elif kind == "release":
            swapped.pop(ev[2])
        else:
            assert pool_sha(pool.k, pool.v) == ev[2], f"pools differ from the reference after step {ev[1]}"
    assert counts["copy"] == 1 and counts["swap_out"] >= 1 and counts["swap_in"] >= 1
    assert counts["step"] == t.stats["steps"] and not swapped
