"""
The reference's own callers, replayed on the B200 drop-ins.

``tests/golden/scheduler_trace.npz`` holds every backend and swap-space call
that the reference's unmodified ``Scheduler`` (serving/scheduler/scheduler.py:
696-771 step, 960-993 swap preemption, 995-1084 resume) made with a
``RadixCache`` wired to the backend's ``copy_block`` (serving/cache/radix.py:
629-677, as serving/server/app.py:1245-1252 wires it) and SWAP preemption
through ``KVSwapSpace`` (serving/scheduler/preemption.py:399-523), on its
``PagedTorchBackend`` — recorded by ``tests/golden/make_trace.py``: chunked
prefill mixed with decodes, radix prefix hits on shared blocks, a
copy-on-write, a victim swapped out under pool exhaustion and resumed into
fresh blocks.

Here the same calls, in the same order, go to ``B200PagedBackend`` and
``B200SwapSpace`` (``append_kv``, ``attend``, ``copy_block``, ``swap_out``,
``swap_in``, ``release``), with a CPU oracle pool fed the same calls beside
them:

* after every scheduler step the B200 pools hash to the reference's pools
  (SHA-256 over every layer's K and V, bit for bit) — appends, the COW copy and
  the swap-in scatter are exact;
* every swapped-out host buffer is the reference's bit for bit;
* every attention output is within 2e-3 of the float64 evaluation on the same
  pool, and within 3e-3 of the reference's own fp16
  output (both sides round probabilities to fp16 at different points).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from llm_serving_layer_b200 import B200PagedBackend, B200SwapSpace, BatchMeta
from oracle import OraclePool, attend_exact  # the checker
from sched_trace import Blocks, load, pool_sha

pytestmark = pytest.mark.gpu

TOL_EXACT = 2e-3
TOL_REF = 3e-3


def _meta(fields: dict, dev) -> BatchMeta:
    i32 = lambda x: torch.from_numpy(np.asarray(x, dtype=np.int32)).to(dev)  # noqa: E731
    return BatchMeta(query_lens=i32(fields["query_lens"]), cu_query_lens=i32(fields["cu_query_lens"]),
                     kv_lens=i32(fields["kv_lens"]),
                     positions=torch.from_numpy(np.asarray(fields["positions"], dtype=np.int64)).to(dev),
                     last_token_ix=i32(fields["last_token_ix"]), kv_indptr=i32(fields["kv_indptr"]),
                     kv_indices=i32(fields["kv_indices"]), kv_last_page_len=i32(fields["kv_last_page_len"]),
                     batch_indices=i32(fields["batch_indices"]), slot_mapping=i32(fields["slot_mapping"]),
                     page_size=16, is_prefill=fields["is_prefill"])


@pytest.mark.parametrize("validate", ["host", "device"])
def test_reference_scheduler_trace_replays_on_b200(validate):
    dev = torch.device("cuda:0")
    t = load()
    bk = B200PagedBackend(t.num_layers, t.num_blocks, t.block_size, t.n_kv_heads, t.n_heads, t.head_dim,
                          device=dev, dtype=torch.float16, validate=validate)
    sw = B200SwapSpace(bk)
    ora = OraclePool(t.num_layers, t.num_blocks, t.block_size, t.n_kv_heads, t.head_dim, dtype=np.float16)
    metas = [_meta(t.meta(i), dev) for i in range(t.n_metas)]
    host_metas = [t.meta(i) for i in range(t.n_metas)]
    handles, kernels = {}, set()
    worst_exact = worst_ref = 0.0
    n_steps = 0
    for ev in t.events():
        kind = ev[0]
        if kind == "append":
            _, step, layer, mi, k, v = ev
            bk.append_kv(layer, torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev), metas[mi])
            ora.append_kv(layer, k, v, host_metas[mi]["slot_mapping"])
        elif kind == "attend":
            _, step, layer, mi, q, ref_out = ev
            out = bk.attend(torch.from_numpy(q).to(dev), layer, t.scale, metas[mi]).float().cpu().numpy()
            kernels.add(bk.last_kernel)
            exact = attend_exact(q, ora.k[layer], ora.v[layer], t.scale, host_metas[mi])
            e1 = float(np.abs(out - exact).max())
            e2 = float(np.abs(out - ref_out.astype(np.float64)).max())
            assert e1 <= TOL_EXACT, f"step {step} layer {layer}: {e1} from the float64 evaluation"
            assert e2 <= TOL_REF, f"step {step} layer {layer}: {e2} from the reference's output"
            worst_exact, worst_ref = max(worst_exact, e1), max(worst_ref, e2)
        elif kind == "copy":
            _, step, src, dst = ev
            bk.copy_block(src, dst)
            ora.copy_block(src, dst)
        elif kind == "swap_out":
            _, step, hid, ids, ntok, kh, vh = ev
            h = sw.swap_out(f"req{hid}", Blocks(ids, ntok))
            assert np.array_equal(h.k.numpy(), kh) and np.array_equal(h.v.numpy(), vh), \
                f"swap-out {hid} differs from the reference's host buffers"
            handles[hid] = h
            ora_k, ora_v = ora.swap_out(ids)
            assert np.array_equal(ora_k, kh)
        elif kind == "swap_in":
            _, step, hid, ids = ev
            h = handles[hid]
            sw.swap_in(h, Blocks(ids, h.num_tokens))
            ora.swap_in(h.k.numpy(), h.v.numpy(), ids)
        elif kind == "release":
            sw.release(handles.pop(ev[2]))
        else:
            _, step, sha = ev
            torch.cuda.synchronize()
            bk.check_status()
            kp = [bk.k_pool[l].cpu().numpy() for l in range(t.num_layers)]
            vp = [bk.v_pool[l].cpu().numpy() for l in range(t.num_layers)]
            assert pool_sha(kp, vp) == sha, f"B200 pools differ from the reference's after step {step}"
            assert pool_sha(ora.k, ora.v) == sha
            n_steps += 1
    assert n_steps == t.stats["steps"] and not handles
    assert {"decode", "prefill"} <= kernels, kernels
    print(f"\n{n_steps} reference scheduler steps replayed ({validate}-validated): pools bit-exact after "
          f"every step; attention max |err| {worst_exact:.2e} vs float64, {worst_ref:.2e} vs the reference")
