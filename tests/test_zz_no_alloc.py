"""
The decode entry point that allocates nothing (``pkv_attend_decode_noalloc``).

Some callers of this library cannot let it allocate device memory: a serving
process that sizes its KV pool to (nearly) all of HBM and allocates nothing
afterwards, or a host application that owns every device allocation. For them
the decode path keeps its per-step scratch (page descriptors, split-K counters
and partial results) in one fixed-size device array inside the library instead
of a workspace the caller passes.

This file checks, through the C ABI, that the entry point returns exactly what
the regular workspace-based entry point (``pkv_attend``) returns for the same
inputs, on two calls in a row (the scratch is shared between calls and keeps
the previous call's contents), that both are within the fp16 tolerance of a
float64 evaluation, that repeated calls leave the device's free memory
unchanged, and that a batch too large for the fixed scratch is refused. It is
named to be collected last.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest
import torch

from helpers import FifoAllocator, Seq, meta_for, slots_meta
from llm_serving_layer_b200 import B200PagedBackend
from llm_serving_layer_b200 import _native as N
from oracle import attend_exact  # the checker

pytestmark = pytest.mark.gpu

TOL = 2e-3  # the fp16 attention tolerance the other GPU tests use


def _batch(m, status):
    i32 = [m.cu_query_lens, m.kv_lens, m.kv_indptr, m.kv_indices, m.kv_last_page_len]
    keep = [t.to(device="cuda:0", dtype=torch.int32).contiguous() for t in i32]
    b = N.BatchDesc(int(m.query_lens.shape[0]), int(m.positions.shape[0]), int(m.kv_indices.shape[0]),
                    keep[0].data_ptr(), keep[1].data_ptr(), keep[2].data_ptr(), keep[3].data_ptr(),
                    keep[4].data_ptr(), status.data_ptr())
    return b, keep


def _decode_case(bk, alloc, rs, n, lognormal):
    if lognormal:
        ctx = np.clip(np.round(rs.lognormal(math.log(256) - 0.32, 0.8, size=n)), 1, 2048).astype(int)
    else:
        ctx = rs.randint(1, 400, size=n)
    seqs = []
    for i, c in enumerate(ctx):
        s = Seq(alloc, i)
        s.append(int(c))
        seqs.append(s)
    slots = np.concatenate([[s.slot_for(p) for p in range(s.num_tokens)] for s in seqs])
    k = (torch.randn(slots.size, 8, 64, device="cuda:0") * 0.7).half()
    v = (torch.randn(slots.size, 8, 64, device="cuda:0") * 0.7).half()
    bk.append_kv(0, k, v, slots_meta(slots))
    q = torch.randn(n, 32, 64, device="cuda:0").half()
    return meta_for(seqs, [1] * n, "cuda:0"), q


def test_noalloc_decode_matches_workspace_decode_twice():
    """Two different batches back to back through both entry points: the same
    plan and decode kernel run on the same grid, so the outputs are bit-identical,
    and both are within the fp16 tolerance of the float64 evaluation. The second
    call must not see the first call's leftovers in the shared scratch."""
    assert torch.cuda.is_available(), "GPU test"
    lib = N.lib()
    nb = 8192
    bk = B200PagedBackend(1, nb, 16, 8, 32, 64, device="cuda:0", dtype=torch.float16)
    rs = np.random.RandomState(5)
    alloc = FifoAllocator(nb, 16, order=rs.permutation(nb))
    status = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    for n, lognormal in ((256, True), (37, False)):
        m, q = _decode_case(bk, alloc, rs, n, lognormal)
        b, keep = _batch(m, status)
        need = lib.pkv_attend_workspace_size(bk._pdesc, 32, b.n_seqs, b.total_pages, 1)
        ws = torch.zeros(need, dtype=torch.uint8, device="cuda:0")
        want = torch.empty_like(q)
        got = torch.full_like(q, float("nan"))
        rc = lib.pkv_attend(bk._pdesc, 0, 32, q.data_ptr(), want.data_ptr(), 0.125, ctypes.byref(b), 1,
                            ws.data_ptr(), need, stream)
        assert rc == 0, lib.pkv_last_error()
        rc = lib.pkv_attend_decode_noalloc(bk._pdesc, 0, 32, q.data_ptr(), got.data_ptr(), 0.125,
                                           ctypes.byref(b), stream)
        assert rc == 0, lib.pkv_last_error()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert torch.equal(got, want), "no-allocation decode differs from the workspace decode"
        exact = attend_exact(q.cpu().numpy(), bk.k_pool[0].cpu().numpy(), bk.v_pool[0].cpu().numpy(), 0.125, m)
        err = float(np.abs(got.float().cpu().numpy() - exact).max())
        assert err <= TOL, f"no-allocation decode off by {err} from the float64 evaluation"
        del keep


def test_noalloc_decode_allocates_no_device_memory():
    """After a first call (which looks up the scratch array's address), further
    calls leave the device's free memory exactly as it was."""
    lib = N.lib()
    nb = 2048
    bk = B200PagedBackend(1, nb, 16, 8, 32, 64, device="cuda:0", dtype=torch.float16)
    rs = np.random.RandomState(11)
    alloc = FifoAllocator(nb, 16, order=rs.permutation(nb))
    status = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    m, q = _decode_case(bk, alloc, rs, 64, False)
    b, keep = _batch(m, status)
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream().cuda_stream

    def call():
        rc = lib.pkv_attend_decode_noalloc(bk._pdesc, 0, 32, q.data_ptr(), out.data_ptr(), 0.125,
                                           ctypes.byref(b), stream)
        assert rc == 0, lib.pkv_last_error()
        torch.cuda.synchronize()

    call()
    free_before, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        call()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before, f"device free memory moved by {free_before - free_after} bytes"
    assert int(status.item()) == 0
    del keep


def test_noalloc_decode_rejects_a_batch_larger_than_its_scratch():
    """A batch whose scratch would not fit the fixed array is refused on the
    host with an argument error that names the sizes; nothing is launched (the
    page table is never read: its pointers only have to be non-NULL)."""
    lib = N.lib()
    bk = B200PagedBackend(1, 64, 16, 8, 32, 64, device="cuda:0", dtype=torch.float16)
    status = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    dummy = torch.zeros(4, dtype=torch.int32, device="cuda:0")
    q = torch.zeros(1, 32, 64, device="cuda:0", dtype=torch.float16)
    b = N.BatchDesc(1, 1, 600_000, dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(),
                    dummy.data_ptr(), status.data_ptr())
    rc = lib.pkv_attend_decode_noalloc(bk._pdesc, 0, 32, q.data_ptr(), q.data_ptr(), 0.125, ctypes.byref(b),
                                       torch.cuda.current_stream().cuda_stream)
    assert rc == N.PKV_ERR_ARG
    msg = lib.pkv_last_error()
    assert b"bytes of scratch" in msg, msg
    torch.cuda.synchronize()
    assert int(status.item()) == 0


def test_noalloc_decode_rejects_what_it_cannot_hold():
    lib = N.lib()
    bk = B200PagedBackend(1, 64, 16, 2, 4, 8, device="cuda:0", dtype=torch.float32)  # not the decode geometry
    status = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    s = Seq(FifoAllocator(64, 16))
    s.append(5)
    m = meta_for([s], [1], "cuda:0")
    b, keep = _batch(m, status)
    q = torch.zeros(1, 4, 8, device="cuda:0")
    rc = lib.pkv_attend_decode_noalloc(bk._pdesc, 0, 4, q.data_ptr(), q.data_ptr(), 1.0, ctypes.byref(b),
                                       torch.cuda.current_stream().cuda_stream)
    assert rc == N.PKV_ERR_UNSUPPORTED
    assert b"no-allocation decode" in lib.pkv_last_error()
