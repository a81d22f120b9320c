"""
``append_attend``: KV-append and attention of one layer in one call, one kernel
launch for a decode step (the decode kernel writes each sequence's new K/V row
to its slot and patches it into the staged copy of the last page).

It must be indistinguishable from ``append_kv`` followed by ``attend`` (the
reference engine's two calls, ``docs/ARCHITECTURE.md:167-172``): the same pool
afterwards, bit for bit, and the same attention output, bit for bit (the same
kernel arithmetic runs on the same staged data), across length skews that make
the decode kernel split sequences, full and partial last pages, every GQA
group size and bf16. A mixed batch takes the two-call path. A slot that is not
the last position of the sequence's last page is reported.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from helpers import FifoAllocator, Seq, meta_for, slots_meta
from llm_serving_layer_b200 import B200PagedBackend

pytestmark = pytest.mark.gpu


def setup(seed, ctx, num_blocks, dtype=torch.float16, Hkv=8, Hq=32, D=64, qlens=None):
    """Two backends with identical pools holding every token but the step's new
    ones, plus the step's meta, new K/V and q."""
    rs = np.random.RandomState(seed)
    alloc = FifoAllocator(num_blocks, 16, order=rs.permutation(num_blocks))
    qlens = qlens or [1] * len(ctx)
    seqs = []
    for i, (c, ql) in enumerate(zip(ctx, qlens)):
        s = Seq(alloc, i)
        s.append(int(c) - ql)
        seqs.append(s)
    hist = np.concatenate([[s.slot_for(p) for p in range(s.num_tokens)] for s in seqs]).astype(np.int64)
    g = torch.Generator(device="cuda:0").manual_seed(seed)
    bks = []
    for _ in range(2):
        bk = B200PagedBackend(2, num_blocks, 16, Hkv, Hq, D, device="cuda:0", dtype=dtype)
        bk._pool.fill_(7.0)  # stale data where nothing was written
        bks.append(bk)
    if hist.size:
        k = (torch.randn(hist.size, Hkv, D, generator=g, device="cuda:0") * 0.7).to(dtype)
        v = (torch.randn(hist.size, Hkv, D, generator=g, device="cuda:0") * 0.7).to(dtype)
        for bk in bks:
            bk.append_kv(1, k, v, slots_meta(hist))
    for s, ql in zip(seqs, qlens):
        s.append(ql)
    m = meta_for(seqs, qlens, device="cuda:0")
    T = sum(qlens)
    kn = (torch.randn(T, Hkv, D, generator=g, device="cuda:0") * 0.7).to(dtype)
    vn = (torch.randn(T, Hkv, D, generator=g, device="cuda:0") * 0.7).to(dtype)
    q = torch.randn(T, Hq, D, generator=g, device="cuda:0").to(dtype)
    return bks, seqs, m, kn, vn, q


def run_both(bks, m, kn, vn, q, layer=1):
    a, b = bks
    a.append_kv(layer, kn, vn, m)
    out_a = a.attend(q, layer, 0.125, m)
    out_b = b.append_attend(layer, kn, vn, q, 0.125, m)
    torch.cuda.synchronize()
    a.check_status()
    b.check_status()
    return out_a, out_b


def lognormal(rs, n):
    return np.clip(np.round(rs.lognormal(math.log(256) - 0.32, 0.8, size=n)), 1, 2048).astype(int)


@pytest.mark.parametrize("case", ["lognormal256", "uniform37", "exact_pages", "single_token", "long_split"])
def test_fused_decode_equals_append_then_attend(case):
    rs = np.random.RandomState(3)
    ctx = {"lognormal256": lognormal(rs, 256),
           "uniform37": rs.randint(1, 400, 37),
           "exact_pages": np.asarray([16, 32, 48, 256, 512, 1024] * 10),
           "single_token": np.ones(50, dtype=int),
           "long_split": np.asarray([2048, 1999, 1500, 7, 2047, 33])}[case]
    need = int(((ctx + 15) // 16).sum()) + 16
    bks, seqs, m, kn, vn, q = setup(11, ctx, need * 2)
    out_a, out_b = run_both(bks, m, kn, vn, q)
    assert bks[1].last_kernel == "decode"
    assert torch.equal(out_a, out_b)
    assert torch.equal(bks[0]._pool, bks[1]._pool)


@pytest.mark.parametrize("Hkv,Hq,dtype", [(8, 8, torch.float16), (4, 32, torch.float16), (8, 16, torch.float16),
                                           (8, 32, torch.bfloat16)])
def test_fused_decode_gqa_groups_and_bf16(Hkv, Hq, dtype):
    rs = np.random.RandomState(Hq)
    ctx = lognormal(rs, 64)
    need = int(((ctx + 15) // 16).sum()) + 16
    bks, seqs, m, kn, vn, q = setup(12, ctx, need * 2, dtype=dtype, Hkv=Hkv, Hq=Hq)
    out_a, out_b = run_both(bks, m, kn, vn, q)
    assert torch.equal(out_a, out_b)
    assert torch.equal(bks[0]._pool, bks[1]._pool)


def test_mixed_batch_takes_the_two_calls():
    ctx = [40, 300, 17, 600]
    bks, seqs, m, kn, vn, q = setup(13, ctx, 512, qlens=[1, 30, 1, 200])
    out_a, out_b = run_both(bks, m, kn, vn, q)
    assert bks[1].last_kernel == "prefill"
    assert torch.equal(out_a, out_b)
    assert torch.equal(bks[0]._pool, bks[1]._pool)


def test_slot_that_is_not_the_last_position_is_reported():
    bks, seqs, m, kn, vn, q = setup(14, [20, 35], 64)
    bad = m.slot_mapping.clone()
    bad[0] = seqs[0].slot_for(3)  # an earlier position of the same sequence
    from dataclasses import replace
    mb = replace(m, slot_mapping=bad)
    bks[1].append_attend(1, kn, vn, q, 0.125, mb)
    torch.cuda.synchronize()
    with pytest.raises(Exception, match="inconsistent|META_BAD|page table"):
        bks[1].check_status()


def test_out_buffer_is_written_in_place_and_checked():
    """``attend`` / ``append_attend`` with ``out=`` (an optional extension of
    the reference signature) write the same bits into the caller's buffer and
    return it; a buffer of the wrong shape, dtype or one overlapping q is refused."""
    ctx = [40, 300, 17, 600, 1]
    bks, seqs, m, kn, vn, q = setup(15, ctx, 512)
    out_a, out_b = run_both(bks, m, kn, vn, q)
    buf = torch.full((2, *q.shape), float("nan"), dtype=q.dtype, device=q.device)
    got = bks[0].attend(q, 1, 0.125, m, out=buf[1])
    torch.cuda.synchronize()
    assert got.data_ptr() == buf[1].data_ptr()
    assert torch.equal(buf[1], out_a)
    assert torch.isnan(buf[0]).all()
    with pytest.raises(ValueError, match="out must be a contiguous"):
        bks[0].attend(q, 1, 0.125, m, out=buf[1, :3])
    with pytest.raises(ValueError, match="out must be a contiguous"):
        bks[0].attend(q, 1, 0.125, m, out=buf[1].float())
    with pytest.raises(ValueError, match="must not overlap q"):
        bks[0].attend(q, 1, 0.125, m, out=q)
