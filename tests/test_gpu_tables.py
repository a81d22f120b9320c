"""
Device-side BatchMeta assembly (``DeviceBlockTables`` / ``pkv_build_batch_meta``)
against the reference's ``build_batch_meta`` (``serving/engine_iface/batch.py:190-318``).

Every field must be bit-identical: to the golden fixture the reference itself
produced (``tests/golden/batch_assembly.npz``), and to the host assembler and
the oracle's restatement of the block-table arithmetic (``slot_for``,
``build_csr``) on random decode / chunked-prefill / mixed steps, across a long
run of steps in which sequences arrive, grow, are copied on write, finish and
their rows are reused. The reference's ``ValueError``s are raised before
anything runs; attention over a device-assembled meta equals attention over
the host-assembled one, bit for bit.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from llm_serving_layer_b200 import B200PagedBackend, DeviceBlockTables, build_meta
from oracle import attend_exact, build_csr, slot_for  # the checker

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden"
FIELDS = ("query_lens", "cu_query_lens", "kv_lens", "positions", "last_token_ix", "kv_indptr", "kv_indices",
          "kv_last_page_len", "batch_indices", "slot_mapping")
DEV = "cuda:0"


def fields_equal(dm, hm):
    torch.cuda.synchronize()
    for f in FIELDS:
        a, b = getattr(dm, f).cpu(), getattr(hm, f).cpu()
        assert a.dtype == b.dtype, f
        assert torch.equal(a, b), f"{f}: device {a[:16].tolist()} host {b[:16].tolist()}"
    assert dm.is_prefill == hm.is_prefill
    assert dm.page_size == hm.page_size


def oracle_check(dm, tables, kv, ql, P):
    """The oracle's slot_for / build_csr against the device fields."""
    ip, idx, lp = build_csr(tables, list(kv), P)
    assert dm.kv_indptr.cpu().tolist() == ip
    assert dm.kv_indices.cpu().tolist() == idx
    assert dm.kv_last_page_len.cpu().tolist() == lp
    slots = []
    for t, k, q in zip(tables, kv, ql):
        slots += [slot_for(t, p, P) for p in range(k - q, k)]
    assert dm.slot_mapping.cpu().tolist() == slots


def test_matches_reference_golden():
    f = np.load(GOLD / "batch_assembly.npz")
    tables = [t.tolist() for t in np.split(f["tables_flat"], np.cumsum(f["tables_len"])[:-1])]
    kv = f["hist"] + f["qlens"]
    bt = DeviceBlockTables(8, 8, 16, num_blocks=64, device=DEV)
    rows = [5, 0, 7, 2, 3]  # rows need not follow batch order
    for r, t in zip(rows, tables):
        bt.bind(r, t)
    m = bt.build_batch_meta(rows, f["qlens"], kv)
    torch.cuda.synchronize()
    for name in FIELDS:
        assert np.array_equal(getattr(m, name).cpu().numpy(), f[name]), name
    assert m.is_prefill == bool(f["is_prefill"])
    m.validate()
    bt.check_status()


def random_step(rs, n, P, kind, max_q=512):
    hist = rs.randint(0, 1500, size=n)
    if kind == "decode":
        ql = np.ones(n, dtype=int)
    elif kind == "prefill":
        ql = rs.randint(2, max_q + 1, size=n)
    else:
        ql = np.where(rs.rand(n) < 0.5, 1, rs.randint(2, max_q + 1, size=n))
    kv = hist + ql
    return ql, kv


@pytest.mark.parametrize("kind,n", [("decode", 256), ("decode", 1), ("decode", 1024), ("prefill", 7),
                                    ("mixed", 40), ("mixed", 300)])
def test_random_steps_match_host_assembler_and_oracle(kind, n):
    rs = np.random.RandomState(n + len(kind))
    P, NB = 16, 200_000
    ql, kv = random_step(rs, n, P, kind)
    pages = (kv + P - 1) // P
    ids = rs.permutation(NB)[: int(pages.sum())]
    tables = [t.tolist() for t in np.split(ids, np.cumsum(pages)[:-1])]
    max_pages = int(pages.max()) + 3
    bt = DeviceBlockTables(n + 5, max_pages, P, num_blocks=NB, device=DEV, max_tokens=int(ql.sum()))
    rows = rs.permutation(n + 5)[:n]
    for r, t in zip(rows, tables):
        bt.bind(int(r), t)
    dm = bt.build_batch_meta(rows, ql, kv)
    hm = build_meta(tables, kv, ql, P, device=DEV)
    fields_equal(dm, hm)
    oracle_check(dm, tables, kv.tolist(), ql.tolist(), P)
    assert dm.max_query_len == int(ql.max()) and dm.min_query_len == int(ql.min())
    assert dm.checked_blocks == NB
    bt.check_status()


def test_exact_page_multiples_and_full_rows():
    P = 16
    kv = np.asarray([16, 32, 1, 15, 17, 128])
    ql = np.asarray([1, 16, 1, 15, 2, 128])
    pages = (kv + P - 1) // P
    ids = np.arange(int(pages.sum()))[::-1] + 3
    tables = [t.tolist() for t in np.split(ids, np.cumsum(pages)[:-1])]
    bt = DeviceBlockTables(6, 8, P, num_blocks=64, device=DEV)  # the last row is exactly full
    for r, t in enumerate(tables):
        bt.bind(r, t)
    dm = bt.build_batch_meta(range(6), ql, kv)
    fields_equal(dm, build_meta(tables, kv, ql, P, device=DEV))
    assert dm.kv_last_page_len.cpu().tolist() == [16, 16, 1, 15, 1, 16]


def test_incremental_steps_with_arrivals_cow_and_row_reuse():
    """60 steps of a continuous batch: new sequences (bind with their prompt's
    blocks), chunked prompts, decodes that cross page boundaries (extend),
    copy-on-write of a last block (set_block), finished sequences (release, row
    reused). Only the changes travel; every step equals the host assembler."""
    rs = np.random.RandomState(5)
    P, NB, MAXS, MAXP = 16, 4096, 48, 40
    free = list(rs.permutation(NB))
    bt = DeviceBlockTables(MAXS, MAXP, P, num_blocks=NB, device=DEV, ring=2)
    live = {}  # row -> dict(table, done, prompt, target)
    free_rows = list(range(MAXS))
    total_updates = 0
    for step in range(60):
        while free_rows and len(live) < 40 and rs.rand() < 0.7:
            r = free_rows.pop(rs.randint(len(free_rows)))
            prompt = int(rs.randint(1, 200))
            live[r] = {"table": [], "done": 0, "prompt": prompt, "target": prompt + int(rs.randint(1, 300))}
        rows, ql, kv, tables = [], [], [], []
        for r, s in live.items():
            q = min(int(rs.randint(1, 96)), s["prompt"] - s["done"]) if s["done"] < s["prompt"] else 1
            k = s["done"] + q
            need = (k + P - 1) // P - len(s["table"])
            new = [int(free.pop()) for _ in range(max(need, 0))]
            if not s["table"]:
                s["table"] = new
                bt.bind(r, new)
            elif new:
                s["table"] += new
                bt.extend(r, new)
            if s["table"] and rs.rand() < 0.05:  # copy-on-write of the last block
                b = int(free.pop())
                free.append(s["table"][-1])
                s["table"][-1] = b
                bt.set_block(r, len(s["table"]) - 1, b)
            s["done"] = k
            rows.append(r)
            ql.append(q)
            kv.append(k)
            tables.append(list(s["table"]))
        if not rows:  # nothing scheduled: the reference skips the step
            continue
        total_updates += bt._n_upd
        dm = bt.build_batch_meta(rows, ql, kv)
        hm = build_meta(tables, kv, ql, P, device=DEV)
        fields_equal(dm, hm)
        for r in [r for r, s in live.items() if s["done"] >= s["target"]]:
            free.extend(live[r]["table"])
            del live[r]
            bt.release(r)
            free_rows.append(r)
    bt.check_status()
    assert total_updates < 3000  # only changes travel


def test_twice_edited_page_takes_the_last_edit():
    bt = DeviceBlockTables(4, 4, 16, num_blocks=100, device=DEV)
    bt.bind(1, [10, 11, 12])
    bt.set_block(1, 2, 50)
    bt.set_block(1, 2, 51)
    bt.bind(2, [20])
    bt.bind(2, [21, 22])
    m = bt.build_batch_meta([1, 2], [1, 1], [48, 32])
    torch.cuda.synchronize()
    assert m.kv_indices.cpu().tolist() == [10, 11, 51, 21, 22]


def test_ring_keeps_recent_metas_intact():
    P = 16
    bt = DeviceBlockTables(4, 8, P, num_blocks=64, device=DEV, ring=3)
    bt.bind(0, [1, 2, 3, 4])
    metas = [bt.build_batch_meta([0], [1], [k]) for k in (20, 40, 60)]
    torch.cuda.synchronize()
    for m, k in zip(metas, (20, 40, 60)):
        assert m.kv_lens.cpu().tolist() == [k]
        assert m.slot_mapping.cpu().tolist() == [[1, 2, 3, 4][(k - 1) // P] * P + (k - 1) % P]


def test_reference_errors_before_launch():
    bt = DeviceBlockTables(4, 4, 16, num_blocks=64, device=DEV, max_tokens=32)
    bt.bind(0, [1, 2])
    bt.bind(1, [3, 4, 5, 6])
    with pytest.raises(ValueError, match="empty sequence list"):
        bt.build_batch_meta([], [], [])
    with pytest.raises(ValueError, match="contributes 0 tokens"):
        bt.build_batch_meta([0], [0], [5])
    with pytest.raises(ValueError, match="holds only"):
        bt.build_batch_meta([0], [6], [5])
    with pytest.raises(ValueError, match="blocks hold fewer than kv_len=33"):
        bt.build_batch_meta([0], [1], [33])
    with pytest.raises(ValueError, match="rows outside"):
        bt.build_batch_meta([4], [1], [1])
    with pytest.raises(ValueError, match="max_tokens"):
        bt.build_batch_meta([1], [40], [40])
    with pytest.raises(IndexError, match="block ids outside"):
        bt.extend(0, [64])
    with pytest.raises(IndexError, match="page 5 does not exist"):
        bt.set_block(0, 5, 3)
    with pytest.raises(ValueError, match="exceed max_pages"):
        bt.extend(0, [5, 6, 7])
    assert bt.n_builds == 0
    m = bt.build_batch_meta([0], [1], [32])  # still usable
    torch.cuda.synchronize()
    assert m.slot_mapping.cpu().tolist() == [2 * 16 + 15]
    bt.check_status()


def test_device_side_checks_flag_without_faulting():
    """Inputs that bypass the host wrapper (the C ABI called directly): a table
    edit and a row outside the table are skipped and flagged; the bad sequence
    gets no pages and slot -1."""
    import ctypes

    from llm_serving_layer_b200 import _native as N

    bt = DeviceBlockTables(4, 4, 16, num_blocks=64, device=DEV)
    bt.bind(0, [7, 8])
    bt.build_batch_meta([0], [1], [20])
    slot = bt._ring[bt._next]
    # rows [0, 9, 0], query lengths [1, 1, 1], kv lengths [20, 20, 17], one edit (row 9, page 1, block 5)
    words = np.asarray([0, 9, 0, 1, 1, 1, 20, 20, 17, 9, 1, 5], dtype=np.int32)
    slot.host_np[: words.shape[0]] = words
    rc = N.lib().pkv_build_batch_meta(bt._desc_ref, slot.host.data_ptr(), slot.dev.data_ptr(), 3, 1,
                                      slot.desc_ref, bt._status_ptr, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    b, off = slot.i32, slot.off
    assert b[off["kv_indptr"]:off["kv_indptr"] + 4].cpu().tolist() == [0, 2, 2, 4]
    assert b[off["kv_indices"]:off["kv_indices"] + 4].cpu().tolist() == [7, 8, 7, 8]
    assert b[off["slot_mapping"]:off["slot_mapping"] + 3].cpu().tolist() == [8 * 16 + 3, -1, 8 * 16 + 0]
    with pytest.raises(N.PkvError, match="page table inconsistent"):
        bt.check_status()
    assert bt.table.cpu()[0, :2].tolist() == [7, 8]


@pytest.mark.parametrize("qlens", [[1] * 9, [1, 40, 1, 7, 1, 1, 100, 1, 1], [5, 40, 3, 7, 2, 9, 100, 8, 2]])
@pytest.mark.parametrize("validate", ["host", "device"])
def test_attention_over_device_meta_equals_host_meta(qlens, validate, monkeypatch):
    rs = np.random.RandomState(len(qlens) + sum(qlens))
    P, NB, L = 16, 2048, 2
    hist = rs.randint(0, 700, size=len(qlens))
    kv = hist + np.asarray(qlens)
    pages = (kv + P - 1) // P
    ids = rs.permutation(NB)[: int(pages.sum())]
    tables = [t.tolist() for t in np.split(ids, np.cumsum(pages)[:-1])]
    bk = B200PagedBackend(L, NB, P, 8, 32, 64, device=DEV, validate=validate)
    g = torch.Generator(device=DEV).manual_seed(3)
    bk._pool.copy_((torch.randn(bk._pool.shape, generator=g, device=DEV) * 0.7).half())
    hm = build_meta(tables, kv, qlens, P, device=DEV)
    T = int(sum(qlens))
    q = torch.randn(T, 32, 64, generator=g, device=DEV).half()
    want = bk.attend(q, 1, 0.125, hm)
    bt = DeviceBlockTables(16, 64, P, num_blocks=NB, device=DEV, status=bk._status)
    for r, t in enumerate(tables):
        bt.bind(r, t)
    dm = bt.build_batch_meta(range(len(qlens)), qlens, kv)
    bk.invalidate_plan()
    if validate == "host":  # the assembler's checks stand in for the read-back
        monkeypatch.setattr(bk, "_host_validate", lambda *a: pytest.fail("page table read back"))
    got = bk.attend(q, 1, 0.125, dm)
    torch.cuda.synchronize()
    bk.check_status()
    assert bk.last_kernel == ("decode" if max(qlens) == 1 else "prefill")
    assert torch.equal(got, want)


@pytest.mark.parametrize("fused", [False, True])
def test_pipelined_decode_steps_match_oracle(fused):
    """The serving loop's fast path, checked step by step against the oracle:
    BatchMeta from DeviceBlockTables (new blocks recorded as sequences cross
    into a new page), the next step planned (``plan``) right after this step's
    layers are issued, outputs written into one buffer through ``out=``, four
    decode steps of 3 layers over a skewed batch."""
    rs = np.random.RandomState(21 + fused)
    P, NB, L, Hkv, Hq, D = 16, 3000, 3, 8, 32, 64
    n = 40
    ctx = np.clip(np.round(rs.lognormal(np.log(120), 0.9, size=n)), 1, 900).astype(int)
    steps = 4
    pages = (ctx + steps + P - 1) // P
    ids = rs.permutation(NB)[: int(pages.sum())]
    tables = [t.tolist() for t in np.split(ids, np.cumsum(pages)[:-1])]
    bk = B200PagedBackend(L, NB, P, Hkv, Hq, D, device=DEV, dtype=torch.float16, validate="device")
    g = torch.Generator(device=DEV).manual_seed(5)
    bk._pool.copy_((torch.randn(bk._pool.shape, generator=g, device=DEV) * 0.7).half())
    bt = DeviceBlockTables(n, int(pages.max()), P, NB, device=DEV, status=bk._status)
    rows = np.arange(n)
    for r in range(n):
        bt.bind(r, tables[r][: (int(ctx[r]) - 1 + P - 1) // P])  # history before the first new token
    out = torch.empty((L, n, Hq, D), dtype=torch.float16, device=DEV)
    kv = ctx.copy()
    bt.extend_to(rows, kv, tables)
    m = bt.build_batch_meta(rows, np.ones(n), kv)
    for step in range(steps):
        q = torch.randn(L, n, Hq, D, generator=g, device=DEV).half()
        k = (torch.randn(L, n, Hkv, D, generator=g, device=DEV) * 0.7).half()
        v = (torch.randn(L, n, Hkv, D, generator=g, device=DEV) * 0.7).half()
        for layer in range(L):
            if fused:
                bk.append_attend(layer, k[layer], v[layer], q[layer], 0.125, m, out=out[layer])
            else:
                bk.append_kv(layer, k[layer], v[layer], m)
                bk.attend(q[layer], layer, 0.125, m, out=out[layer])
        host = build_meta(tables, kv, [1] * n, P)  # the checker's view of this step
        nkv = kv + 1
        bt.extend_to(rows, nkv, tables)
        nm = bt.build_batch_meta(rows, np.ones(n), nkv)
        bk.plan(nm)  # planned while this step's kernels may still run
        torch.cuda.synchronize()
        bk.check_status()
        for layer in range(L):
            want = attend_exact(q[layer].cpu().numpy(), bk.k_pool[layer].cpu().numpy(),
                                bk.v_pool[layer].cpu().numpy(), 0.125, host)
            err = float(np.abs(out[layer].float().cpu().numpy() - want).max())
            assert err <= 2e-3, f"step {step} layer {layer}: {err}"
        kv, m = nkv, nm
