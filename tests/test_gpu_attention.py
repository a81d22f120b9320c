"""
GPU parity of the attention path (append_kv + attend) against the CPU oracle.

Bars: KV-append bit-exact; attention within the stated max-abs tolerance of
the float64 evaluation (``oracle.attend_exact``): 2e-3 for fp16 pools (the
north-star bar), 1e-5 for fp32 pools (the reference tests' TOL), 1e-2 for bf16.
Cases: every golden fixture produced by the reference, the reference tests'
known-answer scenarios (GQA maps, isolation, straddle, page order, causality,
mixed batches), and seeded ragged decode batches large enough that the decode
kernel splits sequences across CTAs.
"""

from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest
import torch

from cases import attn_cases
from helpers import FifoAllocator, Seq, meta_for, slots_meta
from llm_serving_layer_b200 import B200PagedBackend, build_meta
from oracle import OraclePool, attend_exact

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"
TDT = {"float16": torch.float16, "float32": torch.float32, "bfloat16": torch.bfloat16,
       "float64": torch.float64}
ATOL = {torch.float16: 2e-3, torch.float32: 1e-5, torch.bfloat16: 1e-2, torch.float64: 1e-10}


@pytest.fixture(scope="module", autouse=True)
def cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device (run with -m 'not gpu' on CPU)"
    torch.cuda.init()


def run_case_gpu(c, validate="host"):
    dt = TDT[c.dtype]
    bk = B200PagedBackend(1, c.num_blocks, c.block_size, c.n_kv_heads, c.n_heads, c.head_dim,
                          device="cuda:0", dtype=dt, validate=validate)
    if c.poison is not None:
        bk.k_pool[0].fill_(c.poison)
        bk.v_pool[0].fill_(c.poison)
    hs = c.slots("hist")
    if hs.size:
        bk.append_kv(0, torch.from_numpy(c.k_hist).cuda(), torch.from_numpy(c.v_hist).cuda(), slots_meta(hs))
    m = build_meta(c.tables, c.kv_lens, c.qlens, c.block_size, device="cuda:0")
    bk.append_kv(0, torch.from_numpy(c.k_new).cuda(), torch.from_numpy(c.v_new).cuda(), m)
    out = bk.attend(torch.from_numpy(c.q).cuda(), 0, c.scale, m)
    torch.cuda.synchronize()
    bk.check_status()
    return bk, m, out


def oracle_case(c):
    pool = OraclePool(1, c.num_blocks, c.block_size, c.n_kv_heads, c.head_dim, dtype=c.np_dtype)
    if c.poison is not None:
        pool.k[0][:] = c.poison
        pool.v[0][:] = c.poison
    hs = c.slots("hist")
    if hs.size:
        pool.append_kv(0, c.k_hist, c.v_hist, hs)
    m = build_meta(c.tables, c.kv_lens, c.qlens, c.block_size)
    pool.append_kv(0, c.k_new, c.v_new, m.slot_mapping.numpy())
    return pool, m


@pytest.mark.parametrize("case", attn_cases(), ids=lambda c: c.name)
def test_golden_cases(case):
    c = case.materialise()
    f = np.load(GOLD / f"{c.name}.npz")
    assert str(f["checksum"]) == c.checksum()
    bk, m, out = run_case_gpu(c)
    pool, mh = oracle_case(c)
    # append: bit-exact against the oracle's scatter (and the reference's pool)
    assert np.array_equal(bk.k_pool[0].cpu().numpy(), pool.k[0])
    assert np.array_equal(bk.v_pool[0].cpu().numpy(), pool.v[0])
    if f["k_pool"].size:
        assert np.array_equal(bk.k_pool[0].cpu().numpy(), f["k_pool"])
    exact = attend_exact(c.q, pool.k[0], pool.v[0], c.scale, mh)
    got = out.float().cpu().numpy().astype(np.float64)
    err = np.abs(got - exact).max()
    assert err <= ATOL[TDT[c.dtype]], f"max |gpu - fp64| = {err:.3g}"
    # and close to the reference's own output (fp16 probs rounding on its side)
    ref_err = np.abs(got - f["out"].astype(np.float64)).max()
    assert ref_err <= (4e-3 if c.dtype == "float16" else 2e-5)


def random_decode(seed, n, max_ctx, num_blocks, dtype=torch.float16, Hkv=8, Hq=32, D=64, P=16,
                  lognormal=False, kv_std=0.5 ** 0.5):
    """A decode step over a seeded, scattered pool: history written by one
    append, then one new token per sequence appended through the step's meta."""
    rs = np.random.RandomState(seed)
    if lognormal:
        ctx = np.clip(np.round(rs.lognormal(math.log(256) - 0.32, 0.8, size=n)), 1, max_ctx).astype(int)
    else:
        ctx = rs.randint(1, max_ctx + 1, size=n)
    alloc = FifoAllocator(num_blocks, P, order=rs.permutation(num_blocks))
    seqs = []
    for i, c in enumerate(ctx):
        s = Seq(alloc, i)
        s.append(int(c))
        seqs.append(s)
    bk = B200PagedBackend(1, num_blocks, P, Hkv, Hq, D, device="cuda:0", dtype=dtype)
    hist = [np.asarray([s.slot_for(p) for p in range(s.num_tokens - 1)], dtype=np.int64) for s in seqs]
    hist_slots = np.concatenate(hist)
    T = hist_slots.size
    g = torch.Generator(device="cuda:0").manual_seed(seed)
    if T:
        k = (torch.randn(T, Hkv, D, generator=g, device="cuda:0") * kv_std).to(dtype)
        v = (torch.randn(T, Hkv, D, generator=g, device="cuda:0") * kv_std).to(dtype)
        bk.append_kv(0, k, v, slots_meta(hist_slots))
    m = meta_for(seqs, [1] * n, device="cuda:0")
    kn = (torch.randn(n, Hkv, D, generator=g, device="cuda:0") * kv_std).to(dtype)
    vn = (torch.randn(n, Hkv, D, generator=g, device="cuda:0") * kv_std).to(dtype)
    q = torch.from_numpy(rs.standard_normal((n, Hq, D))).to(dtype)
    bk.append_kv(0, kn, vn, m)
    return bk, seqs, m, q


def exact_from_backend(bk, q, m, scale):
    """float64 attention over the backend's own pool (only the pages the step
    references are pulled back, renumbered in order)."""
    idx = m.kv_indices.long()
    kp = bk.k_pool[0][idx].float().cpu().numpy()
    vp = bk.v_pool[0][idx].float().cpu().numpy()
    ip = m.kv_indptr.cpu().numpy()
    return attend_exact(q.float().cpu().numpy(), kp, vp, scale, build_meta(
        None, m.kv_lens.cpu().numpy(), m.query_lens.cpu().numpy(), bk.block_size,
        kv_indptr=ip, kv_indices=np.arange(ip[-1])))


@pytest.mark.parametrize("seed,n,max_ctx,blocks", [
    (0, 1, 5, 64), (1, 3, 40, 64), (2, 37, 300, 1024), (3, 160, 2048, 16000), (4, 600, 64, 4096),
])
def test_decode_kernel_fp16_vs_fp64(seed, n, max_ctx, blocks):
    bk, seqs, m, q = random_decode(seed, n, max_ctx, blocks)
    out = bk.attend(q.cuda(), 0, 0.125, m)
    torch.cuda.synchronize()
    bk.check_status()
    assert bk.n_plans == 1, "decode path (planned split-K kernel) was not taken"
    exact = exact_from_backend(bk, q, m, 0.125)
    err = np.abs(out.float().cpu().numpy() - exact).max()
    assert err <= 2e-3, f"max |gpu - fp64| = {err:.3g}"


def test_decode_kernel_lognormal_batch256():
    """Config-2 shape at one layer: lognormal lengths (mean ~258), cap 2048."""
    bk, seqs, m, q = random_decode(11, 256, 2048, 20000, lognormal=True)
    out = bk.attend(q.cuda(), 0, 0.125, m)
    torch.cuda.synchronize()
    bk.check_status()
    exact = exact_from_backend(bk, q, m, 0.125)
    assert np.abs(out.float().cpu().numpy() - exact).max() <= 2e-3


def test_decode_kernel_bf16():
    bk, seqs, m, q = random_decode(5, 64, 700, 4096, dtype=torch.bfloat16)
    out = bk.attend(q.cuda(), 0, 0.125, m)
    torch.cuda.synchronize()
    bk.check_status()
    exact = exact_from_backend(bk, q, m, 0.125)
    assert np.abs(out.float().cpu().numpy() - exact).max() <= 1e-2


@pytest.mark.parametrize("groups", [1, 2, 8])
def test_decode_kernel_other_gqa_groups(groups):
    Hkv = 8 if groups < 8 else 4
    bk, seqs, m, q = random_decode(20 + groups, 19, 200, 1024, Hkv=Hkv, Hq=Hkv * groups)
    out = bk.attend(q.cuda(), 0, 0.125, m)
    torch.cuda.synchronize()
    bk.check_status()
    exact = exact_from_backend(bk, q, m, 0.125)
    assert np.abs(out.float().cpu().numpy() - exact).max() <= 2e-3


def test_decode_repeated_layers_leave_counters_clean():
    """16 layers of one step reuse one plan; the split-K counters are left at
    zero by every launch, so repeated steps give identical results."""
    bk, seqs, m, q = random_decode(7, 200, 1500, 20000)
    first = bk.attend(q.cuda(), 0, 0.125, m)
    for _ in range(15):
        again = bk.attend(q.cuda(), 0, 0.125, m)
    torch.cuda.synchronize()
    bk.check_status()
    assert torch.equal(first, again)
    assert bk.n_plans == 1 and bk.n_runs == 16


# --- the reference tests' known-answer scenarios, on the GPU kernels ----------


@pytest.mark.parametrize("geom", [(2, 6, 8, torch.float32), (8, 32, 64, torch.float16)])
def test_gqa_value_mapping_is_floor_divide(geom):
    Hkv, Hq, D, dt = geom
    groups = Hq // Hkv
    bk = B200PagedBackend(1, 8, 16, Hkv, Hq, D, device="cuda:0", dtype=dt)
    alloc = FifoAllocator(8, 16)
    s = Seq(alloc)
    s.append(1)
    m = meta_for([s], [1], "cuda:0")
    v = torch.zeros(1, Hkv, D, dtype=dt)
    for j in range(Hkv):
        v[0, j] = j + 1
    bk.append_kv(0, torch.zeros_like(v).cuda(), v.cuda(), m)
    out = bk.attend(torch.randn(1, Hq, D, dtype=dt).cuda(), 0, 1.0, m).float().cpu()
    for h in range(Hq):
        assert torch.allclose(out[0, h], torch.full((D,), float(h // groups + 1))), h


@pytest.mark.parametrize("geom", [(2, 4, 8, torch.float32), (8, 32, 64, torch.float16)])
def test_gqa_key_mapping_is_floor_divide(geom):
    Hkv, Hq, D, dt = geom
    groups = Hq // Hkv
    bk = B200PagedBackend(1, 8, 16, Hkv, Hq, D, device="cuda:0", dtype=dt)
    s = Seq(FifoAllocator(8, 16))
    s.append(2)
    m = meta_for([s], [2], "cuda:0")
    k = torch.zeros(2, Hkv, D, dtype=dt)
    v = torch.zeros(2, Hkv, D, dtype=dt)
    for j in range(Hkv):
        k[0, j, j] = 50.0
        k[1, j, Hkv + j] = 50.0
        v[0, j] = 1.0
        v[1, j] = -1.0
    bk.append_kv(0, k.cuda(), v.cuda(), m)
    q = torch.zeros(2, Hq, D, dtype=dt)
    for h in range(Hq):
        q[:, h, h // groups] = 1.0
    out = bk.attend(q.cuda(), 0, 1.0, m).float().cpu()
    for h in range(Hq):
        assert out[1, h, 0] > 0.99, h


def test_gqa_mapping_in_decode_kernel():
    """The decode kernel (Llama geometry, q_len 1) maps query head h to KV head
    h // 4: one key per sequence, a distinct constant per KV head."""
    Hkv, Hq, D = 8, 32, 64
    bk = B200PagedBackend(1, 64, 16, Hkv, Hq, D, device="cuda:0", dtype=torch.float16)
    alloc = FifoAllocator(64, 16)
    seqs = [Seq(alloc, i) for i in range(5)]
    for s in seqs:
        s.append(1)
    m = meta_for(seqs, [1] * 5, "cuda:0")
    v = torch.zeros(5, Hkv, D, dtype=torch.float16)
    for i in range(5):
        for j in range(Hkv):
            v[i, j] = (i + 1) * 10 + j
    bk.append_kv(0, torch.zeros_like(v).cuda(), v.cuda(), m)
    out = bk.attend(torch.randn(5, Hq, D, dtype=torch.float16).cuda(), 0, 1.0, m).float().cpu()
    assert bk.n_plans == 1
    for i in range(5):
        for h in range(Hq):
            assert torch.all(out[i, h] == (i + 1) * 10 + h // 4), (i, h)


@pytest.mark.parametrize("dt", [torch.float32, torch.float16])
def test_sequences_do_not_see_each_others_kv(dt):
    Hkv, Hq, D = (2, 4, 8) if dt == torch.float32 else (8, 32, 64)
    bk = B200PagedBackend(1, 32, 16, Hkv, Hq, D, device="cuda:0", dtype=dt)
    alloc = FifoAllocator(32, 16)
    lengths = [3, 1, 20]
    seqs, vs = [], []
    for i, n in enumerate(lengths):
        s = Seq(alloc, i)
        s.append(n)
        seqs.append(s)
        vs.append(torch.full((n, Hkv, D), float(i + 1), dtype=dt))
    m = meta_for(seqs, lengths, "cuda:0")
    v = torch.cat(vs)
    bk.append_kv(0, torch.zeros_like(v).cuda(), v.cuda(), m)
    out = bk.attend(torch.randn(sum(lengths), Hq, D, dtype=dt).cuda(), 0, 1.0, m).float().cpu()
    cu = m.cu_query_lens.tolist()
    for i in range(3):
        seg = out[cu[i]: cu[i + 1]]
        assert torch.allclose(seg, torch.full_like(seg, float(i + 1)), atol=1e-5)
    # and the decode kernel (one query each) keeps them apart too
    md = meta_for(seqs, [1, 1, 1], "cuda:0")
    od = bk.attend(torch.randn(3, Hq, D, dtype=dt).cuda(), 0, 1.0, md).float().cpu()
    for i in range(3):
        assert torch.allclose(od[i], torch.full_like(od[i], float(i + 1)), atol=1e-5)


@pytest.mark.parametrize("n", [1, 15, 16, 17, 31, 32, 33])
@pytest.mark.parametrize("qmode", ["prefill", "decode"])
def test_block_straddle_against_poisoned_pool(n, qmode):
    Hkv, Hq, D = 8, 32, 64
    rs = np.random.RandomState(n)
    bk = B200PagedBackend(1, 32, 16, Hkv, Hq, D, device="cuda:0", dtype=torch.float16)
    bk.k_pool[0].fill_(1e3)
    bk.v_pool[0].fill_(1e3)
    s = Seq(FifoAllocator(32, 16, order=rs.permutation(32)))
    s.append(n)
    ql = n if qmode == "prefill" else 1
    m = meta_for([s], [n], "cuda:0")
    k = torch.from_numpy(rs.standard_normal((n, Hkv, D))).half()
    v = torch.from_numpy(rs.standard_normal((n, Hkv, D))).half()
    bk.append_kv(0, k.cuda(), v.cuda(), m)
    mq = meta_for([s], [ql], "cuda:0")
    q = torch.from_numpy(rs.standard_normal((ql, Hq, D))).half()
    out = bk.attend(q.cuda(), 0, 0.125, mq)
    torch.cuda.synchronize()
    exact = exact_from_backend(bk, q, mq, 0.125)
    assert np.abs(out.float().cpu().numpy() - exact).max() <= 2e-3


@pytest.mark.parametrize("qmode", ["prefill", "decode"])
def test_non_contiguous_pages_bit_identical_to_contiguous(qmode):
    Hkv, Hq, D = 8, 32, 64
    rs = np.random.RandomState(7)
    k = torch.from_numpy(rs.standard_normal((40, Hkv, D))).half()
    v = torch.from_numpy(rs.standard_normal((40, Hkv, D))).half()
    ql = 40 if qmode == "prefill" else 1
    q = torch.from_numpy(rs.standard_normal((ql, Hq, D))).half().cuda()
    outs = []
    for order in (None, [21, 4, 13] + [b for b in range(32) if b not in (21, 4, 13)],
                  [7, 3, 0] + [b for b in range(32) if b not in (7, 3, 0)]):
        bk = B200PagedBackend(1, 32, 16, Hkv, Hq, D, device="cuda:0", dtype=torch.float16)
        s = Seq(FifoAllocator(32, 16, order=order))
        s.append(40)
        bk.append_kv(0, k.cuda(), v.cuda(), meta_for([s], [40], "cuda:0"))
        outs.append(bk.attend(q, 0, 0.125, meta_for([s], [ql], "cuda:0")))
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])


def test_mixed_prefill_and_decode_matches_running_each_alone():
    Hkv, Hq, D = 8, 32, 64
    rs = np.random.RandomState(11)
    bk = B200PagedBackend(1, 64, 16, Hkv, Hq, D, device="cuda:0", dtype=torch.float16)
    alloc = FifoAllocator(64, 16, order=rs.permutation(64))
    hist = [6, 18, 16]
    seqs = []
    for i, h in enumerate(hist):
        s = Seq(alloc, i)
        s.append(h)
        seqs.append(s)
    hm = meta_for(seqs, hist, "cuda:0")
    T = sum(hist)
    bk.append_kv(0, torch.randn(T, Hkv, D).half().cuda(), torch.randn(T, Hkv, D).half().cuda(), hm)
    qlens = [4, 1, 1]
    for s, ql in zip(seqs, qlens):
        s.append(ql)
    m = meta_for(seqs, qlens, "cuda:0")
    bk.append_kv(0, torch.randn(6, Hkv, D).half().cuda(), torch.randn(6, Hkv, D).half().cuda(), m)
    q = torch.randn(6, Hq, D).half().cuda()
    batched = bk.attend(q, 0, 0.125, m)
    cu = m.cu_query_lens.tolist()
    for i, ql in enumerate(qlens):
        solo = bk.attend(q[cu[i]: cu[i + 1]], 0, 0.125, meta_for([seqs[i]], [ql], "cuda:0"))
        if ql > 1:  # same kernel either way: batching is invisible, bit for bit
            assert torch.equal(batched[cu[i]: cu[i + 1]], solo), i
        else:       # alone, a q_len-1 batch takes the decode kernel (fp16 P.V)
            assert (batched[cu[i]: cu[i + 1]].float() - solo.float()).abs().max() <= 2e-3, i


def test_prefill_query_cannot_attend_to_future_keys():
    Hkv, Hq, D = 8, 32, 64
    bk = B200PagedBackend(1, 32, 16, Hkv, Hq, D, device="cuda:0", dtype=torch.float16)
    s = Seq(FifoAllocator(32, 16))
    n = 6
    s.append(n)
    m = meta_for([s], [n], "cuda:0")
    bk.append_kv(0, torch.randn(n, Hkv, D).half().cuda(), torch.randn(n, Hkv, D).half().cuda(), m)
    q = torch.randn(n, Hq, D).half().cuda()
    base = bk.attend(q, 0, 0.125, m)
    slot = s.slot_for(n - 1)
    bk.k_pool[0].view(-1, Hkv, D)[slot] = 100.0
    bk.v_pool[0].view(-1, Hkv, D)[slot] = -999.0
    pois = bk.attend(q, 0, 0.125, m)
    assert torch.equal(base[: n - 1], pois[: n - 1])
    assert not torch.allclose(base[n - 1], pois[n - 1])


@pytest.mark.parametrize("dt", [torch.float32, torch.float16])
def test_decode_sees_the_token_just_appended(dt):
    Hkv, Hq, D = (2, 4, 8) if dt == torch.float32 else (8, 32, 64)
    bk = B200PagedBackend(1, 8, 16, Hkv, Hq, D, device="cuda:0", dtype=dt)
    s = Seq(FifoAllocator(8, 16))
    s.append(1)
    m = meta_for([s], [1], "cuda:0")
    bk.append_kv(0, torch.zeros(1, Hkv, D, dtype=dt).cuda(), torch.full((1, Hkv, D), 7.0, dtype=dt).cuda(), m)
    out = bk.attend(torch.randn(1, Hq, D, dtype=dt).cuda(), 0, 1.0, m)
    assert torch.allclose(out.float(), torch.full_like(out.float(), 7.0))


def test_append_lands_in_named_slots_only_and_is_idempotent():
    Hkv, D = 8, 64
    bk = B200PagedBackend(2, 32, 16, Hkv, 32, D, device="cuda:0", dtype=torch.float16)
    s = Seq(FifoAllocator(32, 16, order=np.random.RandomState(3).permutation(32)))
    s.append(20)
    m = meta_for([s], [20], "cuda:0")
    k = torch.randn(20, Hkv, D).half().cuda()
    v = torch.randn(20, Hkv, D).half().cuda()
    bk.append_kv(0, k, v, m)
    kf = bk.k_pool[0].view(-1, Hkv, D)
    vf = bk.v_pool[0].view(-1, Hkv, D)
    slots = m.slot_mapping.cpu().tolist()
    for t, sl in enumerate(slots):
        assert torch.equal(kf[sl], k[t]) and torch.equal(vf[sl], v[t])
    nz = set((kf.abs().sum(dim=(1, 2)) != 0).nonzero().flatten().tolist())
    assert nz == set(slots)
    assert bk.k_pool[1].abs().sum() == 0, "layer 1 disturbed"
    before = bk._pool.clone()
    bk.append_kv(0, k, v, m)
    assert torch.equal(bk._pool, before)


def test_validation_errors_match_the_reference():
    bk = B200PagedBackend(2, 8, 16, 2, 4, 8, device="cuda:0", dtype=torch.float32)
    s = Seq(FifoAllocator(8, 16))
    s.append(16)
    m = meta_for([s], [1], "cuda:0")
    with pytest.raises(ValueError, match="layer_idx"):
        bk.attend(torch.zeros(1, 4, 8).cuda(), 2, 1.0, m)
    with pytest.raises(ValueError, match="q has shape"):
        bk.attend(torch.zeros(1, 3, 8).cuda(), 0, 1.0, m)
    with pytest.raises(ValueError, match="k has shape"):
        bk.append_kv(0, torch.zeros(1, 3, 8).cuda(), torch.zeros(1, 3, 8).cuda(), m)
    import dataclasses
    bad = dataclasses.replace(m, kv_last_page_len=torch.tensor([9], dtype=torch.int32, device="cuda:0"))
    with pytest.raises(ValueError, match="kv_last_page_len"):
        bk.attend(torch.zeros(1, 4, 8).cuda(), 0, 1.0, bad)
    nos = dataclasses.replace(m, slot_mapping=None)
    with pytest.raises(ValueError, match="slot_mapping"):
        bk.append_kv(0, torch.zeros(1, 2, 8).cuda(), torch.zeros(1, 2, 8).cuda(), nos)
    lie = dataclasses.replace(m, is_prefill=True)
    with pytest.raises(ValueError, match="is_prefill"):
        bk.attend(torch.zeros(1, 4, 8).cuda(), 0, 1.0, lie)


def test_device_status_flags_bad_slots_and_tables():
    bk = B200PagedBackend(1, 8, 16, 8, 32, 64, device="cuda:0", dtype=torch.float16, validate="device")
    meta = slots_meta([5, 8 * 16 + 3])  # the second slot is outside the pool
    bk.append_kv(0, torch.ones(2, 8, 64).half().cuda(), torch.ones(2, 8, 64).half().cuda(), meta)
    with pytest.raises(RuntimeError, match="outside the pool"):
        bk.check_status()
    assert bk.k_pool[0].view(-1, 8, 64)[5].float().sum() == 8 * 64  # the valid slot landed
    # a page table whose last_page_len disagrees with kv_lens, decode kernel path
    s = Seq(FifoAllocator(8, 16))
    s.append(20)
    m = meta_for([s], [1], "cuda:0")
    import dataclasses
    bad = dataclasses.replace(m, kv_last_page_len=torch.tensor([3], dtype=torch.int32, device="cuda:0"))
    bk.attend(torch.zeros(1, 32, 64).half().cuda(), 0, 1.0, bad)
    with pytest.raises(RuntimeError, match="inconsistent"):
        bk.check_status()
    # a prefill-shaped batch mislabelled as decode is refused before any launch
    m2 = meta_for([s], [4], "cuda:0")
    lie = dataclasses.replace(m2, is_prefill=False)
    with pytest.raises(ValueError, match="one query per sequence"):
        bk.attend(torch.zeros(4, 32, 64).half().cuda(), 0, 1.0, lie)
    bk.check_status()
