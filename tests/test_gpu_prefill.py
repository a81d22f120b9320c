"""
GPU parity of the chunked-prefill path (tensor-core prefill kernel) against the
CPU oracle's float64 evaluation (``oracle.attend_exact``).

Bars: max-abs 2e-3 for fp16 pools, 1e-2 for bf16.
Cases: first and later 512-token chunks, ragged chunks around tile and page
boundaries, prefill mixed with decode tokens, every GQA group size, poisoned
(including NaN) unwritten page tails, many small tiles, and a radix-sharing
step — several block tables referencing the same prefix blocks, the partial
last prefix block copied on write (``RadixCache.ensure_writable`` →
``copy_block``, ``serving/cache/radix.py:629-677``) — which must give exactly
what private copies of the same KV give.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import FifoAllocator, Seq, meta_for, slots_meta
from llm_serving_layer_b200 import B200PagedBackend

pytestmark = pytest.mark.gpu
TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}


@pytest.fixture(scope="module", autouse=True)
def cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device (run with -m 'not gpu' on CPU)"
    torch.cuda.init()


def build_step(seed, specs, num_blocks, dtype=torch.float16, Hkv=8, Hq=32, D=64, poison=None,
               kv_std=0.5 ** 0.5, layers=1, validate="host"):
    """One prefill step over a seeded, scattered pool. ``specs`` lists
    (tokens already cached, tokens in this step's chunk) per sequence: the
    cached prefix is written by one history append, the chunk's K/V by the
    step's own append_kv (as the engine does before attend)."""
    rs = np.random.RandomState(seed)
    alloc = FifoAllocator(num_blocks, 16, order=rs.permutation(num_blocks))
    bk = B200PagedBackend(layers, num_blocks, 16, Hkv, Hq, D, device="cuda:0", dtype=dtype, validate=validate)
    if poison is not None:
        for l in range(layers):
            bk.k_pool[l].fill_(poison)
            bk.v_pool[l].fill_(poison)
    seqs = []
    for i, (s, _) in enumerate(specs):
        sq = Seq(alloc, i)
        if s:
            sq.append(s)
        seqs.append(sq)
    g = torch.Generator(device="cuda:0").manual_seed(seed)
    hist = [np.asarray([sq.slot_for(p) for p in range(sq.num_tokens)], dtype=np.int64) for sq in seqs]
    hs = np.concatenate(hist) if hist else np.zeros(0, np.int64)
    for l in range(layers):
        if hs.size:
            k = (torch.randn(hs.size, Hkv, D, generator=g, device="cuda:0") * kv_std).to(dtype)
            v = (torch.randn(hs.size, Hkv, D, generator=g, device="cuda:0") * kv_std).to(dtype)
            bk.append_kv(l, k, v, slots_meta(hs))
    qlens = [q for _, q in specs]
    for sq, q in zip(seqs, qlens):
        sq.append(q)
    m = meta_for(seqs, qlens, device="cuda:0")
    T = sum(qlens)
    for l in range(layers):
        kn = (torch.randn(T, Hkv, D, generator=g, device="cuda:0") * kv_std).to(dtype)
        vn = (torch.randn(T, Hkv, D, generator=g, device="cuda:0") * kv_std).to(dtype)
        bk.append_kv(l, kn, vn, m)
    q = torch.from_numpy(rs.standard_normal((T, Hq, D))).to(dtype)
    return bk, seqs, m, q


def exact(bk, q, m, scale, layer=0):
    """float64 attention over the backend's own pool (pages the step references,
    renumbered in listed order)."""
    from oracle import attend_exact
    from llm_serving_layer_b200 import build_meta
    idx = m.kv_indices.long()
    kp = bk.k_pool[layer][idx].double().cpu().numpy()
    vp = bk.v_pool[layer][idx].double().cpu().numpy()
    ip = m.kv_indptr.cpu().numpy()
    return attend_exact(q.double().cpu().numpy(), kp, vp, scale, build_meta(
        None, m.kv_lens.cpu().numpy(), m.query_lens.cpu().numpy(), bk.block_size,
        kv_indptr=ip, kv_indices=np.arange(ip[-1])))


def check(bk, m, q, dtype=torch.float16, scale=0.125, layer=0):
    out = bk.attend(q.cuda(), layer, scale, m)
    torch.cuda.synchronize()
    bk.check_status()
    assert bk.last_kernel == "prefill", f"{bk.last_kernel} kernel ran, not the prefill kernel"
    got = out.double().cpu().numpy()
    assert np.isfinite(got).all()
    err = np.abs(got - exact(bk, q, m, scale, layer)).max()
    assert err <= TOL[dtype], f"max |gpu - fp64| = {err:.3g}"
    return out


def _rand_specs(seed, n, s_max, q_max, q_min=1):
    rs = np.random.RandomState(1000 + seed)
    return [(int(rs.randint(0, s_max + 1)), int(rs.randint(q_min, q_max + 1))) for _ in range(n)]


CASES = {
    "first_chunk_512": [(0, 512)],
    "second_chunk_512": [(512, 512)],
    "chunk_after_odd_prefix": [(700, 311)],
    "full_prompt_1024": [(0, 1024)],
    "tile_and_page_edges": [(0, 1), (5, 3), (16, 16), (17, 15), (31, 33), (15, 17), (0, 2), (32, 31)],
    "ragged_8": _rand_specs(3, 8, 1000, 600),
    "many_small_tiles": _rand_specs(4, 300, 200, 40),
    "mixed_with_decode": [(int(s), 1) for s in np.random.RandomState(5).randint(1, 2048, 60)]
                         + [(300, 512), (0, 200), (1000, 17)],
}


@pytest.mark.parametrize("name", list(CASES))
def test_prefill_kernel_fp16_vs_fp64(name):
    specs = CASES[name]
    need = sum((s + q + 15) // 16 for s, q in specs) + 8
    bk, seqs, m, q = build_step(list(CASES).index(name), specs, max(need * 2, 64))
    check(bk, m, q)


def test_prefill_kernel_bf16():
    bk, seqs, m, q = build_step(7, _rand_specs(7, 6, 900, 500), 2048, dtype=torch.bfloat16)
    check(bk, m, q, dtype=torch.bfloat16)


@pytest.mark.parametrize("Hkv,Hq", [(8, 8), (8, 16), (4, 32), (2, 8), (1, 4)])
def test_prefill_kernel_gqa_groups(Hkv, Hq):
    bk, seqs, m, q = build_step(10 + Hq, _rand_specs(10 + Hq, 5, 400, 300), 1024, Hkv=Hkv, Hq=Hq)
    check(bk, m, q)


@pytest.mark.parametrize("poison", [1e3, float("nan")])
def test_unwritten_page_tail_never_reaches_the_output(poison):
    """Every pool slot no append wrote holds the poison; the last pages of the
    sequences are partial, so only masking keeps it out (the reference tests
    use 1e3; NaN would survive a 0 * NaN product)."""
    specs = [(3, 10), (0, 45), (29, 2), (100, 61)]
    bk, seqs, m, q = build_step(21, specs, 64, poison=poison)
    check(bk, m, q)
    # the decode kernel over the same pool and sequences keeps them out too
    md = meta_for(seqs, [1] * len(seqs), device="cuda:0")
    qd = torch.randn(len(seqs), 32, 64).half()
    out = bk.attend(qd.cuda(), 0, 0.125, md)
    torch.cuda.synchronize()
    assert bk.last_kernel == "decode"
    err = np.abs(out.double().cpu().numpy() - exact(bk, qd, md, 0.125)).max()
    assert err <= 2e-3


def test_prefill_layers_share_one_plan_and_are_deterministic():
    bk, seqs, m, q = build_step(31, _rand_specs(31, 12, 700, 300), 4096, layers=3)
    outs = [check(bk, m, q, layer=l) for l in range(3)]
    again = bk.attend(q.cuda(), 1, 0.125, m)
    torch.cuda.synchronize()
    assert bk.n_plans == 1 and bk.n_runs == 4
    assert torch.equal(outs[1], again)
    assert not torch.equal(outs[0], outs[1])


def test_radix_shared_prefix_with_copy_on_write_matches_private_copies():
    """Four families; each family's members reference the same full prefix
    blocks, and the partial last prefix block is copied on write before each
    member appends its own suffix. A chunk step over all members must equal,
    bit for bit, the same step over a pool where every member owns private
    copies of the same KV."""
    Hkv, Hq, D, P = 8, 32, 64, 16
    rs = np.random.RandomState(41)
    NB = 512
    g = torch.Generator(device="cuda:0").manual_seed(41)
    fams = [(int(rs.randint(64, 200)), [int(x) for x in rs.randint(20, 300, size=3)]) for _ in range(4)]

    def kv(n):
        return ((torch.randn(n, Hkv, D, generator=g, device="cuda:0") * 0.7).half(),
                (torch.randn(n, Hkv, D, generator=g, device="cuda:0") * 0.7).half())

    data = [(kv(pre), [kv(x) for x in tails]) for pre, tails in fams]
    q_all = torch.randn(sum(sum(t) for _, t in fams), Hq, D, generator=g, device="cuda:0").half()

    def run(shared):
        bk = B200PagedBackend(1, NB, P, Hkv, Hq, D, device="cuda:0", dtype=torch.float16)
        alloc = FifoAllocator(NB, P, order=np.random.RandomState(42).permutation(NB))
        seqs, qlens, new_k, new_v = [], [], [], []
        cows = 0
        for (pre, tails), ((pk, pv), tkv) in zip(fams, data):
            owner = Seq(alloc)
            owner.append(pre)
            bk.append_kv(0, pk, pv, slots_meta([owner.slot_for(p) for p in range(pre)]))
            for j, ((tk, tv), tl) in enumerate(zip(tkv, tails)):
                s = Seq(alloc, len(seqs))
                if shared:
                    # attach_prefix: reference the owner's blocks; COW the partial last one
                    s.block_ids = list(owner.block_ids)
                    s.num_tokens = pre
                    if pre % P:
                        new = alloc.allocate(1)[0]
                        bk.copy_block(s.block_ids[-1], new)
                        s.block_ids[-1] = new
                        cows += 1
                else:
                    s.append(pre)
                    bk.append_kv(0, pk, pv, slots_meta([s.slot_for(p) for p in range(pre)]))
                s.append(tl)
                seqs.append(s)
                qlens.append(tl)
                new_k.append(tk)
                new_v.append(tv)
        m = meta_for(seqs, qlens, device="cuda:0")
        bk.append_kv(0, torch.cat(new_k), torch.cat(new_v), m)
        out = bk.attend(q_all, 0, 0.125, m)
        torch.cuda.synchronize()
        bk.check_status()
        assert bk.last_kernel == "prefill"
        return bk, m, out, cows

    bk_s, m_s, out_s, cows = run(True)
    assert cows == sum(len(t) for pre, t in fams if pre % P)
    _, _, out_p, _ = run(False)
    assert torch.equal(out_s, out_p)
    err = np.abs(out_s.double().cpu().numpy() - exact(bk_s, q_all.cpu(), m_s, 0.125)).max()
    assert err <= 2e-3


@pytest.mark.parametrize("validate", ["host", "device"])
def test_mixed_batch_decode_rows_take_the_decode_kernel(validate):
    """A mixed step (decode rows + prefill chunks): the q_len == 1 rows are listed
    by the plan and run on the decode kernel (a second launch), the rest on the
    prefill kernel — in device-validate mode too, where the backend cannot see
    the query lengths. Long decode histories make the decode kernel split them."""
    rs = np.random.RandomState(77)
    specs = ([(int(x), 1) for x in rs.randint(1, 2048, 200)] + [(0, 300), (700, 40), (5, 2)]
             + [(int(x), 1) for x in rs.randint(1, 64, 50)])
    need = sum((s + q + 15) // 16 for s, q in specs) + 8
    bk, seqs, m, q = build_step(78, specs, need * 2, validate=validate)
    out = check(bk, m, q)
    again = bk.attend(q.cuda(), 0, 0.125, m)
    torch.cuda.synchronize()
    assert torch.equal(out, again)
