"""
GPU parity of the byte-moving half of the path — copy_block (copy-on-write)
and the preemption swap — against the oracle and the reference's golden
vectors. Bar: bit-exact.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from cases import COPY_OPS, SWAP_GEOM, SWAP_TOKENS, copy_block_pool
from helpers import FifoAllocator, Seq
from llm_serving_layer_b200 import B200PagedBackend, B200SwapSpace, SwapSpaceFull
from oracle import OraclePool

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module", autouse=True)
def cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"


def make(num_layers=4, num_blocks=8, block_size=4, n_kv=2, n_heads=4, head_dim=8, dtype=torch.float32):
    return B200PagedBackend(num_layers, num_blocks, block_size, n_kv, n_heads, head_dim,
                            device="cuda:0", dtype=dtype)


def fill(bk, block, base):
    for layer in range(bk.num_layers):
        bk.k_pool[layer][block] = base + layer * 100
        bk.v_pool[layer][block] = base + layer * 100 + 50


# --- copy_block: tests/test_copy_block.py, on the CUDA kernel -------------------


def test_copy_block_golden():
    k, v = copy_block_pool()
    L, NB, P, H, D = k.shape
    bk = make(L, NB, P, H, 2 * H, D)
    for l in range(L):
        bk.k_pool[l].copy_(torch.from_numpy(k[l]))
        bk.v_pool[l].copy_(torch.from_numpy(v[l]))
    for s, d in COPY_OPS:
        bk.copy_block(s, d)
    f = np.load(GOLD / "copy_block.npz")
    assert np.array_equal(torch.stack(bk.k_pool).cpu().numpy(), f["k"])
    assert np.array_equal(torch.stack(bk.v_pool).cpu().numpy(), f["v"])


def test_copies_every_layer_not_alias_others_untouched():
    bk = make()
    for b in range(bk.num_blocks):
        fill(bk, b, float(b))
    keep = {b: bk.k_pool[1][b].clone() for b in range(bk.num_blocks) if b not in (1, 2)}
    bk.copy_block(1, 2)
    for layer in range(bk.num_layers):
        assert torch.equal(bk.k_pool[layer][2], bk.k_pool[layer][1])
        assert torch.equal(bk.v_pool[layer][2], bk.v_pool[layer][1])
    for b, want in keep.items():
        assert torch.equal(bk.k_pool[1][b], want)
    before = bk.k_pool[2][1].clone()
    bk.k_pool[2][2] += 99.0
    assert torch.equal(bk.k_pool[2][1], before)


def test_self_copy_is_a_noop_and_range_raises():
    bk = make()
    fill(bk, 3, 5.0)
    before = [bk.k_pool[i][3].clone() for i in range(bk.num_layers)]
    bk.copy_block(3, 3)
    for i, want in enumerate(before):
        assert torch.equal(bk.k_pool[i][3], want)
    for s, d in [(-1, 0), (0, -1), (999, 0), (0, 999)]:
        with pytest.raises(IndexError):
            bk.copy_block(s, d)


def test_copy_blocks_batched_llama_geometry_bit_exact():
    bk = make(16, 256, 16, 8, 32, 64, torch.float16)
    torch.manual_seed(0)
    bk._pool.copy_(torch.randn_like(bk._pool, dtype=torch.float32).half())
    rs = np.random.RandomState(0)
    perm = rs.permutation(256)
    src, dst = perm[:40].tolist(), perm[40:80].tolist()
    host = OraclePool(16, 256, 16, 8, 64, dtype=np.float16)
    for l in range(16):
        host.k[l][:] = bk.k_pool[l].cpu().numpy()
        host.v[l][:] = bk.v_pool[l].cpu().numpy()
    bk.copy_blocks(src, dst)
    for s, d in zip(src, dst):
        host.copy_block(s, d)
    torch.cuda.synchronize()
    bk.check_status()
    for l in range(16):
        assert np.array_equal(bk.k_pool[l].cpu().numpy(), host.k[l])
        assert np.array_equal(bk.v_pool[l].cpu().numpy(), host.v[l])
    with pytest.raises(ValueError, match="also a source"):
        bk.copy_blocks([1, 2], [2, 3])


# --- swap: tests/test_preemption.py:321-458, on the swap engine ------------------


def _fill_seq(bk, seq, base):
    for layer in range(bk.num_layers):
        for i, b in enumerate(seq.block_ids):
            bk.k_pool[layer][b] = base + layer * 100 + i
            bk.v_pool[layer][b] = -(base + layer * 100 + i)


def test_swap_golden_round_trip():
    f = np.load(GOLD / "swap_roundtrip.npz")
    g = SWAP_GEOM
    bk = B200PagedBackend(g["num_layers"], g["num_blocks"], g["block_size"], g["n_kv_heads"],
                          2 * g["n_kv_heads"], g["head_dim"], device="cuda:0", dtype=torch.float64)
    P, H, D = g["block_size"], g["n_kv_heads"], g["head_dim"]
    order = list(f["src_ids"]) + list(f["dst_ids"]) + list(f["decoy_ids"])
    order += [b for b in range(g["num_blocks"]) if b not in order]
    alloc = FifoAllocator(g["num_blocks"], P, order=order)
    src = Seq(alloc, 1)
    src.append(SWAP_TOKENS)
    assert src.block_ids == [int(b) for b in f["src_ids"]]
    for l in range(g["num_layers"]):
        for i, b in enumerate(src.block_ids):
            bk.k_pool[l][b] = 7.0 + l * 100 + i + torch.arange(P * H * D, dtype=torch.float64).view(P, H, D) / 1000
            bk.v_pool[l][b] = -(7.0 + l * 100 + i)
    sw = B200SwapSpace(bk)
    h = sw.swap_out("r", src)
    assert np.array_equal(h.k.numpy(), f["k_host"]) and np.array_equal(h.v.numpy(), f["v_host"])
    assert h.nbytes == int(f["nbytes"])
    dst_ids = [int(b) for b in f["dst_ids"]]
    for l in range(g["num_layers"]):
        for b in f["decoy_ids"]:
            bk.k_pool[l][int(b)] = -99.0
            bk.v_pool[l][int(b)] = -99.0
    dst = Seq(FifoAllocator(g["num_blocks"], P, order=dst_ids), 3)
    dst.append(h.num_tokens)
    sw.swap_in(h, dst)
    torch.cuda.synchronize()
    # every block the reference touched matches its pool after the round trip
    for l in range(g["num_layers"]):
        for b in dst_ids + [int(x) for x in f["decoy_ids"]]:
            assert np.array_equal(bk.k_pool[l][b].cpu().numpy(), f["k_pool"][l, b])
            assert np.array_equal(bk.v_pool[l][b].cpu().numpy(), f["v_pool"][l, b])
    bk.check_status()


@pytest.mark.parametrize("synchronous", [True, False])
def test_swap_round_trip_every_layer_into_different_blocks(synchronous):
    bk = make(2, 16, 4, 2, 4, 8)
    alloc = FifoAllocator(16, 4)
    sw = B200SwapSpace(bk, synchronous=synchronous)
    src = Seq(alloc, 1)
    src.append(10)
    _fill_seq(bk, src, 7.0)
    before = [(bk.k_pool[l][b].clone(), bk.v_pool[l][b].clone()) for l in range(2) for b in src.block_ids]
    orig = list(src.block_ids)
    h = sw.swap_out("r", src)
    src.free()
    # the freed blocks are reused at once and overwritten on the compute stream:
    # with an asynchronous swap the gather must already be ordered before this
    decoy = Seq(alloc, 2)
    decoy.block_ids = list(orig)
    decoy.num_tokens = 10
    _fill_seq(bk, decoy, -99.0)
    dst = Seq(alloc, 3)
    dst.append(h.num_tokens)
    assert set(dst.block_ids).isdisjoint(orig)
    sw.swap_in(h, dst)
    after = [(bk.k_pool[l][b], bk.v_pool[l][b]) for l in range(2) for b in dst.block_ids]
    for (gk, gv), (wk, wv) in zip(after, before):
        assert torch.equal(gk, wk) and torch.equal(gv, wv)
    sw.release(h)
    sw.release(h)
    assert sw.bytes_in_use == 0 and sw.num_swapped == 0


def test_swap_in_rejects_mismatch_and_budget_enforced():
    bk = make(2, 32, 4, 2, 4, 8)
    alloc = FifoAllocator(32, 4)
    sw = B200SwapSpace(bk)
    src = Seq(alloc, 1)
    src.append(9)
    h = sw.swap_out("r", src)
    src.free()
    wrong = Seq(alloc, 2)
    wrong.append(5)
    with pytest.raises(RuntimeError, match="resume mismatch"):
        sw.swap_in(h, wrong)
    same = Seq(alloc, 3)
    same.append(9)
    same.block_ids.pop()
    with pytest.raises(RuntimeError, match="blocks allocated"):
        sw.swap_in(h, same)
    freed = Seq(alloc, 4)
    freed.append(4)
    freed.free()
    with pytest.raises(RuntimeError, match="freed"):
        sw.swap_out("x", freed)
    one = sw.bytes_for(1)
    tight = B200SwapSpace(bk, max_bytes=2 * one)
    a = Seq(alloc, 5)
    a.append(8)
    ha = tight.swap_out("a", a)
    assert tight.bytes_in_use == 2 * one
    b = Seq(alloc, 6)
    b.append(4)
    with pytest.raises(SwapSpaceFull):
        tight.swap_out("b", b)
    tight.release(ha)
    tight.release(ha)
    assert tight.bytes_in_use == 0


def test_swap_many_sequences_llama_geometry_chunked():
    """Llama geometry, 12 victims of 100 tokens, staging smaller than one
    sequence (forces the chunked, double-buffered pipeline); async handles;
    restored into fresh blocks; bit-exact."""
    L, NB = 16, 512
    bk = B200PagedBackend(L, NB, 16, 8, 32, 64, device="cuda:0", dtype=torch.float16)
    torch.manual_seed(1)
    bk._pool.copy_(torch.randn(bk._pool.shape, device="cuda:0").half())
    alloc = FifoAllocator(NB, 16, order=np.random.RandomState(4).permutation(NB))
    sw = B200SwapSpace(bk, staging_bytes=5 * 16384, synchronous=False)
    seqs = []
    for i in range(12):
        s = Seq(alloc, i)
        s.append(100)
        seqs.append(s)
    want = [torch.stack([bk._pool[:, 0, b] for b in s.block_ids], 1).cpu() for s in seqs]
    handles = [sw.swap_out(f"r{i}", s) for i, s in enumerate(seqs)]
    for s in seqs:
        s.free()
    bk._pool.zero_()
    for h in handles:
        sw.wait(h)
        assert h.k.shape == (L, 7, 16, 8, 64)
    dsts = []
    for h in handles:
        d = Seq(alloc, 100)
        d.append(h.num_tokens)
        sw.swap_in(h, d)
        dsts.append(d)
    sw.wait()
    torch.cuda.synchronize()
    bk.check_status()
    for w, d, h in zip(want, dsts, handles):
        got = torch.stack([bk._pool[:, 0, b] for b in d.block_ids], 1).cpu()
        assert torch.equal(got, w)
        assert torch.equal(h.k, w)
        sw.release(h)


def test_swap_staging_ring_reuse_with_mixed_sizes():
    """Staging holding about three victims: several transfers share the ring
    at once, later chunks wrap to its start and wait only for the uses they
    overlap. Victims of mixed lengths, asynchronous handles, swap-outs and
    swap-ins interleaved; everything restored bit-exact into fresh blocks."""
    L, NB = 16, 1024
    bk = B200PagedBackend(L, NB, 16, 8, 32, 64, device="cuda:0", dtype=torch.float16)
    torch.manual_seed(3)
    bk._pool.copy_(torch.randn(bk._pool.shape, device="cuda:0").half())
    rs = np.random.RandomState(9)
    alloc = FifoAllocator(NB, 16, order=rs.permutation(NB))
    per_block = bk.block_bytes()
    sw = B200SwapSpace(bk, staging_bytes=3 * 7 * per_block, synchronous=False)
    seqs = []
    for i in range(14):
        s = Seq(alloc, i)
        s.append(int(rs.randint(20, 200)))
        seqs.append(s)
    want = [torch.stack([bk._pool[:, 0, b] for b in s.block_ids], 1).cpu() for s in seqs]
    handles, dsts = [], []
    for i, s in enumerate(seqs):
        handles.append(sw.swap_out(f"r{i}", s))
        s.free()
        if i % 3 == 2:  # a restore of an earlier victim between the swap-outs
            j = len(dsts)
            d = Seq(alloc, 100 + j)
            d.append(handles[j].num_tokens)
            sw.swap_in(handles[j], d)
            dsts.append(d)
    while len(dsts) < len(handles):
        j = len(dsts)
        d = Seq(alloc, 100 + j)
        d.append(handles[j].num_tokens)
        sw.swap_in(handles[j], d)
        dsts.append(d)
    sw.wait()
    torch.cuda.synchronize()
    bk.check_status()
    for w, d, h in zip(want, dsts, handles):
        got = torch.stack([bk._pool[:, 0, b] for b in d.block_ids], 1).cpu()
        assert torch.equal(got, w)
        assert torch.equal(h.k, w)
        sw.release(h)
