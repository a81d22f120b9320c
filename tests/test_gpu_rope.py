"""
Rotary position embedding in the backend: ``B200PagedBackend.rope`` (the
``pkv_rope`` kernel, one launch for q and k) and ``append_attend(...,
rope=(cos, sin))``, where a decode step rotates q and the new K rows inside its
single launch.

The engine applies RoPE at ``meta.positions`` to the projected q and k before
``append_kv`` / ``attend`` (``docs/ARCHITECTURE.md:167-172``). The rotation must
give the bits of the fp32 elementwise formula ``a*cos - b*sin, a*sin + b*cos``
rounded to the pool dtype (what ``RandomLlama`` computes with torch), and the
fused call must leave the same pool and return the same output, bit for bit,
as rotating first and then calling ``append_attend`` without ``rope``: for
decode steps (the fused launch) and for prefill / mixed steps (rotation kernel,
then the plain call), fp16 and bf16. A position outside the tables is reported.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from helpers import FifoAllocator, Seq, meta_for, slots_meta
from llm_serving_layer_b200 import B200PagedBackend
from llm_serving_layer_b200._native import PkvError
from llm_serving_layer_b200.llama import LlamaConfig, RandomLlama
from oracle import rope as oracle_rope  # the checker

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def tables(max_pos=4096, D=64, theta=500000.0):
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, device=DEV, dtype=torch.float32) / D))
    ang = torch.arange(max_pos, device=DEV, dtype=torch.float32)[:, None] * inv[None, :]
    return torch.cos(ang).contiguous(), torch.sin(ang).contiguous()


def torch_rope(x, pos, cos, sin):
    """The fp32 elementwise formula, as RandomLlama evaluates it."""
    half = x.shape[-1] // 2
    c, s = cos[pos.long()][:, None, :], sin[pos.long()][:, None, :]
    a, b = x[..., :half].float(), x[..., half:].float()
    return torch.cat([a * c - b * s, a * s + b * c], dim=-1).to(x.dtype)


def setup(seed, ctx, qlens, num_blocks=4096, dtype=torch.float16):
    """Two backends with identical pools holding each sequence's history, the
    step's meta and its (unrotated) q / k / v."""
    rs = np.random.RandomState(seed)
    alloc = FifoAllocator(num_blocks, 16, order=rs.permutation(num_blocks))
    seqs = []
    for i, (c, ql) in enumerate(zip(ctx, qlens)):
        s = Seq(alloc, i)
        s.append(int(c) - ql)
        seqs.append(s)
    hist = np.concatenate([[s.slot_for(p) for p in range(s.num_tokens)] for s in seqs]).astype(np.int64)
    g = torch.Generator(device=DEV).manual_seed(seed)
    bks = []
    for _ in range(2):
        bk = B200PagedBackend(2, num_blocks, 16, 8, 32, 64, device=DEV, dtype=dtype)
        bk._pool.fill_(3.0)
        bks.append(bk)
    if hist.size:
        k = (torch.randn(hist.size, 8, 64, generator=g, device=DEV) * 0.7).to(dtype)
        v = (torch.randn(hist.size, 8, 64, generator=g, device=DEV) * 0.7).to(dtype)
        for bk in bks:
            bk.append_kv(1, k, v, slots_meta(hist))
    for s, ql in zip(seqs, qlens):
        s.append(ql)
    m = meta_for(seqs, qlens, device=DEV)
    T = sum(qlens)
    kn = (torch.randn(T, 8, 64, generator=g, device=DEV) * 0.7).to(dtype)
    vn = (torch.randn(T, 8, 64, generator=g, device=DEV) * 0.7).to(dtype)
    q = torch.randn(T, 32, 64, generator=g, device=DEV).to(dtype)
    return bks, m, kn, vn, q


def counting_rope(bk):
    calls = []
    orig = bk.rope

    def wrapped(*args, **kw):
        calls.append(1)
        return orig(*args, **kw)

    bk.rope = wrapped
    return calls


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_rope_kernel_matches_the_fp32_formula_bitwise(dtype):
    cos, sin = tables()
    bk = B200PagedBackend(1, 64, 16, 8, 32, 64, device=DEV, dtype=dtype)
    g = torch.Generator(device=DEV).manual_seed(5)
    T = 777
    pos = torch.randint(0, 4096, (T,), generator=g, device=DEV)
    pos[:3] = torch.tensor([0, 1, 4095], device=DEV)

    class M:
        positions = pos

    q = (torch.randn(T, 32, 64, generator=g, device=DEV) * 3).to(dtype)
    k = (torch.randn(T, 8, 64, generator=g, device=DEV) * 3).to(dtype)
    qo, ko = bk.rope(q, k, M, (cos, sin))
    torch.cuda.synchronize()
    bk.check_status()
    assert torch.equal(qo, torch_rope(q, pos, cos, sin))
    assert torch.equal(ko, torch_rope(k, pos, cos, sin))
    if dtype == torch.float16:  # and the CPU oracle's restatement (numpy has no bf16)
        c, s_, p = cos.cpu().numpy(), sin.cpu().numpy(), pos.cpu().numpy()
        assert np.array_equal(qo.cpu().numpy(), oracle_rope(q.cpu().numpy(), p, c, s_))
        assert np.array_equal(ko.cpu().numpy(), oracle_rope(k.cpu().numpy(), p, c, s_))
    # one tensor alone
    qo2, none = bk.rope(q, None, M, (cos, sin))
    assert none is None and torch.equal(qo2, qo)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("case", ["lognormal", "split_long", "single_token"])
def test_fused_decode_rope_equals_rope_then_append_attend(case, dtype):
    rs = np.random.RandomState(11)
    ctx = {"lognormal": np.clip(np.round(rs.lognormal(math.log(256) - 0.32, 0.8, size=200)), 1, 2048).astype(int),
           "split_long": np.array([1900, 3, 17, 1200, 16, 33]),
           "single_token": np.array([1, 1, 1])}[case]
    bks, m, kn, vn, q = setup(7, ctx, [1] * len(ctx), dtype=dtype)
    cos, sin = tables()
    a, b = bks
    calls = counting_rope(b)
    q0, k0 = q.clone(), kn.clone()
    qr, kr = a.rope(q, kn, m, (cos, sin))
    out_a = a.append_attend(1, kr, vn, qr, 0.125, m)
    out_b = b.append_attend(1, kn, vn, q, 0.125, m, rope=(cos, sin))
    torch.cuda.synchronize()
    a.check_status()
    b.check_status()
    assert not calls, "a decode step must rotate inside its single launch"
    assert b.last_kernel == "decode"
    assert torch.equal(out_a, out_b)
    assert torch.equal(a._pool, b._pool)
    assert torch.equal(q, q0) and torch.equal(kn, k0), "the inputs are not modified"
    # the pool holds the rotated K (against the torch formula)
    slots = m.slot_mapping.long()
    got = b.k_pool[1].reshape(-1, 8, 64)[slots]
    assert torch.equal(got, torch_rope(kn, m.positions, cos, sin))
    if dtype == torch.float16:
        want = oracle_rope(kn.cpu().numpy(), m.positions.cpu().numpy(), cos.cpu().numpy(), sin.cpu().numpy())
        assert np.array_equal(got.cpu().numpy(), want)


@pytest.mark.parametrize("qlens", [[37, 1, 200, 1, 5], [512], [1, 64, 1]])
def test_prefill_and_mixed_rope_equal_rope_then_append_attend(qlens):
    rs = np.random.RandomState(2)
    ctx = [int(ql) + int(rs.randint(0, 700)) for ql in qlens]
    bks, m, kn, vn, q = setup(9, ctx, qlens)
    cos, sin = tables()
    a, b = bks
    calls = counting_rope(b)
    qr, kr = a.rope(q, kn, m, (cos, sin))
    out_a = a.append_attend(1, kr, vn, qr, 0.125, m)
    out_b = b.append_attend(1, kn, vn, q, 0.125, m, rope=(cos, sin))
    torch.cuda.synchronize()
    a.check_status()
    b.check_status()
    assert len(calls) == 1, "a non-decode step rotates with one pkv_rope launch, then the plain call"
    assert torch.equal(out_a, out_b)
    assert torch.equal(a._pool, b._pool)


def test_position_outside_the_tables_is_reported():
    bks, m, kn, vn, q = setup(4, [40, 90], [1, 1])
    cos, sin = tables(max_pos=64)  # the second sequence's position 89 is outside
    bk = bks[0]
    bk.append_attend(1, kn, vn, q, 0.125, m, rope=(cos, sin))
    torch.cuda.synchronize()
    with pytest.raises(PkvError):
        bk.check_status()
    bk.rope(q, kn, m, (cos, sin))
    torch.cuda.synchronize()
    with pytest.raises(PkvError):
        bk.check_status()


def test_bad_tables_are_rejected_before_any_launch():
    bks, m, kn, vn, q = setup(4, [40, 90], [1, 1])
    cos, sin = tables()
    bk = bks[0]
    for bad in [(cos.double(), sin), (cos, sin[:, :16].contiguous()), (cos.cpu(), sin), (cos[:, ::2], sin),
                (cos, sin[:100]), cos]:
        with pytest.raises(ValueError):
            bk.append_attend(1, kn, vn, q, 0.125, m, rope=bad)
    with pytest.raises(ValueError):
        bk.rope(q[:1], kn, m, (cos, sin))
    torch.cuda.synchronize()
    bk.check_status()


def test_llama_with_fused_rope_gives_the_same_logits_as_torch_rope():
    """RandomLlama passes unrotated q / k with rope= to the backend; the logits
    of a chunked-prefill step and of decode steps equal, bit for bit, those of
    the same model rotating with torch and calling append_attend without it."""
    cfg = LlamaConfig(n_layers=2, ffn=1024, vocab=4096)
    model = RandomLlama(cfg, DEV, seed=3)
    rs = np.random.RandomState(8)
    NB = 512
    bks = [B200PagedBackend(cfg.n_layers, NB, 16, cfg.n_kv_heads, cfg.n_heads, cfg.head_dim, device=DEV)
           for _ in range(2)]
    alloc = FifoAllocator(NB, 16, order=rs.permutation(NB))
    plens = [300, 17, 129, 64]
    seqs = [Seq(alloc, i) for i in range(len(plens))]
    toks = [torch.from_numpy(rs.randint(0, cfg.vocab, size=L)) for L in plens]
    steps = [(list(range(len(plens))), plens)] + [(list(range(len(plens))), [1] * len(plens))] * 4
    for n, (batch, qlens) in enumerate(steps):
        for i, ql in zip(batch, qlens):
            seqs[i].append(ql)
        m = meta_for([seqs[i] for i in batch], qlens, device=DEV)
        tokens = torch.cat(toks if n == 0 else [torch.from_numpy(rs.randint(0, cfg.vocab, size=1))
                                                  for _ in batch]).to(DEV)
        logits = []
        for fused, bk in zip((True, False), bks):
            model.fused_rope = fused
            logits.append(model.forward_varlen(tokens, m, bk))
        torch.cuda.synchronize()
        for bk in bks:
            bk.check_status()
        assert torch.equal(logits[0], logits[1]), f"step {n}"
        assert bks[0].last_kernel == ("prefill" if n == 0 else "decode")
    assert torch.equal(bks[0]._pool, bks[1]._pool)


def test_rope_on_a_geometry_without_the_fused_launch():
    """head_dim 128 (the generic attention kernel; the decode kernel takes 64):
    the rotation kernel handles any even head_dim, and a decode step with
    rope= falls back to rotating first and the plain call, with the same
    result as doing that by hand."""
    D, Hkv, Hq = 128, 2, 8
    cos, sin = tables(max_pos=512, D=D)
    rs = np.random.RandomState(6)
    bks = []
    for _ in range(2):
        bk = B200PagedBackend(1, 64, 16, Hkv, Hq, D, device=DEV, dtype=torch.float16)
        bk._pool.fill_(3.0)
        bks.append(bk)
    alloc = FifoAllocator(64, 16, order=rs.permutation(64))
    seqs = []
    for i, c in enumerate([40, 7, 100]):
        s = Seq(alloc, i)
        s.append(c - 1)
        seqs.append(s)
    hist = np.concatenate([[s.slot_for(p) for p in range(s.num_tokens)] for s in seqs]).astype(np.int64)
    g = torch.Generator(device=DEV).manual_seed(6)
    k = (torch.randn(hist.size, Hkv, D, generator=g, device=DEV) * 0.7).half()
    v = (torch.randn(hist.size, Hkv, D, generator=g, device=DEV) * 0.7).half()
    for bk in bks:
        bk.append_kv(0, k, v, slots_meta(hist))
    for s in seqs:
        s.append(1)
    m = meta_for(seqs, [1, 1, 1], device=DEV)
    kn = (torch.randn(3, Hkv, D, generator=g, device=DEV) * 0.7).half()
    vn = (torch.randn(3, Hkv, D, generator=g, device=DEV) * 0.7).half()
    q = torch.randn(3, Hq, D, generator=g, device=DEV).half()
    a, b = bks
    qr, kr = a.rope(q, kn, m, (cos, sin))
    want = oracle_rope(q.cpu().numpy(), m.positions.cpu().numpy(), cos.cpu().numpy(), sin.cpu().numpy())
    assert np.array_equal(qr.cpu().numpy(), want)
    out_a = a.append_attend(0, kr, vn, qr, 0.125, m)
    out_b = b.append_attend(0, kn, vn, q, 0.125, m, rope=(cos, sin))
    torch.cuda.synchronize()
    a.check_status()
    b.check_status()
    assert torch.equal(out_a, out_b)
    assert torch.equal(a._pool, b._pool)
