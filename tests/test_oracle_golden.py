"""
Pin the CPU oracle before trusting it.

Every oracle function is checked against golden vectors produced by running the
reference's own code (``tests/golden/make_golden.py``): attention outputs of
``PagedTorchBackend.attend``, pools after ``append_kv``/``copy_block``, host
buffers and pools after a ``KVSwapSpace`` round trip, and every integer field of
``build_batch_meta``. Plus the known-answer scenarios of the reference's own
tests, restated. When the reference checkout is present in this container, the
oracle is also diffed against the live reference on fresh seeded inputs.
"""

from __future__ import annotations

import os
import sys
import types
from pathlib import Path

import numpy as np
import pytest

from cases import COPY_OPS, SWAP_GEOM, SWAP_TOKENS, attn_cases, copy_block_pool
from llm_serving_layer_b200.meta import build_meta
from oracle import OraclePool, attend_exact, attend_reference, build_csr, last_page_len, rope, slot_for

GOLD = Path(__file__).resolve().parent / "golden"


def ulp_tol(ref: np.ndarray) -> np.ndarray:
    """One unit in the last place of ``ref``'s dtype at each element, plus a
    floor for results that cancel to near zero (the summands are O(1), so
    their rounding is not scaled by the result's magnitude), as float64."""
    floor = 5e-4 if ref.dtype == np.float16 else 1e-6
    return np.spacing(np.abs(ref)).astype(np.float64) + floor


def run_oracle_case(c):
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
def test_oracle_attention_matches_reference_golden(case):
    c = case.materialise()
    f = np.load(GOLD / f"{c.name}.npz")
    assert str(f["checksum"]) == c.checksum(), "regenerated inputs drifted from the fixture's"
    pool, m = run_oracle_case(c)
    got = pool.attend(c.q, 0, c.scale, m).astype(np.float64)
    want = f["out"].astype(np.float64)
    # same steps, same precisions; only the summation order of the matmuls
    # differs, so the results agree to one unit in the last place of the dtype
    assert np.all(np.abs(got - want) <= ulp_tol(f["out"]))
    # the float64 evaluation sits within the fp16 rounding budget of the reference
    exact = pool.attend(c.q, 0, c.scale, m, exact=True)
    assert np.abs(exact - want).max() <= (1e-6 if c.dtype == "float32" else 2e-3)
    if f["k_pool"].size:
        assert np.array_equal(pool.k[0], f["k_pool"]) and np.array_equal(pool.v[0], f["v_pool"])


def test_oracle_copy_block_matches_reference_golden():
    k, v = copy_block_pool()
    L, NB, P, H, D = k.shape
    pool = OraclePool(L, NB, P, H, D, dtype=np.float32)
    for l in range(L):
        pool.k[l][:] = k[l]
        pool.v[l][:] = v[l]
    for s, d in COPY_OPS:
        pool.copy_block(s, d)
    f = np.load(GOLD / "copy_block.npz")
    assert np.array_equal(np.stack(pool.k), f["k"]) and np.array_equal(np.stack(pool.v), f["v"])
    for s, d in [(-1, 0), (0, -1), (NB, 0), (0, NB)]:
        with pytest.raises(IndexError):
            pool.copy_block(s, d)
    assert f["raised"].sum() == 4


def test_oracle_swap_matches_reference_golden():
    f = np.load(GOLD / "swap_roundtrip.npz")
    g = SWAP_GEOM
    pool = OraclePool(g["num_layers"], g["num_blocks"], g["block_size"], g["n_kv_heads"],
                      g["head_dim"], dtype=np.float64)
    src = [int(b) for b in f["src_ids"]]
    P, H, D = g["block_size"], g["n_kv_heads"], g["head_dim"]
    for l in range(g["num_layers"]):
        for i, b in enumerate(src):
            pool.k[l][b] = 7.0 + l * 100 + i + np.arange(P * H * D, dtype=np.float64).reshape(P, H, D) / 1000
            pool.v[l][b] = -(7.0 + l * 100 + i)
    kh, vh = pool.swap_out(src)
    assert np.array_equal(kh, f["k_host"]) and np.array_equal(vh, f["v_host"])
    assert kh.nbytes + vh.nbytes == int(f["nbytes"])
    for l in range(g["num_layers"]):
        for b in f["decoy_ids"]:
            pool.k[l][b] = -99.0
            pool.v[l][b] = -99.0
    pool.swap_in(kh, vh, [int(b) for b in f["dst_ids"]])
    assert np.array_equal(np.stack(pool.k), f["k_pool"]) and np.array_equal(np.stack(pool.v), f["v_pool"])
    assert len(src) == (SWAP_TOKENS + P - 1) // P
    with pytest.raises(RuntimeError, match="resume mismatch"):
        pool.swap_in(kh, vh, [0])


def test_batch_assembly_matches_reference_golden():
    f = np.load(GOLD / "batch_assembly.npz")
    flat, lens = f["tables_flat"], f["tables_len"]
    tables = np.split(flat, np.cumsum(lens)[:-1])
    kv = f["hist"] + f["qlens"]
    m = build_meta([t.tolist() for t in tables], kv, f["qlens"], 16)
    for name in ("query_lens", "cu_query_lens", "kv_lens", "positions", "last_token_ix",
                 "kv_indptr", "kv_indices", "kv_last_page_len", "batch_indices", "slot_mapping"):
        assert np.array_equal(getattr(m, name).numpy(), f[name]), name
    assert m.is_prefill == bool(f["is_prefill"])
    m.validate()
    # the oracle's restatement of the block-table arithmetic agrees too
    ip, idx, lp = build_csr([t.tolist() for t in tables], kv.tolist(), 16)
    assert ip == f["kv_indptr"].tolist() and idx == f["kv_indices"].tolist()
    assert lp == f["kv_last_page_len"].tolist()
    slots = []
    for t, h, q in zip(tables, f["hist"], f["qlens"]):
        slots += [slot_for(t.tolist(), p, 16) for p in range(h, h + q)]
    assert slots == f["slot_mapping"].tolist()


@pytest.mark.parametrize("n", [1, 15, 16, 17, 31, 32, 33])
def test_last_page_len_reports_block_size_not_zero(n):
    assert last_page_len(n, 16) == (n % 16 or 16)


# --- known-answer scenarios of the reference's tests, restated -------------


def _meta_for(tables, kv, ql, P=16):
    return build_meta(tables, kv, ql, P)


def test_oracle_gqa_value_mapping_is_floor_divide():
    """tests/test_paged_torch.py:420-452: kv_len 1, distinct constant per KV head."""
    H, Hq, D = 2, 6, 8
    pool = OraclePool(1, 8, 16, H, D, dtype=np.float32)
    v = np.zeros((1, H, D), np.float32)
    for j in range(H):
        v[0, j] = j + 1
    pool.append_kv(0, np.zeros_like(v), v, [0])
    q = np.random.RandomState(0).standard_normal((1, Hq, D)).astype(np.float32)
    out = pool.attend(q, 0, 1.0, _meta_for([[0]], [1], [1]))
    for h in range(Hq):
        assert np.allclose(out[0, h], h // 3 + 1)


def test_oracle_causality_poison():
    """tests/test_paged_torch.py:595-628: a later key never changes earlier queries."""
    rs = np.random.RandomState(21)
    H, Hq, D, n = 2, 4, 8, 6
    pool = OraclePool(1, 8, 16, H, D, dtype=np.float32)
    pool.append_kv(0, rs.standard_normal((n, H, D)), rs.standard_normal((n, H, D)), np.arange(n))
    m = _meta_for([[0]], [n], [n])
    q = rs.standard_normal((n, Hq, D)).astype(np.float32)
    base = pool.attend(q, 0, 0.35, m)
    pool.k[0][0, n - 1] = 100.0
    pool.v[0][0, n - 1] = -999.0
    pois = pool.attend(q, 0, 0.35, m)
    assert np.array_equal(base[: n - 1], pois[: n - 1])
    assert not np.allclose(base[n - 1], pois[n - 1])


def test_oracle_detects_a_wrong_gqa_mapping():
    """A mistake planted in the oracle's inputs (h % Hkv instead of h // groups)
    is visible to the comparison the GPU tests make."""
    c = attn_cases()[3].materialise()
    pool, m = run_oracle_case(c)
    good = attend_exact(c.q, pool.k[0], pool.v[0], c.scale, m)
    # with 4 query heads over 2 KV heads, swapping query heads 1 and 2 before
    # attention (and the outputs after) gives exactly the `h % Hkv` mapping
    assert (c.n_heads, c.n_kv_heads) == (4, 2)
    qb = c.q.copy()
    qb[:, [1, 2]] = qb[:, [2, 1]]
    bad = attend_exact(qb, pool.k[0], pool.v[0], c.scale, m)
    bad[:, [1, 2]] = bad[:, [2, 1]]
    assert np.abs(bad - good).max() > 1e-2


REF = os.environ.get("LLM_SERVING_LAYER_REF", "")


@pytest.mark.skipif(not REF or not Path(REF, "serving", "backends", "paged_torch.py").is_file(),
                    reason="set LLM_SERVING_LAYER_REF to a reference checkout to compare against it live "
                           "(the committed fixtures pin the oracle without it)")
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_oracle_matches_live_reference(seed):
    """Fresh seeded ragged batches: oracle vs the reference's PagedTorchBackend."""
    import torch

    import llm_serving_layer_b200.meta as meta_mod
    eng = types.ModuleType("engine")
    eng.attention_backend = meta_mod
    sys.modules.setdefault("engine", eng)
    sys.modules.setdefault("engine.attention_backend", meta_mod)
    if REF not in sys.path:
        sys.path.append(REF)
    from serving.backends.paged_torch import PagedTorchBackend

    rs = np.random.RandomState(1000 + seed)
    H, Hq, D, P, NB = 8, 32, 64, 16, 128
    n = 5
    hist = rs.randint(0, 120, size=n)
    ql = rs.randint(1, 20, size=n)
    kv = hist + ql
    free = list(rs.permutation(NB))
    tables = []
    for x in kv:
        need = (int(x) + P - 1) // P
        tables.append([int(b) for b in free[:need]])
        del free[:need]
    m = build_meta(tables, kv, ql, P)
    T = int(ql.sum())
    k = rs.standard_normal((T, H, D)).astype(np.float16)
    v = rs.standard_normal((T, H, D)).astype(np.float16)
    q = rs.standard_normal((T, Hq, D)).astype(np.float16)
    bk = PagedTorchBackend(1, NB, P, H, Hq, D, device="cpu", dtype=torch.float16)
    pool = OraclePool(1, NB, P, H, D, dtype=np.float16)
    hist_rows = rs.standard_normal((NB, P, H, D)).astype(np.float16)
    bk.k_pool[0].copy_(torch.from_numpy(hist_rows))
    bk.v_pool[0].copy_(torch.from_numpy(-hist_rows))
    pool.k[0][:] = hist_rows
    pool.v[0][:] = -hist_rows
    bk.append_kv(0, torch.from_numpy(k), torch.from_numpy(v), m)
    pool.append_kv(0, k, v, m.slot_mapping.numpy())
    assert np.array_equal(bk.k_pool[0].numpy(), pool.k[0])
    want = bk.attend(torch.from_numpy(q), 0, 0.125, m).numpy().astype(np.float64)
    got = attend_reference(q, pool.k[0], pool.v[0], 0.125, m).astype(np.float64)
    assert np.all(np.abs(got - want) <= ulp_tol(want.astype(np.float16)))


def test_oracle_rope_matches_reference_golden():
    """``oracle.rope`` against the reference's own rotary embedding (``_rope``
    of its paged-model tests, tests/test_preemption.py:85-102: float64, theta
    10000), run by make_golden.py. The tables are recomputed here from the same
    expression; numpy's and torch's pow / cos may differ in the last bit, which
    an angle of a few thousand radians turns into ~1e-12, so the pin is 1e-9:
    a wrong pairing, sign or position gives O(1) differences."""
    g = np.load(GOLD / "rope.npz")
    x, pos, out = g["x"], g["positions"], g["out"]
    half = x.shape[-1] // 2
    inv = float(g["theta"]) ** (-np.arange(half, dtype=np.float64) / half)
    ang = np.arange(int(pos.max()) + 1, dtype=np.float64)[:, None] * inv[None, :]
    got = rope(x, pos, np.cos(ang), np.sin(ang))
    assert got.dtype == np.float64
    np.testing.assert_allclose(got, out, rtol=0, atol=1e-9)
    # a planted mistake is caught: rotating by position + 1
    bad = rope(x, pos + 1, np.cos(np.vstack([ang, ang[-1:] + inv])), np.sin(np.vstack([ang, ang[-1:] + inv])))
    assert np.abs(bad - out).max() > 1e-2


def test_oracle_rope_float32_is_the_torch_formula_bit_for_bit():
    """In float32 with fp16 data the oracle gives the bits of the formula as the
    random-init Llama evaluates it with torch (each product rounded, then the
    difference / sum, then fp16): the reference point of the CUDA kernels'
    bit-exact RoPE tests."""
    import torch

    rs = np.random.RandomState(3)
    x = (rs.standard_normal((50, 4, 64)) * 2).astype(np.float16)
    pos = rs.randint(0, 2048, 50)
    inv = 1.0 / (500000.0 ** (torch.arange(0, 64, 2, dtype=torch.float32) / 64))
    ang = torch.arange(2048, dtype=torch.float32)[:, None] * inv[None, :]
    cos, sin = torch.cos(ang), torch.sin(ang)
    xt = torch.from_numpy(x)
    c, s_ = cos[torch.from_numpy(pos)][:, None, :], sin[torch.from_numpy(pos)][:, None, :]
    a, b = xt[..., :32].float(), xt[..., 32:].float()
    want = torch.cat([a * c - b * s_, a * s_ + b * c], dim=-1).to(torch.float16).numpy()
    got = rope(x, pos, cos.numpy(), sin.numpy())
    assert got.dtype == np.float16
    assert np.array_equal(got.view(np.uint16), want.view(np.uint16))
