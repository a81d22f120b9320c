"""
Seeded input cases shared by the golden-fixture generator and the tests.

Inputs are regenerated from ``numpy.random.RandomState`` (whose stream is
frozen across numpy versions); each fixture stores a checksum of the inputs it
was made from so a drift in regeneration is caught rather than silently
compared against the wrong outputs.

Geometry names follow the reference: ``num_layers`` (L), ``num_blocks`` (NB),
``block_size`` (P, tokens per page), ``n_kv_heads`` (Hkv), ``n_heads`` (Hq),
``head_dim`` (D).
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass, field

import numpy as np

LLAMA = dict(n_kv_heads=8, n_heads=32, head_dim=64, block_size=16)


@dataclass
class AttnCase:
    """One attention step over a seeded, scattered pool.

    ``hist[i]`` tokens of history are written first (one prefill-shaped append),
    then a step appends ``qlens[i]`` more tokens and attends with ``qlens[i]``
    queries per sequence (``kv_len = hist + qlen``).
    """

    name: str
    seed: int
    num_blocks: int
    block_size: int
    n_kv_heads: int
    n_heads: int
    head_dim: int
    hist: list[int]
    qlens: list[int]
    dtype: str = "float16"
    kv_std: float = 1.0
    q_std: float = 1.0
    poison: float | None = None
    scale: float | None = None
    # filled by materialise()
    tables: list[list[int]] = field(default_factory=list)
    kv_lens: list[int] = field(default_factory=list)
    k_hist: np.ndarray | None = None
    v_hist: np.ndarray | None = None
    k_new: np.ndarray | None = None
    v_new: np.ndarray | None = None
    q: np.ndarray | None = None

    @property
    def np_dtype(self):
        return np.dtype(self.dtype)

    def materialise(self) -> "AttnCase":
        rs = np.random.RandomState(self.seed)
        free = list(rs.permutation(self.num_blocks))  # seeded scatter of the free list
        P = self.block_size
        self.kv_lens = [h + q for h, q in zip(self.hist, self.qlens)]
        self.tables = []
        for n in self.kv_lens:
            need = (n + P - 1) // P
            self.tables.append([int(b) for b in free[:need]])
            del free[:need]
        H, D, Hq = self.n_kv_heads, self.head_dim, self.n_heads
        dt = self.np_dtype
        th, tq = sum(self.hist), sum(self.qlens)
        self.k_hist = (rs.standard_normal((th, H, D)) * self.kv_std).astype(dt)
        self.v_hist = (rs.standard_normal((th, H, D)) * self.kv_std).astype(dt)
        self.k_new = (rs.standard_normal((tq, H, D)) * self.kv_std).astype(dt)
        self.v_new = (rs.standard_normal((tq, H, D)) * self.kv_std).astype(dt)
        self.q = (rs.standard_normal((tq, Hq, D)) * self.q_std).astype(dt)
        if self.scale is None:
            self.scale = 1.0 / float(np.sqrt(D))
        return self

    def slots(self, which: str) -> np.ndarray:
        """Flat slots of the history tokens (``which='hist'``) or the step's new tokens."""
        P = self.block_size
        out = []
        for t, h, q in zip(self.tables, self.hist, self.qlens):
            rng = range(0, h) if which == "hist" else range(h, h + q)
            out.extend(t[p // P] * P + p % P for p in rng)
        return np.asarray(out, dtype=np.int64)

    def checksum(self) -> str:
        h = hashlib.sha256()
        for a in (self.k_hist, self.v_hist, self.k_new, self.v_new, self.q):
            h.update(np.ascontiguousarray(a).tobytes())
        h.update(repr((self.tables, self.kv_lens, self.scale)).encode())
        return h.hexdigest()


def attn_cases() -> list[AttnCase]:
    rs = np.random.RandomState(1)
    cfg1_ctx = [int(x) for x in rs.randint(1, 513, size=8)]
    return [
        # config 1: one layer of Llama-3.2-1B geometry, 8 sequences, ctx ~ U[1,512],
        # 512-block pool scattered by a seeded permutation, Q/K/V ~ N(0,1), fp32,
        # scale 1/8; decode step (the last token of each context is this step's).
        AttnCase("cfg1_decode_f32", 101, 512, dtype="float32",
                 hist=[c - 1 for c in cfg1_ctx], qlens=[1] * 8, scale=0.125, **LLAMA),
        # fp16 decode at Llama geometry across every page-boundary case, pool
        # poisoned with 1e3 so reading the unwritten tail of a last page shows.
        AttnCase("straddle_decode_f16", 102, 256, dtype="float16", kv_std=0.5 ** 0.5,
                 hist=[0, 14, 15, 16, 30, 31, 32, 99, 256, 511],
                 qlens=[1] * 10, poison=1e3, **LLAMA),
        # fp16 chunked prefill mixed with decodes at Llama geometry.
        AttnCase("mixed_prefill_f16", 103, 256, dtype="float16", kv_std=0.5 ** 0.5,
                 hist=[6, 18, 16, 0, 64, 100], qlens=[4, 1, 1, 37, 16, 77],
                 poison=1e3, **LLAMA),
        # the reference tests' small geometry, fp32: 2 KV heads, 4 query heads, D=8.
        AttnCase("small_mixed_f32", 104, 32, 16, 2, 4, 8,
                 hist=[6, 18, 16, 0], qlens=[4, 1, 1, 33], dtype="float32"),
        # GQA 6/2 with block_size 4 (reference copy/swap geometry), fp32.
        AttnCase("small_bs4_f32", 105, 64, 4, 2, 6, 8,
                 hist=[0, 3, 4, 9], qlens=[5, 1, 1, 2], dtype="float32"),
    ]


def copy_block_pool(num_layers=4, num_blocks=8, block_size=4, n_kv=2, head_dim=8):
    """Pattern of the reference's copy_block tests: block b of layer l holds
    ``b + l*100`` in K and ``b + l*100 + 50`` in V (``tests/test_copy_block.py:39-47``)."""
    k = np.zeros((num_layers, num_blocks, block_size, n_kv, head_dim), np.float32)
    v = np.zeros_like(k)
    for l in range(num_layers):
        for b in range(num_blocks):
            k[l, b] = b + l * 100
            v[l, b] = b + l * 100 + 50
    return k, v


COPY_OPS = [(1, 2), (0, 5), (3, 3), (7, 0)]

# swap: 2 layers, block_size 4, 2 KV heads, head_dim 8, float64, 16-block pool
SWAP_GEOM = dict(num_layers=2, num_blocks=16, block_size=4, n_kv_heads=2, head_dim=8)
SWAP_TOKENS = 10
