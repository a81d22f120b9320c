"""
Step descriptor for one forward pass over a ragged batch: ``BatchMeta``.

The serving layer's engine (an un-vendored submodule of the reference) owns the
authoritative ``BatchMeta``; this module provides a field-for-field compatible
dataclass so the backend can be driven without that engine. The field list,
dtypes and ``validate()`` messages follow the contract written in the
reference's ``docs/ARCHITECTURE.md:88-120`` and the rejection tests in
``tests/test_batch_assembly.py:345-384`` (``AssertionError`` whose text names
the broken field: ``kv_last_page_len``, ``pages allocated``, ``batch_indices``).

The backend itself only duck-types ``meta``: any object exposing these
attributes (the engine's own class included) is accepted.

Also here: ``build_meta``, a vectorised host-side assembler from per-sequence
block tables (numpy, one H2D copy per field), restating the slot arithmetic of
``serving/memory/block_table.py:100-109`` (``slot = block_ids[p // P] * P +
p % P``) and the CSR flattening of ``block_table.py:184-208`` /
``serving/engine_iface/batch.py:190-318``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Protocol, Sequence

import numpy as np
import torch

__all__ = ["BatchMeta", "AttentionBackend", "build_meta"]


@dataclass(frozen=True)
class BatchMeta:
    """One forward pass: sequences' new tokens packed along axis 0, in order.

    query_lens      (n,)   int32  new tokens this step, per sequence
    cu_query_lens   (n+1,) int32  exclusive prefix sum of query_lens
    kv_lens         (n,)   int32  KV length AFTER this step's append
    positions       (T,)   int64  absolute RoPE position of each token
    last_token_ix   (n,)   int32  index of each sequence's last token
    kv_indptr       (n+1,) int32  CSR offsets into kv_indices
    kv_indices      (P,)   int32  physical page ids, in logical order
    kv_last_page_len (n,)  int32  occupancy of the last page, in [1, page_size]
    batch_indices   (T,)   int32  owning sequence of each token
    slot_mapping    (T,)   int32  flat physical slot of each new token, or None

    Optional host-side facts, known to an assembler without reading the device
    tensors back (``None`` / 0 when not supplied): ``max_query_len`` and
    ``min_query_len``, and ``checked_blocks`` — when nonzero, the assembler has
    already made the page-table checks a backend would otherwise make by reading
    the fields back (query and kv lengths, page counts) and every block id in
    the page table lies in ``[0, checked_blocks)``.
    """

    query_lens: torch.Tensor
    cu_query_lens: torch.Tensor
    kv_lens: torch.Tensor
    positions: torch.Tensor
    last_token_ix: torch.Tensor
    kv_indptr: torch.Tensor
    kv_indices: torch.Tensor
    kv_last_page_len: torch.Tensor
    batch_indices: torch.Tensor
    slot_mapping: torch.Tensor | None = None
    page_size: int = 16
    is_prefill: bool = False
    max_query_len: int | None = None
    min_query_len: int | None = None
    checked_blocks: int = 0

    @property
    def n_seqs(self) -> int:
        return int(self.query_lens.shape[0])

    @property
    def n_tokens(self) -> int:
        return int(self.positions.shape[0])

    def validate(self) -> None:
        """Check the invariants whose violation is silent downstream.

        Raises ``AssertionError`` naming the offending field, as the engine's
        own ``validate()`` does.
        """
        ql = self.query_lens.tolist()
        cu = self.cu_query_lens.tolist()
        kl = self.kv_lens.tolist()
        ip = self.kv_indptr.tolist()
        lp = self.kv_last_page_len.tolist()
        P = self.page_size
        n = len(ql)
        t = sum(ql)
        assert len(cu) == n + 1 and cu[0] == 0, "cu_query_lens must have n_seqs+1 entries starting at 0"
        assert len(ip) == n + 1 and ip[0] == 0, "kv_indptr must have n_seqs+1 entries starting at 0"
        assert len(kl) == n and len(lp) == n, "kv_lens / kv_last_page_len must have n_seqs entries"
        for i in range(n):
            assert cu[i + 1] - cu[i] == ql[i], f"cu_query_lens disagrees with query_lens at seq {i}"
            assert 1 <= lp[i] <= P, f"kv_last_page_len[{i}]={lp[i]} outside [1, {P}]"
            pages = ip[i + 1] - ip[i]
            assert pages == (kl[i] + P - 1) // P, (
                f"seq {i}: {pages} pages allocated for kv_len {kl[i]} (page_size {P})"
            )
            assert (pages - 1) * P + lp[i] == kl[i], (
                f"seq {i}: kv_last_page_len {lp[i]} disagrees with kv_lens {kl[i]}"
            )
            assert ql[i] <= kl[i], f"seq {i}: query_len {ql[i]} exceeds kv_len {kl[i]}"
        assert int(self.kv_indices.shape[0]) == ip[-1], "kv_indices length != kv_indptr[-1]"
        assert int(self.batch_indices.shape[0]) == t, "batch_indices length != tokens"
        assert int(self.positions.shape[0]) == t, "positions length != tokens"
        assert int(self.last_token_ix.shape[0]) == n, "last_token_ix length != n_seqs"
        if self.slot_mapping is not None:
            assert int(self.slot_mapping.shape[0]) == t, "slot_mapping length != tokens"


class AttentionBackend(Protocol):
    """The engine-facing protocol (reference ``docs/ARCHITECTURE.md:155-160``)."""

    def append_kv(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor, meta: BatchMeta) -> None: ...

    def attend(self, q: torch.Tensor, layer_idx: int, scale: float, meta: BatchMeta) -> torch.Tensor: ...


def build_meta(
    block_tables: Sequence[Sequence[int]] | None,
    kv_lens: Sequence[int],
    query_lens: Sequence[int],
    page_size: int,
    device: str | torch.device = "cpu",
    *,
    kv_indptr: np.ndarray | None = None,
    kv_indices: np.ndarray | None = None,
    pin: bool = False,
) -> BatchMeta:
    """Assemble a ``BatchMeta`` from block tables, vectorised in numpy.

    ``block_tables[i]`` lists sequence ``i``'s physical pages in logical order
    and must already cover ``kv_lens[i]`` (the length AFTER this step's append,
    the ordering contract of ``serving/engine_iface/batch.py:40-46``).
    Alternatively pass the CSR pair ``kv_indptr``/``kv_indices`` directly.
    Raises ``ValueError`` on an empty batch, a non-positive query length, a
    query longer than its history, or a table too short for its ``kv_len``.
    """
    kv = np.asarray(kv_lens, dtype=np.int64)
    ql = np.asarray(query_lens, dtype=np.int64)
    n = int(kv.shape[0])
    if n == 0:
        raise ValueError("build_meta() called with an empty sequence list")
    if page_size <= 0:
        raise ValueError(f"page_size must be positive, got {page_size}")
    if ql.shape[0] != n:
        raise ValueError(f"{ql.shape[0]} query lengths for {n} sequences")
    if (ql <= 0).any():
        i = int(np.nonzero(ql <= 0)[0][0])
        raise ValueError(f"seq {i} contributes {int(ql[i])} tokens; every sequence must contribute >= 1")
    if (ql > kv).any():
        i = int(np.nonzero(ql > kv)[0][0])
        raise ValueError(
            f"seq {i} contributes {int(ql[i])} tokens but holds only {int(kv[i])}; "
            "grow the block table (blocks.append) before assembly"
        )
    pages = (kv + page_size - 1) // page_size
    if kv_indptr is None:
        assert block_tables is not None
        if len(block_tables) != n:
            raise ValueError(f"{len(block_tables)} block tables for {n} sequences")
        have = np.fromiter((len(b) for b in block_tables), dtype=np.int64, count=n)
        if (have < pages).any():
            i = int(np.nonzero(have < pages)[0][0])
            raise ValueError(f"seq {i}: {int(have[i])} blocks hold fewer than kv_len={int(kv[i])} tokens")
        indptr = np.zeros(n + 1, dtype=np.int64)
        np.cumsum(pages, out=indptr[1:])
        indices = np.concatenate(
            [np.asarray(b[: int(p)], dtype=np.int64) for b, p in zip(block_tables, pages)]
        ) if int(indptr[-1]) else np.zeros(0, dtype=np.int64)
    else:
        indptr = np.asarray(kv_indptr, dtype=np.int64)
        indices = np.asarray(kv_indices, dtype=np.int64)
        if not np.array_equal(np.diff(indptr), pages):
            raise ValueError("kv_indptr page counts disagree with kv_lens")

    cu = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(ql, out=cu[1:])
    T = int(cu[-1])
    batch_idx = np.repeat(np.arange(n, dtype=np.int64), ql)
    # absolute positions kv_len - q_len .. kv_len - 1 of each sequence
    start = kv - ql
    positions = np.arange(T, dtype=np.int64) - np.repeat(cu[:-1], ql) + np.repeat(start, ql)
    # slot = page_id(position // P) * P + position % P
    page_of_tok = indices[np.repeat(indptr[:-1], ql) + positions // page_size]
    slots = page_of_tok * page_size + positions % page_size
    rem = kv % page_size
    last_page = np.where(rem == 0, page_size, rem)

    def put(a: np.ndarray, dt: torch.dtype) -> torch.Tensor:
        t = torch.from_numpy(np.ascontiguousarray(a)).to(dt)
        if torch.device(device).type == "cuda":
            if pin:
                t = t.pin_memory()
            return t.to(device, non_blocking=pin)
        return t

    i32 = torch.int32
    return BatchMeta(
        query_lens=put(ql, i32),
        cu_query_lens=put(cu, i32),
        kv_lens=put(kv, i32),
        positions=put(positions, torch.int64),
        last_token_ix=put(cu[1:] - 1, i32),
        kv_indptr=put(indptr, i32),
        kv_indices=put(indices, i32),
        kv_last_page_len=put(last_page, i32),
        batch_indices=put(batch_idx, i32),
        slot_mapping=put(slots, i32),
        page_size=int(page_size),
        is_prefill=bool((ql > 1).any()),
        max_query_len=int(ql.max()),
        min_query_len=int(ql.min()),
    )
