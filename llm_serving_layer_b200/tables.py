"""
DeviceBlockTables — per-sequence block tables kept on the device, and each
step's ``BatchMeta`` assembled there.

The reference rebuilds the step descriptor on the host every step
(``build_batch_meta``, ``serving/engine_iface/batch.py:190-318``): Python loops
over every sequence and token (``SequenceBlocks.slots_for_new_tokens``,
``serving/memory/block_table.py:100-121``; ``build_csr``, ``block_table.py:184-208``)
followed by one host-to-device copy per field. Here each sequence owns a row of
a device table ``[max_seqs][max_pages]`` of physical block ids in logical
order; the host records only what changed (``bind`` a whole row, ``extend`` it
with newly allocated blocks, ``set_block`` after a copy-on-write), and
``build_batch_meta(rows, query_lens, kv_lens)`` sends the step's rows and
lengths plus those changes in ONE pinned copy, after which two kernels
(``pkv_build_batch_meta``, ``include/pkv.h``) write every field.

The host keeps the reference's checks and messages (``ValueError`` for an empty
batch, a sequence contributing no tokens, a query longer than its history, a
table too short for its ``kv_len``) and checks every block id against the pool
when it is recorded, so the returned meta carries ``checked_blocks`` and a
backend need not read the page table back.

Lifetime: the fields of a returned ``BatchMeta`` are views into one of
``ring`` output buffers, overwritten (in stream order) by the ``ring``-th
later ``build_batch_meta``; work that reads a meta must be issued before then.
"""

from __future__ import annotations

import ctypes
from typing import Sequence

import numpy as np
import torch

from . import _native as N
from .meta import BatchMeta

__all__ = ["DeviceBlockTables"]


class _Slot:
    """One output buffer of the ring, with its pinned / device input staging."""

    def __init__(self, device: torch.device, seqs_cap: int, tokens_cap: int, pages_cap: int, in_words: int):
        self.i32 = torch.empty(6 * seqs_cap + 2 + 2 * tokens_cap + pages_cap, dtype=torch.int32, device=device)
        self.pos = torch.empty(max(tokens_cap, 1), dtype=torch.int64, device=device)
        self.seqs_cap, self.tokens_cap, self.pages_cap = seqs_cap, tokens_cap, pages_cap
        o = 0
        self.off = {}
        for name, size in (("query_lens", seqs_cap), ("cu_query_lens", seqs_cap + 1), ("kv_lens", seqs_cap),
                           ("last_token_ix", seqs_cap), ("kv_indptr", seqs_cap + 1),
                           ("kv_last_page_len", seqs_cap), ("batch_indices", tokens_cap),
                           ("slot_mapping", tokens_cap), ("kv_indices", pages_cap)):
            self.off[name] = o
            o += size
        base, es = self.i32.data_ptr(), self.i32.element_size()
        self.desc = N.MetaOutDesc(
            *(base + self.off[f] * es for f in ("query_lens", "cu_query_lens", "kv_lens")),
            self.pos.data_ptr(),
            *(base + self.off[f] * es for f in ("last_token_ix", "kv_indptr", "kv_indices", "kv_last_page_len",
                                                "batch_indices", "slot_mapping")),
            seqs_cap, 0, tokens_cap, pages_cap)
        self.desc_ref = ctypes.byref(self.desc)
        self.event = torch.cuda.Event()
        self.used = False
        self.resize_input(device, in_words)

    def resize_input(self, device: torch.device, words: int) -> None:
        self.host = torch.empty(words, dtype=torch.int32).pin_memory()
        self.host_np = self.host.numpy()
        self.host_ptr = self.host.data_ptr()
        self.dev = torch.empty(words, dtype=torch.int32, device=device)


class DeviceBlockTables:
    """Block tables of up to ``max_seqs`` sequences (rows), ``max_pages`` pages
    each, mirrored on ``device``; ``build_batch_meta`` assembles a step's
    ``BatchMeta`` on the device.

    ``num_blocks`` is the pool size every recorded block id is checked against
    (``IndexError`` outside ``[0, num_blocks)``); ``max_tokens`` bounds the
    tokens of one step; ``status`` is the int32 device word the kernels flag
    violations into (pass the backend's, or leave None for an own one,
    read by ``check_status``)."""

    def __init__(self, max_seqs: int, max_pages: int, block_size: int, num_blocks: int,
                 device: str | torch.device = "cuda:0", *, max_tokens: int | None = None, ring: int = 3,
                 status: torch.Tensor | None = None):
        for name, val in (("max_seqs", max_seqs), ("max_pages", max_pages), ("block_size", block_size),
                          ("num_blocks", num_blocks), ("ring", ring)):
            if int(val) <= 0:
                raise ValueError(f"{name} must be positive, got {val}")
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError(f"DeviceBlockTables requires a CUDA device, got {self.device}; it has no CPU path")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self._dev_index = self.device.index
        self._lib = N.lib()
        self.max_seqs, self.max_pages, self.block_size = int(max_seqs), int(max_pages), int(block_size)
        self.num_blocks = int(num_blocks)
        self.max_tokens = int(max_tokens) if max_tokens is not None else max(self.max_seqs, 8192)
        self.table = torch.full((self.max_seqs, self.max_pages), -1, dtype=torch.int32, device=self.device)
        self._desc = N.BlockTablesDesc(self.table.data_ptr(), self.max_seqs, self.max_pages, self.block_size, 0)
        self._desc_ref = ctypes.byref(self._desc)
        self.status = status if status is not None else torch.zeros(1, dtype=torch.int32, device=self.device)
        self._status_ptr = self.status.data_ptr()
        self.pages = np.zeros(self.max_seqs, dtype=np.int64)  # entries recorded per row (host count)
        self._upd: list[tuple[np.ndarray, np.ndarray, np.ndarray]] = []
        self._n_upd = 0
        self._upd_rows: set[int] = set()  # rows edited since the last build
        self._upd_dup = False  # some row was edited twice: the last edit of a page must win
        pages_cap = self.max_seqs * self.max_pages
        in_words = 3 * self.max_seqs + 3 * max(self.max_seqs, 1024)
        self._ring = [_Slot(self.device, self.max_seqs, self.max_tokens, pages_cap, in_words)
                      for _ in range(int(ring))]
        self._next = 0
        self.n_builds = 0

    # -- table edits (recorded on the host, applied by the next build) ---------

    def bind(self, row: int, block_ids: Sequence[int] | np.ndarray) -> None:
        """Row ``row`` now holds ``block_ids`` (logical page order), replacing
        what it held (a new sequence, or one resumed into fresh blocks)."""
        ids = self._ids(row, block_ids)
        self._record(row, 0, ids)
        self.pages[row] = ids.shape[0]

    def extend(self, row: int, block_ids: Sequence[int] | np.ndarray) -> None:
        """Append newly allocated blocks to row ``row``'s table."""
        ids = self._ids(row, block_ids)
        start = int(self.pages[row])
        if start + ids.shape[0] > self.max_pages:
            raise ValueError(f"row {row}: {start + ids.shape[0]} pages exceed max_pages={self.max_pages}")
        self._record(row, start, ids)
        self.pages[row] = start + ids.shape[0]

    def set_block(self, row: int, page: int, block_id: int) -> None:
        """Replace page ``page`` of row ``row`` (the block a copy-on-write
        allocated, ``RadixCache.ensure_writable``, ``serving/cache/radix.py:629-677``)."""
        self._row(row)
        if not 0 <= page < int(self.pages[row]):
            raise IndexError(f"row {row} holds {int(self.pages[row])} pages; page {page} does not exist")
        self._record(row, int(page), self._ids(row, [block_id]))

    def release(self, row: int) -> None:
        """Forget row ``row`` (its sequence finished or was swapped out)."""
        self._row(row)
        self.pages[row] = 0

    def extend_to(self, rows: Sequence[int] | np.ndarray, kv_lens: Sequence[int] | np.ndarray,
                  block_tables: Sequence[Sequence[int]]) -> int:
        """Record, for every row whose table is shorter than ``ceil(kv_len / block_size)``
        pages, the missing pages from the host-side ``block_tables[i]`` (the
        allocator's lists, sequence i = rows[i]). Returns the pages recorded."""
        rows = np.asarray(rows, dtype=np.int64)
        kv = np.asarray(kv_lens, dtype=np.int64)
        if rows.size and (int(rows.min()) < 0 or int(rows.max()) >= self.max_seqs):
            raise IndexError(f"rows outside [0, {self.max_seqs})")
        need = (kv + self.block_size - 1) // self.block_size
        have = self.pages[rows]
        short = np.nonzero(need > have)[0]
        if not short.size:
            return 0
        if int(need[short].max()) > self.max_pages:
            i = int(short[np.argmax(need[short])])
            raise ValueError(f"row {int(rows[i])}: {int(need[i])} pages exceed max_pages={self.max_pages}")
        ids: list[int] = []
        for i in short.tolist():  # the new blocks of every growing row, in row order
            t, h, w = block_tables[i], int(have[i]), int(need[i])
            if len(t) < w:
                raise ValueError(f"seq {i}: {len(t)} blocks hold fewer than kv_len={int(kv[i])} tokens")
            ids.extend(t[h:w])
        idv = np.asarray(ids, dtype=np.int64)
        if int(idv.min()) < 0 or int(idv.max()) >= self.num_blocks:
            raise IndexError(f"block ids outside [0, {self.num_blocks})")
        cnt = need[short] - have[short]
        r = rows[short]
        first = np.cumsum(cnt) - cnt
        page = np.arange(idv.shape[0], dtype=np.int64) - np.repeat(first, cnt) + np.repeat(have[short], cnt)
        self._upd.append((np.repeat(r, cnt).astype(np.int32), page.astype(np.int32), idv.astype(np.int32)))
        self._n_upd += int(idv.shape[0])
        rl = r.tolist()
        if len(set(rl)) < len(rl) or not self._upd_rows.isdisjoint(rl):
            self._upd_dup = True
        self._upd_rows.update(rl)
        self.pages[r] = need[short]
        return int(idv.shape[0])

    # -- assembly -----------------------------------------------------------------

    def build_batch_meta(self, rows: Sequence[int] | np.ndarray, query_lens: Sequence[int] | np.ndarray,
                         kv_lens: Sequence[int] | np.ndarray) -> BatchMeta:
        """The ``BatchMeta`` of one step: sequence i is table row ``rows[i]``
        with ``query_lens[i]`` new tokens and ``kv_lens[i]`` tokens after this
        step's append (the reference's ordering contract, ``batch.py:40-46``).
        Applies the recorded table edits first. Fields are computed on the
        device, in stream order on the current stream."""
        rows = np.asarray(rows, dtype=np.int32)
        ql = np.asarray(query_lens, dtype=np.int64)
        kv = np.asarray(kv_lens, dtype=np.int64)
        n = int(rows.shape[0])
        if n == 0:
            raise ValueError("build_batch_meta() called with an empty sequence list")
        if ql.shape[0] != n or kv.shape[0] != n:
            raise ValueError(f"{n} rows but {ql.shape[0]} query lengths and {kv.shape[0]} kv lengths")
        if n > self.max_seqs:
            raise ValueError(f"{n} sequences exceed max_seqs={self.max_seqs}")
        q_min, q_max = int(ql.min()), int(ql.max())
        if q_min <= 0:
            i = int(np.argmax(ql <= 0))
            raise ValueError(f"seq {i} contributes {int(ql[i])} tokens; every sequence must contribute >= 1")
        if (ql > kv).any():
            i = int(np.argmax(ql > kv))
            raise ValueError(f"seq {i} contributes {int(ql[i])} tokens but holds only {int(kv[i])}; "
                             "grow the block table (blocks.append) before assembly")
        if int(rows.min()) < 0 or int(rows.max()) >= self.max_seqs:
            raise ValueError(f"rows outside [0, {self.max_seqs})")
        need = (kv + self.block_size - 1) // self.block_size
        have = self.pages[rows]
        if (have < need).any():
            i = int(np.argmax(have < need))
            raise ValueError(f"seq {i}: {int(have[i])} blocks hold fewer than kv_len={int(kv[i])} tokens")
        T, TP = int(ql.sum()), int(need.sum())
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed max_tokens={self.max_tokens}")
        slot = self._ring[self._next]
        self._next = (self._next + 1) % len(self._ring)
        if slot.used:
            slot.event.synchronize()  # its staging copy (and earlier readers) are done
        if self._upd_dup:
            self._dedupe()
        nu = self._n_upd
        words = 3 * n + 3 * nu
        if words > slot.host_np.shape[0]:
            slot.resize_input(self.device, max(words, 2 * slot.host_np.shape[0]))
        h = slot.host_np
        h[:n] = rows
        h[n:2 * n] = ql
        h[2 * n:3 * n] = kv
        if nu:
            o = 3 * n
            for part in range(3):
                h[o + part * nu:o + (part + 1) * nu] = np.concatenate([u[part] for u in self._upd])
        N.check(self._lib.pkv_build_batch_meta(self._desc_ref, slot.host_ptr, slot.dev.data_ptr(), n, nu,
                                               slot.desc_ref, self._status_ptr, N.raw_stream(self._dev_index)),
                "build_batch_meta")
        slot.event.record(torch.cuda.current_stream(self.device))  # the stream the kernels went to
        slot.used = True
        self._upd.clear()
        self._n_upd = 0
        self._upd_rows.clear()
        self._upd_dup = False
        self.n_builds += 1
        b, off = slot.i32, slot.off
        return BatchMeta(
            query_lens=b[off["query_lens"]:off["query_lens"] + n],
            cu_query_lens=b[off["cu_query_lens"]:off["cu_query_lens"] + n + 1],
            kv_lens=b[off["kv_lens"]:off["kv_lens"] + n],
            positions=slot.pos[:T],
            last_token_ix=b[off["last_token_ix"]:off["last_token_ix"] + n],
            kv_indptr=b[off["kv_indptr"]:off["kv_indptr"] + n + 1],
            kv_indices=b[off["kv_indices"]:off["kv_indices"] + TP],
            kv_last_page_len=b[off["kv_last_page_len"]:off["kv_last_page_len"] + n],
            batch_indices=b[off["batch_indices"]:off["batch_indices"] + T],
            slot_mapping=b[off["slot_mapping"]:off["slot_mapping"] + T],
            page_size=self.block_size,
            is_prefill=q_max > 1,
            max_query_len=q_max,
            min_query_len=q_min,
            checked_blocks=self.num_blocks,
        )

    def check_status(self) -> None:
        """Synchronise and raise if an assembly kernel flagged a violation."""
        bits = int(self.status.item())
        if bits:
            self.status.zero_()
            raise N.PkvError(N.PKV_ERR_DEVICE, f"device status {bits:#x}: {N.describe_status(bits)}")

    # -- helpers -------------------------------------------------------------------

    def _row(self, row: int) -> None:
        if not 0 <= int(row) < self.max_seqs:
            raise IndexError(f"row {row} outside [0, {self.max_seqs})")

    def _ids(self, row: int, block_ids: Sequence[int] | np.ndarray) -> np.ndarray:
        self._row(row)
        ids = np.asarray(block_ids, dtype=np.int64).reshape(-1)
        if ids.shape[0] > self.max_pages:
            raise ValueError(f"row {row}: {ids.shape[0]} pages exceed max_pages={self.max_pages}")
        if ids.shape[0] and (int(ids.min()) < 0 or int(ids.max()) >= self.num_blocks):
            raise IndexError(f"row {row}: block ids outside [0, {self.num_blocks})")
        return ids

    def _record(self, row: int, start: int, ids: np.ndarray) -> None:
        k = ids.shape[0]
        if not k:
            return
        self._upd.append((np.full(k, row, dtype=np.int32), np.arange(start, start + k, dtype=np.int32),
                          ids.astype(np.int32)))
        self._n_upd += k
        if row in self._upd_rows:
            self._upd_dup = True
        self._upd_rows.add(int(row))

    def _dedupe(self) -> None:
        """Keep only the last recorded edit of each (row, page): the kernel
        applies edits in parallel, in no particular order."""
        r, p, b = (np.concatenate([u[i] for u in self._upd]) for i in range(3))
        key = r.astype(np.int64) * self.max_pages + p
        _, first_in_reversed = np.unique(key[::-1], return_index=True)
        keep = np.sort(key.shape[0] - 1 - first_in_reversed)
        self._upd = [(r[keep], p[keep], b[keep])]
        self._n_upd = int(keep.shape[0])
