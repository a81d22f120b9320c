"""
Test-side stand-ins for the block manager the backend sits behind.

``FifoAllocator`` / ``Seq`` restate the behaviour of the reference's
``BlockAllocator`` (FIFO free list: blocks freed in some order are handed back
in that order, ``serving/memory/allocator.py:53-262``) and ``SequenceBlocks``
(``serving/memory/block_table.py:37-181``) — just enough to build fragmented,
scattered page tables on a machine where the reference is not installed.
"""

from __future__ import annotations

from collections import deque

import numpy as np
import torch

from llm_serving_layer_b200.meta import BatchMeta, build_meta


class FifoAllocator:
    def __init__(self, num_blocks: int, block_size: int, order=None):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self._free = deque(range(num_blocks) if order is None else [int(b) for b in order])

    def allocate(self, n: int) -> list[int]:
        if n > len(self._free):
            raise RuntimeError(f"out of blocks: want {n}, have {len(self._free)}")
        return [self._free.popleft() for _ in range(n)]

    def free(self, ids) -> None:
        self._free.extend(int(b) for b in ids)


class Seq:
    def __init__(self, alloc: FifoAllocator, seq_id: int = 0):
        self.alloc = alloc
        self.seq_id = seq_id
        self.block_size = alloc.block_size
        self.block_ids: list[int] = []
        self.num_tokens = 0
        self.is_freed = False

    def append(self, n: int) -> None:
        total = self.num_tokens + n
        need = (total + self.block_size - 1) // self.block_size - len(self.block_ids)
        if need > 0:
            self.block_ids.extend(self.alloc.allocate(need))
        self.num_tokens = total

    def slot_for(self, p: int) -> int:
        return self.block_ids[p // self.block_size] * self.block_size + p % self.block_size

    def free(self) -> None:
        if not self.is_freed:
            self.alloc.free(self.block_ids)
            self.block_ids = []
            self.num_tokens = 0
            self.is_freed = True


def meta_for(seqs: list[Seq], qlens: list[int], device="cpu") -> BatchMeta:
    return build_meta([s.block_ids for s in seqs], [s.num_tokens for s in seqs], qlens,
                      seqs[0].block_size, device=device)


def slots_meta(slots) -> BatchMeta:
    """A write-only descriptor for appending arbitrary slots (history writes)."""
    s = torch.as_tensor(np.asarray(slots), dtype=torch.int32)
    n = int(s.shape[0])
    z = torch.zeros(1, dtype=torch.int32)
    return BatchMeta(query_lens=z, cu_query_lens=torch.zeros(2, dtype=torch.int32), kv_lens=z,
                     positions=torch.zeros(n, dtype=torch.int64), last_token_ix=z,
                     kv_indptr=torch.zeros(2, dtype=torch.int32), kv_indices=torch.zeros(0, dtype=torch.int32),
                     kv_last_page_len=z, batch_indices=torch.zeros(n, dtype=torch.int32), slot_mapping=s)
