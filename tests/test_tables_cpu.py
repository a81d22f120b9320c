"""
Host-side bookkeeping of ``DeviceBlockTables`` (no GPU): the table edits it
records (bind / extend / extend_to / set_block / release), the reduction of two
edits of one (row, page) to the last, and the reference's errors that
``build_batch_meta`` raises before anything is queued (``ValueError`` for an
empty batch, a sequence contributing no tokens, a query longer than its
history, a table shorter than ``kv_len``; ``IndexError`` for block ids outside
the pool). The device side is ``tests/test_gpu_tables.py``.
"""

from __future__ import annotations

import numpy as np
import pytest

from llm_serving_layer_b200.tables import DeviceBlockTables


def host_tables(max_seqs=8, max_pages=6, block_size=16, num_blocks=100, max_tokens=64):
    """The object without its device buffers: only the host bookkeeping."""
    bt = object.__new__(DeviceBlockTables)
    bt.max_seqs, bt.max_pages, bt.block_size = max_seqs, max_pages, block_size
    bt.num_blocks, bt.max_tokens = num_blocks, max_tokens
    bt.pages = np.zeros(max_seqs, dtype=np.int64)
    bt._upd, bt._n_upd, bt._upd_rows, bt._upd_dup = [], 0, set(), False
    return bt


def edits(bt):
    if not bt._upd:
        return []
    r, p, b = (np.concatenate([u[i] for u in bt._upd]) for i in range(3))
    return list(zip(r.tolist(), p.tolist(), b.tolist()))


def test_bind_extend_set_release_record_the_changed_entries():
    bt = host_tables()
    bt.bind(2, [10, 11])
    bt.extend(2, [12])
    bt.set_block(2, 1, 40)
    assert bt.pages[2] == 3
    assert edits(bt) == [(2, 0, 10), (2, 1, 11), (2, 2, 12), (2, 1, 40)]
    assert bt._upd_dup  # row 2 edited more than once
    bt._dedupe()
    assert sorted(edits(bt)) == [(2, 0, 10), (2, 1, 40), (2, 2, 12)]
    bt.release(2)
    assert bt.pages[2] == 0


def test_extend_to_records_only_the_missing_pages():
    bt = host_tables()
    tables = [[5, 6, 7, 8], [9, 10], [11, 12, 13]]
    assert bt.extend_to([3, 0, 6], [40, 17, 33], tables) == 8
    assert edits(bt) == [(3, 0, 5), (3, 1, 6), (3, 2, 7), (0, 0, 9), (0, 1, 10), (6, 0, 11), (6, 1, 12), (6, 2, 13)]
    assert bt.pages[[3, 0, 6]].tolist() == [3, 2, 3]
    bt._upd.clear()
    bt._n_upd = 0
    assert bt.extend_to([3, 0, 6], [41, 20, 33], tables) == 0  # still inside their pages
    assert bt.extend_to([3, 0, 6], [64, 20, 33], tables) == 1
    assert edits(bt) == [(3, 3, 8)]


def test_edit_errors():
    bt = host_tables()
    with pytest.raises(IndexError, match="block ids outside"):
        bt.bind(0, [100])
    with pytest.raises(IndexError, match="row 8 outside"):
        bt.bind(8, [1])
    with pytest.raises(ValueError, match="exceed max_pages"):
        bt.bind(0, list(range(7)))
    bt.bind(0, [1, 2])
    with pytest.raises(IndexError, match="page 2 does not exist"):
        bt.set_block(0, 2, 3)
    with pytest.raises(ValueError, match="blocks hold fewer than kv_len=48"):
        bt.extend_to([1], [48], [[4, 5]])
    with pytest.raises(ValueError, match="exceed max_pages"):
        bt.extend_to([1], [7 * 16], [list(range(7))])
    with pytest.raises(IndexError, match="rows outside"):
        bt.extend_to([9], [3], [[1]])


def test_build_errors_before_any_device_work():
    bt = host_tables()
    bt.bind(0, [1, 2])
    with pytest.raises(ValueError, match="empty sequence list"):
        bt.build_batch_meta([], [], [])
    with pytest.raises(ValueError, match="contributes 0 tokens"):
        bt.build_batch_meta([0], [0], [5])
    with pytest.raises(ValueError, match="holds only"):
        bt.build_batch_meta([0], [6], [5])
    with pytest.raises(ValueError, match="blocks hold fewer than kv_len=33"):
        bt.build_batch_meta([0], [1], [33])
    with pytest.raises(ValueError, match="rows outside"):
        bt.build_batch_meta([8], [1], [1])
    with pytest.raises(ValueError, match="max_tokens"):
        bt.bind(1, [3, 4, 5, 6, 7])
        bt.build_batch_meta([1], [65], [65])
