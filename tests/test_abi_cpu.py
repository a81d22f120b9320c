"""
CPU-side checks of the C-ABI library and the host logic (no GPU, no compute):
the library builds, loads and exports exactly what ``include/pkv.h`` declares;
argument validation rejects bad input before touching a device; the Python
drop-ins refuse a non-CUDA device instead of falling back.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from llm_serving_layer_b200 import _native as N
from llm_serving_layer_b200 import build as B
from llm_serving_layer_b200.meta import BatchMeta, build_meta

HEADER = Path(__file__).resolve().parents[1] / "include" / "pkv.h"


@pytest.fixture(scope="module")
def lib():
    B.build()
    return N.lib()


def declared_symbols() -> set[str]:
    return set(re.findall(r"^PKV_API\s+[\w\s\*]+?\b(pkv_\w+)\s*\(", HEADER.read_text(), flags=re.M))


def test_library_exports_every_declared_symbol(lib):
    names = declared_symbols()
    assert len(names) >= 17
    for n in names:
        assert hasattr(lib, n), f"{n} declared in pkv.h but not exported"
    assert names == set(N.SIGNATURES), "ctypes signature table out of sync with pkv.h"
    assert lib.pkv_version() >= 100


def test_argument_errors_are_reported_without_a_device(lib):
    assert lib.pkv_append_kv(None, 0, None, None, None, 1, None, None) == N.PKV_ERR_ARG
    assert b"NULL" in lib.pkv_last_error()
    pool = N.PoolDesc(0x1000, 0, 1, 16, 8, 64, 0, 0)  # num_blocks 0
    assert lib.pkv_copy_block(ctypes.byref(pool), 0, 1, None) == N.PKV_ERR_ARG
    pool = N.PoolDesc(0x1000, 8, 2, 16, 8, 64, 0, 0)
    assert lib.pkv_copy_block(ctypes.byref(pool), 0, 8, None) == N.PKV_ERR_ARG
    assert b"outside [0, 8)" in lib.pkv_last_error()
    assert lib.pkv_append_kv(ctypes.byref(pool), 2, None, None, None, 1, None, None) == N.PKV_ERR_ARG
    assert b"layer_idx 2" in lib.pkv_last_error()
    pool_bad = N.PoolDesc(0x1001, 8, 2, 16, 8, 64, 0, 0)  # misaligned base
    assert lib.pkv_swap_gather(ctypes.byref(pool_bad), None, 1, None, None, None) == N.PKV_ERR_ARG
    pool_dt = N.PoolDesc(0x1000, 8, 2, 16, 8, 64, 9, 0)
    assert lib.pkv_plan(ctypes.byref(pool_dt), 32, None, None, 0, None) == N.PKV_ERR_ARG
    # zero-size work is a successful no-op that launches nothing
    assert lib.pkv_append_kv(ctypes.byref(pool), 0, None, None, None, 0, None, None) == N.PKV_OK
    assert lib.pkv_copy_block(ctypes.byref(pool), 3, 3, None) == N.PKV_OK


def test_workspace_size_covers_the_page_table(lib):
    pool = N.PoolDesc(0x1000, 8, 2, 16, 8, 64, 0, 0)
    a = lib.pkv_attend_workspace_size(ctypes.byref(pool), 32, 256, 4300, 1)
    b = lib.pkv_attend_workspace_size(ctypes.byref(pool), 32, 256, 8600, 1)
    assert b - a >= 4300 * 8 - 256  # one 8-byte descriptor per page (256-byte aligned)


def test_backend_refuses_cpu_device():
    from llm_serving_layer_b200 import B200PagedBackend
    with pytest.raises(ValueError, match="CUDA device"):
        B200PagedBackend(1, 8, 16, 2, 4, 8, device="cpu", dtype=torch.float32)
    with pytest.raises(ValueError, match="divisible"):
        B200PagedBackend(1, 8, 16, 3, 4, 8, device="cpu")
    with pytest.raises(ValueError, match="must be positive"):
        B200PagedBackend(0, 8, 16, 2, 4, 8, device="cpu")


def test_build_meta_fields_and_rejections():
    m = build_meta([[5, 2], [9]], [21, 1], [1, 1], 16)
    assert m.slot_mapping.tolist() == [2 * 16 + 4, 9 * 16 + 0]
    assert m.kv_last_page_len.tolist() == [5, 1]
    assert m.positions.tolist() == [20, 0]
    assert m.kv_indptr.tolist() == [0, 2, 3] and m.kv_indices.tolist() == [5, 2, 9]
    assert not m.is_prefill
    m.validate()
    with pytest.raises(ValueError, match="empty"):
        build_meta([], [], [], 16)
    with pytest.raises(ValueError, match="contributes 0"):
        build_meta([[1]], [4], [0], 16)
    with pytest.raises(ValueError, match="blocks.append"):
        build_meta([[1]], [2], [5], 16)
    with pytest.raises(ValueError, match="fewer than"):
        build_meta([[1]], [17], [1], 16)
    # a full last page reports block_size, never 0
    m = build_meta([[3, 4]], [32], [32], 16)
    assert m.kv_last_page_len.tolist() == [16] and m.is_prefill


def test_batchmeta_validate_messages():
    import dataclasses
    m = build_meta([[0, 1]], [32], [1], 16)
    with pytest.raises(AssertionError, match="kv_last_page_len"):
        dataclasses.replace(m, kv_last_page_len=torch.tensor([0], dtype=torch.int32)).validate()
    with pytest.raises(AssertionError, match="pages allocated"):
        dataclasses.replace(m, kv_lens=torch.tensor([999], dtype=torch.int32)).validate()
    with pytest.raises(AssertionError, match="batch_indices"):
        dataclasses.replace(m, batch_indices=torch.tensor([0, 0], dtype=torch.int32)).validate()


def test_kernel_selection_for_batch_shapes(lib):
    """pkv_attend_kernel is host-only: which kernel each batch shape and hint
    takes (decode for pure decode, the tensor-core prefill kernel for
    chunked / mixed batches, the generic kernel elsewhere)."""
    import ctypes
    buf = (ctypes.c_char * 64)()
    base = (ctypes.addressof(buf) + 15) & ~15

    def pool(dtype, n_kv=8, head_dim=64, block=16):
        return N.PoolDesc(base, 64, 2, block, n_kv, head_dim, dtype, 0)

    K = {0: "generic", 1: "decode", 2: "prefill"}
    f16, f32 = 0, 2
    cases = [
        (pool(f16), 32, 256, 256, 1, "decode"),
        (pool(f16), 32, 4, 700, 0, "prefill"),     # chunked prefill / mixed
        (pool(f16), 32, 4, 700, 2, "prefill"),     # pure prefill
        (pool(f16), 32, 3, 3, 0, "generic"),       # q_lens like [2, 0, 1]: n_tokens == n_seqs, not decode
        (pool(f32), 32, 256, 256, 1, "generic"),   # fp32 pools: CUDA-core kernel
        (pool(f16, head_dim=128), 32, 4, 700, 0, "generic"),
        (pool(f16, n_kv=8), 24, 4, 700, 0, "generic"),  # 3 query heads per KV head
        (pool(f16, n_kv=4), 32, 8, 8, 1, "decode"),     # 8 query heads per KV head
        (pool(1), 32, 4, 700, 0, "prefill"),       # bf16
    ]
    for p, hq, n, t, hint, want in cases:
        got = lib.pkv_attend_kernel(ctypes.byref(p), hq, n, t, hint)
        assert K[got] == want, (p.dtype, p.head_dim, p.n_kv_heads, hq, n, t, hint, got)
    assert lib.pkv_attend_kernel(ctypes.byref(pool(f16)), 30, 4, 700, 0) < 0  # 30 % 8 != 0
