"""
Greedy sampling on the GPU (``pkv_sample_greedy`` through ``sample_greedy``)
against numpy's argmax of the same rows: the scheduler's
``torch.argmax(logits, dim=-1)`` (serving/scheduler/scheduler.py:756-757), whose
result is the first index of each row's maximum, a NaN counting as the maximum.

Covers fp32 / fp16 / bf16 logits; one row to more rows than the GPU has SMs
(rows split over thread-block clusters and rows one CTA each); Llama's 128256
vocabulary and odd sizes; ties placed inside one CTA's share and across the
shares of a cluster; NaNs; -0 against +0; rows of -inf; strided and unaligned
rows (the scalar path); and the token-table scatter (rows skipped with -1, a
row index past the table flagged and skipped), and the one-step-late readback.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from llm_serving_layer_b200 import TokenReadback, sample_greedy
from llm_serving_layer_b200 import _native as N

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
DTYPES = [torch.float32, torch.float16, torch.bfloat16]


def want_argmax(x: torch.Tensor) -> np.ndarray:
    """numpy's argmax of the rows, on an exact fp32 copy (first maximum; the
    first NaN when a row holds one)."""
    return np.argmax(x.float().cpu().numpy(), axis=1).astype(np.int64)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n,vocab", [(1, 128256), (3, 128256), (37, 128256), (300, 128256), (1100, 4096),
                                     (5, 1), (7, 7), (64, 50001), (2, 100003)])
def test_greedy_matches_numpy_argmax(dtype, n, vocab):
    g = torch.Generator(device=DEV).manual_seed(n * 7919 + vocab)
    x = torch.randn(n, vocab, device=DEV, generator=g).to(dtype)
    got = sample_greedy(x)
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy(), want_argmax(x))
    assert torch.equal(got, x.argmax(-1))


@pytest.mark.parametrize("dtype", DTYPES)
def test_ties_go_to_the_first_index_within_and_across_cluster_shares(dtype):
    n, vocab = 6, 128256
    x = torch.randn(n, vocab, device=DEV).to(dtype)
    spots = [[5, 100, 7000], [vocab - 1, vocab - 2], [64000, 64001, 127999], [3, 64128, 96192],
             [0, vocab - 1], [31, 32, 33, 40000]]
    for r, idx in enumerate(spots):
        x[r, idx] = 40.0
    got = sample_greedy(x).cpu().numpy()
    assert got.tolist() == [min(s) for s in spots]
    assert np.array_equal(got, want_argmax(x))


@pytest.mark.parametrize("dtype", DTYPES)
def test_nan_signed_zero_and_infinities(dtype):
    vocab = 20000
    x = torch.randn(5, vocab, device=DEV).to(dtype)
    x[0, 9] = float("nan")
    x[0, 3] = float("nan")           # the first NaN wins
    x[0, 1] = float("inf")
    x[1] = -0.0
    x[1, 10] = 0.0                   # -0 == +0: the first zero wins
    x[2] = float("-inf")             # all -inf: index 0
    x[3, 77] = float("inf")
    x[3, 12000] = float("inf")
    x[4] = -1e4 if dtype != torch.float16 else -6e4
    x[4, 19999] = -1.0
    got = sample_greedy(x).cpu().numpy()
    assert got.tolist() == [3, 0, 0, 77, 19999]
    assert np.array_equal(got, want_argmax(x))


@pytest.mark.parametrize("dtype", DTYPES)
def test_strided_and_unaligned_rows(dtype):
    base = torch.randn(9, 30011, device=DEV).to(dtype)
    for view in (base[:, :30000], base[:, 1:], base[1:, 3:30003]):
        got = sample_greedy(view)
        assert np.array_equal(got.cpu().numpy(), want_argmax(view))


def test_token_table_scatter_skips_and_flags():
    n, vocab = 40, 128256
    x = torch.randn(n, vocab, device=DEV, dtype=torch.float16)
    table = torch.full((64,), -7, dtype=torch.int64, device=DEV)
    rows = torch.arange(n, dtype=torch.int32, device=DEV) + 10
    rows[::3] = -1                   # rows that sample nothing into the table (mid-prefill)
    rows[5] = 64                     # past the table: skipped, flagged
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.empty(n, dtype=torch.int64, device=DEV)
    sample_greedy(x, out=out, tokens=table, rows=rows, status=status)
    torch.cuda.synchronize()
    want = want_argmax(x)
    assert np.array_equal(out.cpu().numpy(), want)
    t = table.cpu().numpy()
    r = rows.cpu().numpy()
    expect = np.full(64, -7)
    for i in range(n):
        if 0 <= r[i] < 64:
            expect[r[i]] = want[i]
    assert np.array_equal(t, expect)
    assert int(status.item()) == N.DEV_SLOT_OOB


def test_readback_one_step_late_returns_every_step_in_order():
    rb = TokenReadback(DEV)
    table = torch.zeros(16, dtype=torch.int64, device=DEV)
    rows = torch.arange(16, dtype=torch.int32, device=DEV)
    seen, wants = [], []
    for step in range(5):
        x = torch.randn(16, 5000, device=DEV, dtype=torch.bfloat16)
        wants.append(want_argmax(x))
        rb.submit(sample_greedy(x, tokens=table, rows=rows), tag=step)
        seen += rb.collect(keep=1)
        assert len(rb) == 1
    seen += rb.collect(keep=0)
    assert [t for t, _ in seen] == list(range(5))
    for (_, host), w in zip(seen, wants):
        assert np.array_equal(host.numpy(), w)
    assert np.array_equal(table.cpu().numpy(), wants[-1])


def test_argument_errors():
    x = torch.randn(4, 10, device=DEV)
    with pytest.raises(ValueError):
        sample_greedy(x.double())
    with pytest.raises(ValueError):
        sample_greedy(x[0])
    with pytest.raises(ValueError):
        sample_greedy(x, rows=torch.zeros(4, dtype=torch.int32, device=DEV))
    lib = N.lib()
    assert lib.pkv_sample_greedy(2, x.data_ptr(), 4, 10, 5, None, None, 0, x.data_ptr(), None, None) == N.PKV_ERR_ARG
    assert b"row_stride" in lib.pkv_last_error()
