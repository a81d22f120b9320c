"""
Greedy sampling on the GPU, replacing the reference scheduler's
``next_ids = torch.argmax(logits, dim=-1).tolist()`` (serving/scheduler/
scheduler.py:756-757), which makes the host wait for every step it issues.

* ``sample_greedy`` runs ``pkv_sample_greedy`` (one launch): the argmax of each
  logits row with ``torch.argmax``'s result (first index of the maximum, NaN
  counted as the maximum), written to a compact ``[n_rows]`` int64 tensor and,
  when a token table and a row map are given, to ``tokens[rows[i]]`` — the
  table a device-fed decode loop assembles the next step's input from.
* ``TokenReadback`` moves each step's sampled tokens to pinned host memory on a
  side stream and hands them to the host one step later, so the host schedules
  step s+1 while step s still runs (the host needs only lengths to schedule).
"""

from __future__ import annotations

from collections import deque
from typing import Any

import torch

from . import _native as N

_LOGIT_DTYPES = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}


def sample_greedy(logits: torch.Tensor, out: torch.Tensor | None = None, tokens: torch.Tensor | None = None,
                  rows: torch.Tensor | None = None, status: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy token of each row of ``logits`` ``[n_rows, vocab]`` (fp16, bf16 or
    fp32 on a CUDA device, unit stride along the vocabulary).

    Returns ``out`` (int64 ``[n_rows]``, allocated when not given). With
    ``tokens`` (a device int64 token table) and ``rows`` (int32 ``[n_rows]``, on
    the device), row ``i``'s token is also written to ``tokens[rows[i]]``; a
    negative ``rows[i]`` writes nothing there. ``status`` (a device int32 word)
    receives ``PKV_DEV_SLOT_OOB`` for a row index past the table."""
    if logits.dim() != 2:
        raise ValueError(f"logits must be 2-D [n_rows, vocab], got shape {tuple(logits.shape)}")
    if logits.dtype not in _LOGIT_DTYPES:
        raise ValueError(f"logits dtype {logits.dtype} not supported (fp16, bf16, fp32)")
    if logits.device.type != "cuda":
        raise ValueError("sample_greedy runs on the GPU; logits are on " + str(logits.device))
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    n, vocab = logits.shape
    dev = logits.device
    if out is None:
        out = torch.empty(n, dtype=torch.int64, device=dev)
    elif out.dtype != torch.int64 or out.device != dev or out.numel() < n or not out.is_contiguous():
        raise ValueError("out must be a contiguous int64 tensor of n_rows entries on the logits' device")
    tok_ptr, tok_len, row_ptr = None, 0, None
    if tokens is not None:
        if tokens.dtype != torch.int64 or tokens.device != dev or not tokens.is_contiguous():
            raise ValueError("tokens must be a contiguous int64 tensor on the logits' device")
        if rows is None:
            raise ValueError("a token table needs rows (the table entry of each logits row)")
        tok_ptr, tok_len = tokens.data_ptr(), tokens.numel()
    if rows is not None:
        if tokens is None:
            raise ValueError("rows given without a token table")
        if rows.dtype != torch.int32 or rows.device != dev or rows.numel() != n or not rows.is_contiguous():
            raise ValueError("rows must be a contiguous int32 tensor of n_rows entries on the logits' device")
        row_ptr = rows.data_ptr()
    if n == 0:
        return out
    with torch.cuda.device(dev):
        N.check(N.lib().pkv_sample_greedy(_LOGIT_DTYPES[logits.dtype], logits.data_ptr(), n, vocab,
                                          logits.stride(0), row_ptr, tok_ptr, tok_len, out.data_ptr(),
                                          N.ptr(status), N.raw_stream(dev.index)),
                "sample_greedy")
    return out


class TokenReadback:
    """Sampled tokens to the host one step late.

    ``submit(sampled, tag)`` queues a copy of this step's device tokens into
    pinned host memory on a side stream (after the work already queued on the
    current stream); ``collect(keep)`` waits for and returns, oldest first, the
    ``(tag, tokens)`` of all submissions but the newest ``keep``. With
    ``keep=1`` after each step the host receives step s-1's tokens while step s
    runs; ``collect(0)`` drains everything."""

    def __init__(self, device: torch.device | str):
        self.device = torch.device(device)
        self.stream = torch.cuda.Stream(self.device)
        self._pending: deque[tuple[Any, torch.Tensor, torch.cuda.Event]] = deque()

    def submit(self, sampled: torch.Tensor, tag: Any = None) -> None:
        host = torch.empty(sampled.shape, dtype=sampled.dtype, pin_memory=True)
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(ready)
            host.copy_(sampled, non_blocking=True)
            sampled.record_stream(self.stream)
            done = torch.cuda.Event()
            done.record(self.stream)
        self._pending.append((tag, host, done))

    def collect(self, keep: int = 1) -> list[tuple[Any, torch.Tensor]]:
        got = []
        while len(self._pending) > keep:
            tag, host, done = self._pending.popleft()
            done.synchronize()
            got.append((tag, host))
        return got

    def __len__(self) -> int:
        return len(self._pending)
