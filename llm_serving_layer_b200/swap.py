"""
B200SwapSpace — preemption swap between the device pool and pinned host memory.

A drop-in for the reference's ``KVSwapSpace`` (``serving/scheduler/preemption.py:
335-523``): same constructor (``backend, max_bytes=None``), same methods
(``swap_out``, ``swap_in``, ``release``, ``bytes_for``), same accounting
(``bytes_in_use``, ``peak_bytes``, ``last_swap_out_seconds``, ``num_swapped``),
same errors (``RuntimeError`` "resume mismatch" / freed sequence, the budget
exception ``SwapSpaceFull``) and the same host layout: a handle's ``k`` / ``v``
are ``(num_layers, nb, block_size, n_kv_heads, head_dim)`` pinned tensors,
host index ``i`` = the sequence's ``i``-th block.

Mechanism (``libpkv`` swap engine): one gather kernel per chunk copies the
sequence's scattered 16 KiB page tiles into a bounded, double-buffered device
staging area; the copy engine moves each chunk to pinned host memory on a
private stream while the next chunk is gathered. Events order it against the
compute stream: the gather starts after everything already queued there, and
compute work queued afterwards waits only for the gather (not the PCIe
transfer), so the caller may free the blocks as soon as ``swap_out`` returns —
the race the reference avoids with a synchronous copy is closed by an event.
Swap-in runs the reverse (host -> staging -> scatter kernel).

``synchronous=True`` (the default, the reference's semantics) waits for the
transfer before returning, so ``handle.k`` / ``handle.v`` are readable at once.
With ``synchronous=False`` they become readable after ``wait(handle)``;
``swap_in`` and ``release`` order themselves after the transfer automatically.
"""

from __future__ import annotations

import ctypes
import sys
import time
from dataclasses import dataclass, field
from typing import Any

import torch

from . import _native as N
from .backend import B200PagedBackend

__all__ = ["B200SwapSpace", "SwapHandle", "SwapSpaceFull"]


class SwapSpaceFull(RuntimeError):
    """Host swap budget exhausted. Callers degrade to recompute rather than fail."""


def _host_full_exception() -> type[Exception]:
    """The serving scheduler catches ``serving.scheduler.preemption.SwapSpaceFull``;
    when that module is loaded, raise its class so the drop-in is caught there."""
    mod = sys.modules.get("serving.scheduler.preemption")
    exc = getattr(mod, "SwapSpaceFull", None) if mod is not None else None
    return exc if isinstance(exc, type) and issubclass(exc, Exception) else SwapSpaceFull


@dataclass
class SwapHandle:
    """One sequence's KV parked on the host (fields of ``preemption.py:303-333``)."""

    request_id: str
    seq_id: int
    num_tokens: int
    num_blocks: int
    k: torch.Tensor
    v: torch.Tensor
    nbytes: int
    block_size: int
    n_kv_heads: int
    head_dim: int
    released: bool = False
    ticket: int = 0
    _keep: list = field(default_factory=list, repr=False)


class B200SwapSpace:
    def __init__(self, backend: B200PagedBackend, max_bytes: int | None = None, *,
                 staging_bytes: int = 64 << 20, synchronous: bool = True,
                 full_exc: type[Exception] | None = None):
        for attr in ("k_pool", "v_pool", "num_layers", "block_size", "n_kv_heads", "head_dim"):
            if not hasattr(backend, attr):
                raise TypeError(
                    f"B200SwapSpace needs a paged backend exposing .{attr}; got {type(backend).__name__}"
                )
        if not hasattr(backend, "_pdesc"):
            raise TypeError("B200SwapSpace moves the pool of a B200PagedBackend")
        self.backend = backend
        self.max_bytes = max_bytes
        self.bytes_in_use = 0
        self.peak_bytes = 0
        self.last_swap_out_seconds = 0.0
        self.last_swap_in_seconds = 0.0
        self.synchronous = synchronous
        self.full_exc = full_exc or _host_full_exception()
        self._live: dict[int, SwapHandle] = {}
        self._pending: list[tuple[int, list]] = []
        self.device = backend.device
        self.dtype = backend.dtype
        self._lib = N.lib()
        bb = backend.block_bytes() // (2 * backend.num_layers)  # one block of one layer, K or V
        staging_bytes = max(int(staging_bytes), 2 * bb)
        self._staging = torch.empty(staging_bytes, dtype=torch.uint8, device=self.device)
        sw = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            N.check(self._lib.pkv_swapper_create(self._staging.data_ptr(), staging_bytes, ctypes.byref(sw)),
                    "swapper_create")
        self._sw = sw

    def __del__(self):
        sw = getattr(self, "_sw", None)
        if sw is not None and sw.value:
            try:
                with torch.cuda.device(self.device):
                    self._lib.pkv_swapper_destroy(sw)
            except Exception:
                pass
            self._sw = None

    # -- accounting ------------------------------------------------------------------

    def bytes_for(self, num_blocks: int) -> int:
        """Host bytes a ``num_blocks``-long sequence occupies: K and V, all layers."""
        return self.backend.block_bytes() * num_blocks

    @property
    def num_swapped(self) -> int:
        return len(self._live)

    # -- movement ---------------------------------------------------------------------

    def swap_out(self, request_id: str, blocks: Any) -> SwapHandle:
        """Copy every block of ``blocks`` (a ``SequenceBlocks``) to pinned host
        memory. Does not free them; the caller may free them on return."""
        if blocks.is_freed:
            raise RuntimeError(
                f"swap_out on freed SequenceBlocks(seq_id={blocks.seq_id}); its blocks may already "
                "belong to another sequence and the copy would capture someone else's KV."
            )
        ids = list(blocks.block_ids)
        nb = len(ids)
        want = self.bytes_for(nb)
        if self.max_bytes is not None and self.bytes_in_use + want > self.max_bytes:
            raise self.full_exc(
                f"swapping {nb} blocks needs {want} B; {self.bytes_in_use} B of "
                f"{self.max_bytes} B host swap space already in use"
            )
        t0 = time.perf_counter()
        bk = self.backend
        shape = (bk.num_layers, nb, bk.block_size, bk.n_kv_heads, bk.head_dim)
        k_host = torch.empty(shape, dtype=self.dtype, pin_memory=True)
        v_host = torch.empty(shape, dtype=self.dtype, pin_memory=True)
        handle = SwapHandle(request_id, blocks.seq_id, blocks.num_tokens, nb, k_host, v_host, want,
                            bk.block_size, bk.n_kv_heads, bk.head_dim)
        if nb:
            idx = self._ids(ids)
            ticket = ctypes.c_uint64(0)
            with torch.cuda.device(self.device):
                N.check(self._lib.pkv_swap_out(
                    self._sw, bk._pdesc, idx.data_ptr(), nb, k_host.data_ptr(), v_host.data_ptr(),
                    N.stream_ptr(self.device), bk._status.data_ptr(), ctypes.byref(ticket)), "swap_out")
            handle.ticket = ticket.value
            handle._keep.append(idx)
            if self.synchronous:
                self.wait(handle)
        self._live[id(handle)] = handle
        self.bytes_in_use += want
        self.peak_bytes = max(self.peak_bytes, self.bytes_in_use)
        self.last_swap_out_seconds = time.perf_counter() - t0
        return handle

    def swap_in(self, handle: SwapHandle, blocks: Any) -> None:
        """Restore a handle into freshly allocated blocks (``blocks`` already
        grown to ``handle.num_tokens``); the block COUNT must match exactly."""
        if handle.released:
            raise RuntimeError(f"swap_in on a released handle for {handle.request_id!r}")
        if blocks.num_tokens != handle.num_tokens:
            raise RuntimeError(
                f"resume mismatch for {handle.request_id!r}: block table holds "
                f"{blocks.num_tokens} tokens, handle holds {handle.num_tokens}"
            )
        if len(blocks.block_ids) != handle.num_blocks:
            raise RuntimeError(
                f"resume mismatch for {handle.request_id!r}: {len(blocks.block_ids)} blocks allocated, "
                f"{handle.num_blocks} swapped out. Logical block order would shift and attention "
                "would read a different history."
            )
        if handle.block_size != self.backend.block_size:
            raise RuntimeError(
                f"handle block_size={handle.block_size} != backend {self.backend.block_size}"
            )
        if handle.num_blocks == 0:
            return
        t0 = time.perf_counter()
        idx = self._ids(list(blocks.block_ids))
        ticket = ctypes.c_uint64(0)
        with torch.cuda.device(self.device):
            N.check(self._lib.pkv_swap_in(
                self._sw, self.backend._pdesc, idx.data_ptr(), handle.num_blocks, handle.k.data_ptr(),
                handle.v.data_ptr(), N.stream_ptr(self.device), self.backend._status.data_ptr(),
                ctypes.byref(ticket)), "swap_in")
        # the host buffers and ids must outlive the transfer
        self._pending.append((ticket.value, [idx, handle.k, handle.v]))
        if self.synchronous:
            self._wait_ticket(ticket.value)
        self._reap()
        self.last_swap_in_seconds = time.perf_counter() - t0

    def wait(self, handle: SwapHandle | None = None) -> None:
        """Block until ``handle``'s transfer (or every transfer) completed."""
        if handle is None:
            N.check(self._lib.pkv_swapper_wait(self._sw, 0), "swapper_wait")
            self._pending.clear()
            return
        if handle.ticket:
            self._wait_ticket(handle.ticket)
            handle.ticket = 0
            handle._keep.clear()

    def release(self, handle: SwapHandle) -> None:
        """Drop a handle's host memory. Idempotent."""
        if handle.released:
            return
        self.wait(handle)
        handle.released = True
        self._live.pop(id(handle), None)
        self.bytes_in_use -= handle.nbytes
        handle.k = torch.empty(0)
        handle.v = torch.empty(0)

    # -- internals ----------------------------------------------------------------------

    def _ids(self, ids: list[int]) -> torch.Tensor:
        t = torch.tensor(ids, dtype=torch.int32)
        if ids and (min(ids) < 0 or max(ids) >= self.backend.num_blocks):
            raise IndexError(f"block ids outside [0, {self.backend.num_blocks})")
        return t.pin_memory().to(self.device, non_blocking=True)

    def _wait_ticket(self, ticket: int) -> None:
        with torch.cuda.device(self.device):
            N.check(self._lib.pkv_swapper_wait(self._sw, ticket), "swapper_wait")

    def _reap(self) -> None:
        keep = []
        for t, refs in self._pending:
            if not self._lib.pkv_swapper_done(self._sw, t):
                keep.append((t, refs))
        self._pending = keep
