"""
B200PagedBackend — the paged-KV attention backend on hand-written sm_100a kernels.

A drop-in for the reference's ``PagedTorchBackend``
(``serving/backends/paged_torch.py:71-509``) and ``FlashInferBackend``
(``serving/backends/flashinfer_backend.py:233-734``): the same constructor, the
same ``append_kv`` / ``attend`` / ``copy_block`` methods, the same accounting
helpers, the same validation errors (``ValueError`` for shapes, layer index
and page-table inconsistencies; ``IndexError`` for ``copy_block`` ranges), and
``k_pool`` / ``v_pool`` as per-layer ``[num_blocks, block_size, n_kv_heads,
head_dim]`` tensors — here views into ONE allocation laid out
``[num_layers][K|V][num_blocks][block_size][n_kv_heads][head_dim]`` so that the
kernels address every layer from one base pointer and one TMA descriptor.

Every operation launches this package's CUDA kernels through ``libpkv.so``
(C ABI, ``include/pkv.h``) on ``torch.cuda.current_stream()``; there is no
torch or CPU fallback, and construction fails on a non-CUDA device.
"""

from __future__ import annotations

import ctypes
from typing import Any, Sequence

import torch

from . import _native as N

__all__ = ["B200PagedBackend"]


class B200PagedBackend:
    """Paged KV storage plus attention on B200 kernels.

    ``validate``:
      * ``"host"`` (default) — once per ``BatchMeta`` (cached by identity, as
        ``FlashInferBackend._ensure_planned`` caches its plan) the page table is
        read back and checked on the host, raising the reference's
        ``ValueError``s before any kernel runs; ``is_prefill`` is cross-checked
        against ``query_lens``.
      * ``"device"`` — no host round trip: kernels check the page table and OR
        violations into a device status word; ``check_status()`` raises them.
    """

    def __init__(
        self,
        num_layers: int,
        num_blocks: int,
        block_size: int,
        n_kv_heads: int,
        n_heads: int,
        head_dim: int,
        device: str | torch.device = "cuda:0",
        dtype: torch.dtype = torch.float16,
        *,
        validate: str = "host",
    ):
        if n_heads % n_kv_heads != 0:
            raise ValueError(
                f"n_heads={n_heads} must be divisible by n_kv_heads={n_kv_heads}; "
                "GQA maps query head h to KV head h // (n_heads // n_kv_heads)."
            )
        for name, val in (
            ("num_layers", num_layers), ("num_blocks", num_blocks), ("block_size", block_size),
            ("n_kv_heads", n_kv_heads), ("n_heads", n_heads), ("head_dim", head_dim),
        ):
            if val <= 0:
                raise ValueError(f"{name} must be positive, got {val}")
        if validate not in ("host", "device"):
            raise ValueError(f"validate must be 'host' or 'device', got {validate!r}")
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError(
                f"B200PagedBackend requires a CUDA device, got {self.device}; it has no CPU path"
            )
        if dtype not in N.DTYPE_CODE:
            raise ValueError(f"unsupported pool dtype {dtype}")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self._lib = N.lib()

        self.num_layers = num_layers
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.n_kv_heads = n_kv_heads
        self.n_heads = n_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.groups = n_heads // n_kv_heads
        self.validate = validate

        self._pool = torch.zeros(
            (num_layers, 2, num_blocks, block_size, n_kv_heads, head_dim), dtype=dtype, device=self.device
        )
        self.k_pool: list[torch.Tensor] = [self._pool[l, 0] for l in range(num_layers)]
        self.v_pool: list[torch.Tensor] = [self._pool[l, 1] for l in range(num_layers)]
        self._desc = N.PoolDesc(
            self._pool.data_ptr(), num_blocks, num_layers, block_size, n_kv_heads, head_dim,
            N.DTYPE_CODE[dtype], 0,
        )
        self._pdesc = ctypes.byref(self._desc)
        self._status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._status_ptr = self._status.data_ptr()
        self._dev_index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self._slots_meta: Any = None  # the meta whose int32 slot map is cached in _slots
        self._slots: torch.Tensor | None = None
        self._pos_meta: Any = None  # the meta whose int64 device positions are cached in _pos
        self._pos: torch.Tensor | None = None
        self._ws: torch.Tensor | None = None
        # per-step state, keyed by BatchMeta identity (a strong reference keeps
        # the id from being recycled while it is cached)
        self._meta: Any = None
        self._meta_state: dict[str, Any] = {}
        self.n_plans = 0
        self.n_runs = 0
        self.last_kernel: str | None = None  # "decode" | "prefill" | "generic": kernel of the last attend

    # -- accounting (paged_torch.py:139-177) ----------------------------------

    def zeros_like_pool(self) -> torch.Tensor:
        return torch.zeros(
            (self.num_blocks, self.block_size, self.n_kv_heads, self.head_dim),
            dtype=self.dtype, device=self.device,
        )

    def pool_bytes(self) -> int:
        return self._pool.numel() * self._pool.element_size()

    def block_bytes(self) -> int:
        return self.pool_bytes() // self.num_blocks

    def workspace_bytes(self) -> int:
        return 0 if self._ws is None else self._ws.numel()

    def tokens_capacity(self) -> int:
        return self.num_blocks * self.block_size

    @staticmethod
    def estimate_pool_bytes(num_layers: int, num_blocks: int, block_size: int, n_kv_heads: int,
                            head_dim: int, dtype: torch.dtype = torch.float16) -> int:
        elem = torch.empty((), dtype=dtype).element_size()
        return num_layers * 2 * num_blocks * block_size * n_kv_heads * head_dim * elem

    # -- write path ------------------------------------------------------------

    def copy_block(self, src: int, dst: int) -> None:
        """Duplicate one block, every layer, K and V (copy-on-write;
        ``paged_torch.py:181-207``). ``IndexError`` out of range; no-op if equal."""
        src, dst = int(src), int(dst)
        if not (0 <= src < self.num_blocks and 0 <= dst < self.num_blocks):
            raise IndexError(f"copy_block({src} -> {dst}) outside [0, {self.num_blocks})")
        if src == dst:
            return
        N.check(self._lib.pkv_copy_block(self._pdesc, src, dst, N.stream_ptr(self.device)),
                "copy_block", IndexError)

    def copy_blocks(self, src: Sequence[int] | torch.Tensor, dst: Sequence[int] | torch.Tensor) -> None:
        """Batched ``copy_block``: all pairs, all layers, one launch. The
        destination set must not intersect the source set (a chain a->b->c would
        depend on order); pairs with src == dst are skipped."""
        s = torch.as_tensor(src, dtype=torch.int32).flatten()
        d = torch.as_tensor(dst, dtype=torch.int32).flatten()
        if s.shape != d.shape:
            raise ValueError(f"{s.numel()} sources but {d.numel()} destinations")
        if s.numel() == 0:
            return
        hs, hd = s.cpu(), d.cpu()
        lo = int(torch.minimum(hs.min(), hd.min()))
        hi = int(torch.maximum(hs.max(), hd.max()))
        if lo < 0 or hi >= self.num_blocks:
            raise IndexError(f"copy_blocks ids outside [0, {self.num_blocks})")
        moving = hs != hd
        if bool(torch.isin(hd[moving], hs[moving]).any()):
            raise ValueError("copy_blocks: a destination is also a source; issue the pairs in order")
        if len(set(hd[moving].tolist())) != int(moving.sum()):
            raise ValueError("copy_blocks: duplicate destination block")
        s, d = s.to(self.device), d.to(self.device)
        N.check(self._lib.pkv_copy_blocks(self._pdesc, s.data_ptr(), d.data_ptr(), s.numel(),
                                          self._status.data_ptr(), N.stream_ptr(self.device)),
                "copy_blocks")

    def append_kv(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor, meta: Any) -> None:
        """Scatter this step's K/V into the pool at ``meta.slot_mapping``
        (``paged_torch.py:209-276``). Idempotent."""
        k, v, slots, tokens = self._append_args(layer_idx, k, v, meta)
        if tokens == 0:
            return
        N.check(self._lib.pkv_append_kv(self._pdesc, layer_idx, k.data_ptr(), v.data_ptr(),
                                        slots.data_ptr(), tokens, self._status_ptr,
                                        N.raw_stream(self._dev_index)), "append_kv")

    def append_attend(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor, q: torch.Tensor,
                      scale: float, meta: Any, *, out: torch.Tensor | None = None,
                      rope: tuple[torch.Tensor, torch.Tensor] | None = None) -> torch.Tensor:
        """``append_kv(layer_idx, k, v, meta)`` then ``attend(q, layer_idx, scale,
        meta)`` in one call, with the same checks, errors and results. A decode
        step is ONE kernel launch: the decode kernel writes each sequence's new
        K/V row to its slot and attends over it (no reference counterpart; the
        engine makes the two calls, ``docs/ARCHITECTURE.md:167-172``).

        ``rope=(cos, sin)``: q and k are given before the rotary embedding, which
        is applied at ``meta.positions`` with these fp32 tables
        ``[max_pos, head_dim // 2]`` (see ``rope``); the pool receives the
        rotated K and the result is that of ``rope`` followed by this call, bit
        for bit. For a decode step the rotation happens inside the single
        launch; other steps run ``rope`` first (one launch for q and k)."""
        if rope is not None:
            return self._append_attend_rope(layer_idx, k, v, q, scale, meta, out, rope)
        k, v, slots, tokens = self._append_args(layer_idx, k, v, meta)
        if q.shape != (tokens, self.n_heads, self.head_dim):
            raise ValueError(
                f"q has shape {tuple(q.shape)}, expected ({tokens}, {self.n_heads}, {self.head_dim})"
            )
        st = self._step_state(meta)
        if st["n_tokens"] != tokens:
            raise ValueError(f"meta describes {st['n_tokens']} tokens but q has {tokens}")
        q = self._own(q, self.dtype)
        out = self._out(q, out)
        if tokens == 0:
            return out
        self.n_runs += 1
        self.last_kernel = st["kernel"]
        N.check(self._lib.pkv_append_attend_planned(
            self._pdesc, layer_idx, self.n_heads, k.data_ptr(), v.data_ptr(), slots.data_ptr(), q.data_ptr(),
            out.data_ptr(), float(scale), st["batch_ref"], st["hint"], st["ws_ptr"], st["ws_bytes"],
            N.raw_stream(self._dev_index)), "append_attend")
        return out

    def _append_attend_rope(self, layer_idx, k, v, q, scale, meta, out, rope) -> torch.Tensor:
        cos, sin, pos = self._rope_args(rope, meta)
        k, v, slots, tokens = self._append_args(layer_idx, k, v, meta)
        if pos.shape[0] != tokens:
            raise ValueError(f"meta.positions has {pos.shape[0]} entries but {tokens} tokens were supplied")
        if q.shape != (tokens, self.n_heads, self.head_dim):
            raise ValueError(
                f"q has shape {tuple(q.shape)}, expected ({tokens}, {self.n_heads}, {self.head_dim})"
            )
        st = self._step_state(meta)
        if st["n_tokens"] != tokens:
            raise ValueError(f"meta describes {st['n_tokens']} tokens but q has {tokens}")
        q = self._own(q, self.dtype)
        out = self._out(q, out)
        if tokens == 0:
            return out
        rc = self._lib.pkv_append_attend_rope_planned(
            self._pdesc, layer_idx, self.n_heads, k.data_ptr(), v.data_ptr(), slots.data_ptr(), q.data_ptr(),
            out.data_ptr(), float(scale), st["batch_ref"], st["hint"], st["ws_ptr"], st["ws_bytes"],
            pos.data_ptr(), cos.data_ptr(), sin.data_ptr(), cos.shape[0], N.raw_stream(self._dev_index))
        if rc == N.PKV_ERR_UNSUPPORTED:  # not a single-launch decode step: rotate, then the plain call
            q, k = self.rope(q, k, meta, rope)
            return self.append_attend(layer_idx, k, v, q, scale, meta, out=out)
        N.check(rc, "append_attend")
        self.n_runs += 1
        self.last_kernel = st["kernel"]
        return out

    def rope(self, q: torch.Tensor | None, k: torch.Tensor | None, meta: Any,
             rope: tuple[torch.Tensor, torch.Tensor]) -> tuple[torch.Tensor | None, torch.Tensor | None]:
        """Rotary position embedding of q ``(T, n_heads, head_dim)`` and k
        ``(T, n_kv_heads, head_dim)`` at ``meta.positions``, returned as new
        tensors in the pool dtype (either input may be None). ``rope = (cos,
        sin)``: fp32 tables ``[max_pos, head_dim // 2]`` on this device; pair
        (i, i + head_dim/2) of each head of token t is rotated by
        cos/sin[positions[t], i] — ``a*cos - b*sin, a*sin + b*cos`` with each
        product rounded to fp32, then rounded to the pool dtype, the bits of
        that formula evaluated elementwise in fp32. One kernel launch
        (``pkv_rope``). A position outside the tables raises on the next
        ``check_status`` (and leaves its token unrotated)."""
        cos, sin, pos = self._rope_args(rope, meta)
        T = int(pos.shape[0])
        qo = ko = None
        args = []
        for x, heads, name in ((q, self.n_heads, "q"), (k, self.n_kv_heads, "k")):
            if x is None:
                args.append((None, None, 0))
                continue
            if x.shape != (T, heads, self.head_dim):
                raise ValueError(f"{name} has shape {tuple(x.shape)}, expected ({T}, {heads}, {self.head_dim})")
            x = self._own(x, self.dtype)
            y = torch.empty_like(x)
            args.append((x, y, heads))
        (xq, qo, hq), (xk, ko, hk) = args
        N.check(self._lib.pkv_rope(
            N.DTYPE_CODE[self.dtype], N.ptr(xq), N.ptr(qo), hq, N.ptr(xk), N.ptr(ko), hk, T, self.head_dim,
            pos.data_ptr(), cos.data_ptr(), sin.data_ptr(), cos.shape[0], self._status_ptr,
            N.raw_stream(self._dev_index)), "rope")
        return qo, ko

    def _rope_args(self, rope, meta):
        try:
            cos, sin = rope
        except (TypeError, ValueError):
            raise ValueError("rope must be a (cos, sin) pair of tensors") from None
        half = self.head_dim // 2
        for t, name in ((cos, "cos"), (sin, "sin")):
            if (not isinstance(t, torch.Tensor) or t.dim() != 2 or t.shape[1] != half or t.shape[0] < 1
                    or t.dtype != torch.float32 or not t.is_cuda or t.get_device() != self._dev_index
                    or not t.is_contiguous() or t.data_ptr() % 16):
                raise ValueError(
                    f"rope {name} must be a contiguous 16-byte aligned float32 [max_pos, {half}] tensor on "
                    f"{self.device}")
        if cos.shape != sin.shape:
            raise ValueError(f"rope cos {tuple(cos.shape)} and sin {tuple(sin.shape)} differ in shape")
        if getattr(meta, "positions", None) is None:
            raise ValueError("the rotary embedding needs meta.positions")
        if self._pos_meta is not meta:  # the int64 device positions, once per meta
            self._pos = self._own(meta.positions, torch.int64)
            if self._pos.dim() != 1:
                raise ValueError("meta.positions must be one-dimensional")
            self._pos_meta = meta
        return cos, sin, self._pos

    def _append_args(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor, meta: Any):
        self._check_layer(layer_idx)
        if getattr(meta, "slot_mapping", None) is None:
            raise ValueError(
                "B200PagedBackend.append_kv requires meta.slot_mapping (the flat "
                "per-token physical slot)."
            )
        tokens = k.shape[0]
        if k.shape != (tokens, self.n_kv_heads, self.head_dim):
            raise ValueError(
                f"k has shape {tuple(k.shape)}, expected ({tokens}, {self.n_kv_heads}, {self.head_dim})"
            )
        if v.shape != k.shape:
            raise ValueError(f"v shape {tuple(v.shape)} != k shape {tuple(k.shape)}")
        if meta.slot_mapping.shape[0] != tokens:
            raise ValueError(
                f"slot_mapping has {meta.slot_mapping.shape[0]} entries but {tokens} tokens were supplied"
            )
        k = self._own(k, self.dtype)
        v = self._own(v, self.dtype)
        if not tokens:
            return k, v, None, tokens
        if self._slots_meta is not meta:  # the int32 device slot map, once per meta
            self._slots = self._i32(meta.slot_mapping)
            self._slots_meta = meta
        return k, v, self._slots, tokens

    # -- read path -------------------------------------------------------------

    def attend(self, q: torch.Tensor, layer_idx: int, scale: float, meta: Any, *,
               out: torch.Tensor | None = None) -> torch.Tensor:
        """Attention over each sequence's full KV history including this step's
        append (``paged_torch.py:280-485``): GQA ``h // groups``, bottom-right
        causal mask, pages read in listed order, the unwritten tail of the last
        page never read. Returns ``(tokens, n_heads, head_dim)`` in the pool dtype:
        a new tensor, or ``out`` (an optional extension of the reference's
        signature: a contiguous tensor of that shape and dtype on this device,
        written in place)."""
        self._check_layer(layer_idx)
        tokens = q.shape[0]
        if q.shape != (tokens, self.n_heads, self.head_dim):
            raise ValueError(
                f"q has shape {tuple(q.shape)}, expected ({tokens}, {self.n_heads}, {self.head_dim})"
            )
        st = self._step_state(meta)
        if st["n_tokens"] != tokens:
            raise ValueError(f"meta describes {st['n_tokens']} tokens but q has {tokens}")
        q = self._own(q, self.dtype)
        out = self._out(q, out)
        if tokens == 0:
            return out
        self.n_runs += 1
        self.last_kernel = st["kernel"]
        N.check(self._lib.pkv_attend_planned(
            self._pdesc, layer_idx, self.n_heads, q.data_ptr(), out.data_ptr(), float(scale),
            st["batch_ref"], st["hint"], st["ws_ptr"], st["ws_bytes"],
            N.raw_stream(self._dev_index)), "attend")
        return out

    # -- per-step plan -----------------------------------------------------------

    def plan(self, meta: Any) -> None:
        """Prepare ``meta`` for this step's layers now (validation, device copies
        of the page table, the decode kernel's page schedule). ``attend`` does
        this itself on first sight of a ``meta``; calling it up front keeps that
        work out of the first layer (and inside a captured CUDA graph, if any)."""
        self._step_state(meta)

    def reserve_workspace(self, n_seqs: int, total_pages: int) -> None:
        """Allocate the attention workspace for batches up to this size now, so
        no allocation happens later (e.g. during CUDA-graph capture)."""
        need = int(self._lib.pkv_attend_workspace_size(self._pdesc, self.n_heads, int(n_seqs),
                                                        int(total_pages), 1))
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device=self.device)
            self.invalidate_plan()

    def _step_state(self, meta: Any) -> dict[str, Any]:
        if self._meta is meta:
            return self._meta_state
        n = int(meta.query_lens.shape[0])
        n_tokens = int(meta.positions.shape[0]) if getattr(meta, "positions", None) is not None \
            else int(meta.batch_indices.shape[0])
        total_pages = int(meta.kv_indices.shape[0])
        if n <= 0:
            raise ValueError("BatchMeta has no sequences")
        # hint for the attention entry point: 1 = every query length is 1 (decode
        # kernel), 2 = none is (pure prefill), 0 = unknown / mixed (the q_len == 1
        # rows of a mixed batch run on the decode kernel)
        checked = int(getattr(meta, "checked_blocks", 0) or 0)
        if self.validate == "host" and not (0 < checked <= self.num_blocks
                                            and getattr(meta, "max_query_len", None) is not None):
            decode, hint = self._host_validate(meta, n, total_pages)
        else:
            # device validation, or an assembler that made the host checks already
            # (DeviceBlockTables: lengths, page counts, block ids inside this pool)
            # is_prefill decides decode vs not (a batch mislabelled as decode is
            # refused below); the query-length bounds only sharpen the hint
            mql = getattr(meta, "max_query_len", None)
            mnql = getattr(meta, "min_query_len", None)
            decode = not bool(meta.is_prefill) if hasattr(meta, "is_prefill") else int(mql) == 1
            hint = 1 if decode else (2 if mnql is not None and int(mnql) > 1 else 0)
        if decode and n_tokens != n:
            raise ValueError(
                f"BatchMeta describes a decode step (is_prefill=False) but has {n_tokens} tokens for "
                f"{n} sequences; a decode step has exactly one query per sequence"
            )
        t = {
            "cu": self._i32(meta.cu_query_lens),
            "kl": self._i32(meta.kv_lens) if getattr(meta, "kv_lens", None) is not None else None,
            "ip": self._i32(meta.kv_indptr),
            "ix": self._i32(meta.kv_indices),
            "lp": self._i32(meta.kv_last_page_len),
        }
        batch = N.BatchDesc(
            n, n_tokens, total_pages, t["cu"].data_ptr(), N.ptr(t["kl"]), t["ip"].data_ptr(),
            t["ix"].data_ptr() if total_pages else None, t["lp"].data_ptr(), self._status.data_ptr(),
        )
        need = int(self._lib.pkv_attend_workspace_size(self._pdesc, self.n_heads, n, total_pages, int(decode)))
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device=self.device)
        ws_ptr, ws_bytes = self._ws.data_ptr(), self._ws.numel()
        kernel = int(self._lib.pkv_attend_kernel(self._pdesc, self.n_heads, n, n_tokens, hint))
        if kernel < 0:
            N.check(-kernel, "attend")
        if n_tokens > 0 and (decode or kernel == N.PKV_KERNEL_PREFILL):
            N.check(self._lib.pkv_plan(self._pdesc, self.n_heads, ctypes.byref(batch), ws_ptr, ws_bytes,
                                       N.stream_ptr(self.device)), "plan")
            self.n_plans += 1
        self._meta = meta
        self._meta_state = {"batch": batch, "batch_ref": ctypes.byref(batch), "tensors": t, "decode": decode,
                            "hint": hint, "n_tokens": n_tokens,
                            "ws_ptr": ws_ptr, "ws_bytes": ws_bytes, "kernel": N.KERNEL_NAMES[kernel]}
        return self._meta_state

    def _host_validate(self, meta: Any, n: int, total_pages: int) -> tuple[bool, int]:
        """The reference's page-table checks (``paged_torch.py:379-392``) and
        FlashInfer's ``is_prefill`` cross-check (``flashinfer_backend.py:604-618``),
        once per step. Returns (pure decode step, attention hint: 1 all q_len == 1,
        2 none, 0 mixed)."""
        ql = meta.query_lens.tolist()
        ip = meta.kv_indptr.tolist()
        lp = meta.kv_last_page_len.tolist()
        kl = meta.kv_lens.tolist() if getattr(meta, "kv_lens", None) is not None else None
        P = self.block_size
        if len(ip) != n + 1 or ip[0] != 0 or ip[-1] != total_pages:
            raise ValueError(f"kv_indptr must have {n + 1} entries from 0 to {total_pages}")
        for i in range(n):
            pages = ip[i + 1] - ip[i]
            kv_len = kl[i] if kl is not None else (pages - 1) * P + lp[i]
            need = (kv_len + P - 1) // P
            if pages != need:
                raise ValueError(
                    f"{pages} pages supplied but kv_len={kv_len} with block_size={P} needs {need}"
                )
            tail = kv_len - (pages - 1) * P
            if lp[i] != tail:
                raise ValueError(
                    f"kv_last_page_len={lp[i]} but kv_len={kv_len} over {pages} pages implies "
                    f"{tail}. An exact multiple of block_size must report {P}, not 0."
                )
            if ql[i] > kv_len:
                raise ValueError(f"seq {i}: query_len {ql[i]} exceeds kv_len {kv_len}")
        if total_pages:
            ix = meta.kv_indices
            lo, hi = int(ix.min()), int(ix.max())
            if lo < 0 or hi >= self.num_blocks:
                raise ValueError(f"kv_indices outside [0, {self.num_blocks})")
        use_prefill = any(x > 1 for x in ql)
        if hasattr(meta, "is_prefill") and bool(meta.is_prefill) != use_prefill:
            raise ValueError(
                f"BatchMeta.is_prefill={meta.is_prefill} disagrees with query_lens (max={max(ql)}); "
                "is_prefill must be True iff some sequence contributes more than one token"
            )
        if not use_prefill:
            return True, 1
        return False, (0 if any(x == 1 for x in ql) else 2)

    def invalidate_plan(self) -> None:
        """Forget the cached per-step state (for a caller that mutates a
        BatchMeta's tensors in place and reuses the object)."""
        self._meta = None
        self._meta_state = {}
        self._slots_meta = None
        self._slots = None
        self._pos_meta = None
        self._pos = None

    # -- status -----------------------------------------------------------------

    def check_status(self) -> None:
        """Synchronise and raise if any kernel recorded a violation since the
        last check (out-of-pool ids, inconsistent page tables, q_len != 1 in the
        decode kernel, a timed-out device wait)."""
        bits = int(self._status.item())
        if bits:
            self._status.zero_()
            raise N.PkvError(N.PKV_ERR_DEVICE, f"device status {bits:#x}: {N.describe_status(bits)}")

    # -- misc -----------------------------------------------------------------------

    def _i32(self, t: torch.Tensor) -> torch.Tensor:
        return t.to(device=self.device, dtype=torch.int32).contiguous()

    def _out(self, q: torch.Tensor, out: torch.Tensor | None) -> torch.Tensor:
        if out is None:
            return torch.empty_like(q)
        if (out.shape != q.shape or out.dtype != self.dtype or not out.is_cuda
                or out.get_device() != self._dev_index or not out.is_contiguous()):
            raise ValueError(f"out must be a contiguous {tuple(q.shape)} {self.dtype} tensor on {self.device}")
        nb = q.numel() * q.element_size()
        if out.data_ptr() < q.data_ptr() + nb and q.data_ptr() < out.data_ptr() + nb:
            raise ValueError("out must not overlap q (other CTAs may still read a row being written)")
        return out

    def _own(self, t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
        """t on this device in `dtype`, contiguous (no op when it already is)."""
        if t.is_cuda and t.dtype == dtype and t.get_device() == self._dev_index and t.is_contiguous():
            return t
        return t.to(device=self.device, dtype=dtype).contiguous()

    def _check_layer(self, layer_idx: int) -> None:
        if layer_idx is None or not 0 <= layer_idx < self.num_layers:
            raise ValueError(f"layer_idx {layer_idx} out of range [0, {self.num_layers})")

    def reset(self) -> None:
        """Zero every pool and drop the cached step state. Tests only."""
        self._pool.zero_()
        self.invalidate_plan()

    def __repr__(self) -> str:
        mib = self.pool_bytes() / (1024 * 1024)
        return (
            f"B200PagedBackend(layers={self.num_layers}, blocks={self.num_blocks}, "
            f"block_size={self.block_size}, kv_heads={self.n_kv_heads}, heads={self.n_heads}, "
            f"head_dim={self.head_dim}, dtype={self.dtype}, device={self.device}, pool={mib:.1f} MiB)"
        )
