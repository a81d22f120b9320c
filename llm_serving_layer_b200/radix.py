"""
Block allocator and radix prefix cache with logarithmic eviction — drop-ins for
the reference's ``serving.memory.allocator.BlockAllocator`` and
``serving.cache.radix.RadixCache`` / ``attach_prefix``: the same constructors,
methods, attributes, statistics, results and exceptions, so the reference's
``Scheduler`` and ``build_default_app`` (serving/server/app.py:1230-1252) take
them unchanged.

What differs is the cost of the two host-side operations that grow with the
pool and the cache:

* ``RadixCache._evict_one`` — the reference scans every resident node for the
  least-recently-accessed leaf that no live sequence holds
  (serving/cache/radix.py:546-572: O(nodes) per evicted block). Here evictable
  leaves sit in a min-heap keyed by their last access, so an eviction costs
  O(log nodes) amortised. The heap is lazy: an entry whose node has since been
  touched, gained a child or left the cache is dropped when it surfaces. When
  the allocator is this module's, it reports every block whose reference count
  falls back to 1 (the cache's own reference), so a leaf some sequence holds is
  dropped from the heap and re-entered when released; with another allocator
  such leaves are set aside and put back after the search. The victim is the
  reference's: the evictable leaf with the smallest last access (distinct
  leaves never share one: a lookup stamps one root-to-leaf path, of which only
  the deepest surviving node can be a leaf).
* ``BlockAllocator.check_invariants`` — the reference walks every block in
  Python (serving/memory/allocator.py:219-245: O(num_blocks)). Here every
  allocate / incref / free keeps the invariant "refcount 0 exactly when on the
  free list" for the blocks it touches (a per-block flag), so
  ``check_invariants(full=False)`` is O(1); the default full check compares
  the refcount table with the free list in numpy.

The trie semantics are the reference's: whole-block keys, a lookup never
returns the whole prompt (one block is recomputed so the request has a token
to run), partially matching blocks are reported and recomputed, publication
takes the cache's own reference on each new block and leaves the existing node
in place on a repeated path, copy-on-write of a sequence's last block only.
"""

from __future__ import annotations

import heapq
import sys
from array import array
from collections import deque
from dataclasses import dataclass, field
from typing import Any, Callable, Iterable, Sequence

import numpy as np

__all__ = ["AllocationError", "BlockAllocator", "RadixNode", "MatchResult", "CacheStats", "RadixCache",
           "attach_prefix"]


class AllocationError(RuntimeError):
    """A request the pool cannot satisfy; nothing is allocated."""


def _alloc_error() -> type[Exception]:
    """The reference's scheduler catches ``serving.memory.allocator.AllocationError``;
    when that module is loaded, raise its class so this allocator is caught there."""
    mod = sys.modules.get("serving.memory.allocator")
    exc = getattr(mod, "AllocationError", None) if mod is not None else None
    return exc if isinstance(exc, type) and issubclass(exc, Exception) else AllocationError


# ---------------------------------------------------------------------------
# allocator
# ---------------------------------------------------------------------------


class BlockAllocator:
    """Fixed pool of physical KV blocks with reference counts and a FIFO free
    list (a freed block is handed out again as late as possible)."""

    def __init__(self, num_blocks: int, block_size: int = 16, watermark_blocks: int = 0):
        if num_blocks <= 0:
            raise ValueError(f"num_blocks must be positive, got {num_blocks}")
        if block_size <= 0:
            raise ValueError(f"block_size must be positive, got {block_size}")
        if not 0 <= watermark_blocks < num_blocks:
            raise ValueError(f"watermark_blocks must lie in [0, {num_blocks}), got {watermark_blocks}")
        self._num_blocks = num_blocks
        self._block_size = block_size
        self._watermark = watermark_blocks
        self._free: deque[int] = deque(range(num_blocks))
        self._refcount = array("i", bytes(4 * num_blocks))  # int32 counts, viewed by numpy without a copy
        self._on_free = bytearray(b"\x01") * num_blocks  # per-block: currently on the free list
        self._listeners: list[Callable[[int], None]] = []
        self._returned_by_reset = 0
        self.total_allocated = 0
        self.total_freed = 0
        self.peak_used = 0

    # -- introspection --------------------------------------------------------
    @property
    def num_blocks(self) -> int:
        return self._num_blocks

    @property
    def block_size(self) -> int:
        return self._block_size

    @property
    def watermark_blocks(self) -> int:
        return self._watermark

    @property
    def num_free(self) -> int:
        return len(self._free)

    @property
    def num_used(self) -> int:
        return self._num_blocks - len(self._free)

    @property
    def utilization(self) -> float:
        return self.num_used / self._num_blocks

    def refcount(self, block_id: int) -> int:
        self._check_id(block_id)
        return self._refcount[block_id]

    def tokens_capacity(self) -> int:
        return self._num_blocks * self._block_size

    # -- allocation -----------------------------------------------------------
    def can_allocate(self, n_blocks: int) -> bool:
        """May admission take ``n_blocks`` and still leave the watermark free?"""
        if n_blocks < 0:
            raise ValueError(f"n_blocks must be non-negative, got {n_blocks}")
        return len(self._free) - n_blocks >= self._watermark

    def allocate(self, n_blocks: int) -> list[int]:
        """``n_blocks`` blocks from the head of the free list, refcount 1 each;
        all or nothing."""
        if n_blocks < 0:
            raise ValueError(f"n_blocks must be non-negative, got {n_blocks}")
        if n_blocks == 0:
            return []
        if n_blocks > len(self._free):
            raise _alloc_error()(
                f"Cannot allocate {n_blocks} blocks: only {len(self._free)} free of {self._num_blocks} "
                f"(watermark {self._watermark}); preemption should have made room first.")
        rc, on_free, pop = self._refcount, self._on_free, self._free.popleft
        out = [pop() for _ in range(n_blocks)]
        for b in out:
            if rc[b] != 0 or not on_free[b]:
                raise AssertionError(f"Block {b} came off the free list with refcount {rc[b]}: "
                                     "allocator state is corrupt.")
            rc[b] = 1
            on_free[b] = 0
        self.total_allocated += n_blocks
        used = self._num_blocks - len(self._free)
        if used > self.peak_used:
            self.peak_used = used
        return out

    # -- reference counting ----------------------------------------------------
    def incref(self, block_ids: Iterable[int]) -> None:
        """One more holder of each block (prefix reuse); a free block cannot be claimed."""
        rc = self._refcount
        for b in block_ids:
            self._check_id(b)
            if rc[b] == 0:
                raise _alloc_error()(f"Cannot incref block {b}: refcount is 0 (it is free and its "
                                     "contents are not guaranteed); allocate it instead.")
            rc[b] += 1

    def free(self, block_ids: Sequence[int]) -> None:
        """Drop one reference per id; a block rejoins the tail of the free list
        when its count reaches 0. A double free raises."""
        rc, on_free = self._refcount, self._on_free
        for b in block_ids:
            self._check_id(b)
            c = rc[b]
            if c == 0:
                raise _alloc_error()(f"Double free of block {b}: refcount is already 0, so another "
                                     "holder's block would be handed out.")
            c -= 1
            rc[b] = c
            if c == 0:
                if on_free[b]:
                    raise AssertionError(f"Block {b} reached refcount 0 while already on the free list")
                on_free[b] = 1
                self._free.append(b)
                self.total_freed += 1
            elif c == 1 and self._listeners:
                for fn in self._listeners:
                    fn(b)

    def add_release_listener(self, fn: Callable[[int], None]) -> None:
        """``fn(block)`` is called whenever a free leaves a block with exactly one
        reference (how the radix cache learns a cached block became evictable)."""
        self._listeners.append(fn)

    # -- integrity --------------------------------------------------------------
    def check_invariants(self, full: bool = True) -> None:
        """Refcount 0 exactly for the blocks on the free list, each once, no
        negative count. ``full=False``: the O(1) check of the counters the
        operations maintain (each operation already checks the blocks it
        touches); ``full=True`` (default): the whole table against the free list,
        vectorised."""
        if not full:
            # every block starts free; each allocation takes one off, each last free puts one back
            if self.total_allocated - self.total_freed - self._returned_by_reset != self.num_used:
                raise AssertionError(f"{self.total_allocated} blocks allocated and {self.total_freed} returned, "
                                     f"but {self.num_used} in use — the free list and the counts diverged")
            return
        rc = (np.frombuffer(self._refcount, dtype=np.int32) if isinstance(self._refcount, array)
              else np.asarray(self._refcount, dtype=np.int64))
        fl = np.fromiter(self._free, dtype=np.int64, count=len(self._free))
        if fl.size and (fl.min() < 0 or fl.max() >= self._num_blocks):
            raise AssertionError("Free list holds an id outside the pool")
        cnt = np.bincount(fl, minlength=self._num_blocks)
        dup = np.nonzero(cnt > 1)[0]
        if dup.size:
            raise AssertionError(f"Free list contains duplicates: {dup.tolist()[:16]}")
        neg = np.nonzero(rc < 0)[0]
        if neg.size:
            raise AssertionError(f"Block {int(neg[0])} has negative refcount {int(rc[neg[0]])}")
        leaked = np.nonzero((rc == 0) & (cnt == 0))[0]
        if leaked.size:
            raise AssertionError(f"Block {int(leaked[0])} has refcount 0 but is not on the free list — leaked")
        live = np.nonzero((rc > 0) & (cnt > 0))[0]
        if live.size:
            b = int(live[0])
            raise AssertionError(f"Block {b} has refcount {int(rc[b])} but IS on the free list — it is "
                                 "about to be handed to a second owner")

    def reset(self) -> None:
        """Every block back to the pool. Tests only."""
        self._returned_by_reset += self.num_used
        self._free = deque(range(self._num_blocks))
        self._refcount = array("i", bytes(4 * self._num_blocks))
        self._on_free = bytearray(b"\x01") * self._num_blocks

    def _check_id(self, block_id: int) -> None:
        if not 0 <= block_id < self._num_blocks:
            raise ValueError(f"Block id {block_id} out of range [0, {self._num_blocks})")

    def __repr__(self) -> str:
        return (f"BlockAllocator(num_blocks={self._num_blocks}, block_size={self._block_size}, "
                f"free={self.num_free}, used={self.num_used}, watermark={self._watermark})")


# ---------------------------------------------------------------------------
# radix cache
# ---------------------------------------------------------------------------


class RadixNode:
    """One block of tokens under its prefix: the physical block holding their KV.
    Hashes by identity (equal keys under different prefixes are different KV)."""

    __slots__ = ("key", "block_id", "parent", "children", "last_access", "depth", "resident")

    def __init__(self, key: tuple = (), block_id: int = -1, parent: "RadixNode | None" = None,
                 last_access: int = 0, depth: int = 0):
        self.key = key
        self.block_id = block_id
        self.parent = parent
        self.children: dict[tuple, RadixNode] = {}
        self.last_access = last_access
        self.depth = depth
        self.resident = True

    @property
    def is_leaf(self) -> bool:
        return not self.children

    def __repr__(self) -> str:  # pragma: no cover - diagnostics
        return (f"RadixNode(depth={self.depth}, block={self.block_id}, children={len(self.children)}, "
                f"last_access={self.last_access})")


@dataclass
class MatchResult:
    """One prefix walk: the reusable whole blocks and what the walk saw."""

    block_ids: list[int] = field(default_factory=list)
    n_tokens: int = 0
    depth: int = 0
    blocks_required: int = 0
    truncated_partial_block: bool = False
    truncated_tokens: int = 0

    @property
    def hit(self) -> bool:
        return bool(self.block_ids)

    @property
    def hit_rate(self) -> float:
        return (len(self.block_ids) / self.blocks_required) if self.blocks_required else 0.0


@dataclass
class CacheStats:
    lookups: int = 0
    hits: int = 0
    blocks_reused: int = 0
    blocks_required: int = 0
    partial_block_truncations: int = 0
    truncated_tokens: int = 0
    inserts: int = 0
    evictions: int = 0
    cow_copies: int = 0
    partial_hit_depths: list[int] = field(default_factory=list)

    @property
    def hit_rate(self) -> float:
        return (self.blocks_reused / self.blocks_required) if self.blocks_required else 0.0

    @property
    def request_hit_rate(self) -> float:
        return (self.hits / self.lookups) if self.lookups else 0.0

    @property
    def mean_partial_hit_depth(self) -> float:
        d = self.partial_hit_depths
        return (sum(d) / len(d)) if d else 0.0


class RadixCache:
    """Block-granular token trie over a ``BlockAllocator``; LRU eviction of
    leaves no live sequence holds, in O(log nodes) per block."""

    def __init__(self, allocator: Any, *, max_cached_blocks: int | None = None,
                 block_copy: Callable[[int, int], None] | None = None, enabled: bool = True):
        self.allocator = allocator
        self.block_size = allocator.block_size
        self.enabled = enabled
        self.max_cached_blocks = max_cached_blocks
        self._block_copy = block_copy
        self.root = RadixNode()
        self._nodes: set[RadixNode] = set()
        self._by_block: dict[int, RadixNode] = {}
        self._clock = 0
        self._heap: list[tuple[int, int, RadixNode]] = []
        self._seq = 0
        self.stats = CacheStats()
        hook = getattr(allocator, "add_release_listener", None)
        self._notified = callable(hook)
        if self._notified:
            hook(self._on_release)

    # -- bookkeeping ------------------------------------------------------------
    def _tick(self) -> int:
        self._clock += 1
        return self._clock

    def _push(self, node: RadixNode) -> None:
        self._seq += 1
        heapq.heappush(self._heap, (node.last_access, self._seq, node))

    def _on_release(self, block: int) -> None:
        node = self._by_block.get(block)
        if node is not None and not node.children:
            self._push(node)

    def _users(self, node: RadixNode) -> int:
        """Live sequences holding the node's block (the cache holds one reference)."""
        return self.allocator.refcount(node.block_id) - 1

    # -- introspection ------------------------------------------------------------
    @property
    def num_nodes(self) -> int:
        return len(self._nodes)

    @property
    def cached_blocks(self) -> int:
        return len(self._by_block)

    @property
    def max_depth(self) -> int:
        return max((n.depth for n in self._nodes), default=0)

    @property
    def shared_blocks(self) -> int:
        return sum(1 for b in self._by_block if self.allocator.refcount(b) > 1)

    # -- lookup -------------------------------------------------------------------
    def _keys(self, token_ids: Sequence[int]) -> list[tuple]:
        bs = self.block_size
        return [tuple(token_ids[i * bs:(i + 1) * bs]) for i in range(len(token_ids) // bs)]

    def match(self, token_ids: Sequence[int]) -> MatchResult:
        """The reusable whole blocks of ``token_ids``; changes nothing."""
        bs = self.block_size
        res = MatchResult(blocks_required=(len(token_ids) + bs - 1) // bs)
        if not self.enabled or not token_ids:
            return res
        keys = self._keys(token_ids)
        node, path = self.root, []
        for k in keys:
            nxt = node.children.get(k)
            if nxt is None:
                break
            path.append(nxt)
            node = nxt
        if len(path) < len(keys):
            # the walk stopped inside a block: how far do the offered siblings agree?
            miss = keys[len(path)]
            best = 0
            for sib in node.children:
                n = 0
                while n < bs and sib[n] == miss[n]:
                    n += 1
                best = max(best, n)
            if best:
                res.truncated_partial_block = True
                res.truncated_tokens = best
        # at least one token must be left to compute: never the whole prompt
        while path and len(path) * bs >= len(token_ids):
            path.pop()
        res.block_ids = [n.block_id for n in path]
        res.depth = len(path)
        res.n_tokens = len(path) * bs
        return res

    def acquire(self, token_ids: Sequence[int]) -> MatchResult:
        """``match`` plus a reference on each matched block and a fresh access stamp."""
        res = self.match(token_ids)
        st = self.stats
        st.lookups += 1
        st.blocks_required += res.blocks_required
        if res.truncated_partial_block:
            st.partial_block_truncations += 1
            st.truncated_tokens += res.truncated_tokens
        if not res.block_ids:
            st.partial_hit_depths.append(0)
            return res
        self.allocator.incref(res.block_ids)
        now = self._tick()
        for b in res.block_ids:
            self._by_block[b].last_access = now
        if not self._notified:
            # entries of the touched path are stale now; the deepest matched node may
            # be a leaf that becomes evictable again when released
            leaf = self._by_block[res.block_ids[-1]]
            if not leaf.children:
                self._push(leaf)
        st.hits += 1
        st.blocks_reused += len(res.block_ids)
        st.partial_hit_depths.append(res.depth)
        return res

    # -- publication ----------------------------------------------------------------
    def insert(self, token_ids: Sequence[int], block_ids: Sequence[int]) -> int:
        """Publish the whole blocks of ``token_ids`` held in ``block_ids``; returns
        how many nodes were created. An existing node on the path is kept (and
        touched); a block already cached elsewhere, or free, stops the walk."""
        if not self.enabled:
            return 0
        bs = self.block_size
        n = min(len(token_ids) // bs, len(block_ids))
        node, created = self.root, 0
        for i in range(n):
            key = tuple(token_ids[i * bs:(i + 1) * bs])
            nxt = node.children.get(key)
            if nxt is not None:
                nxt.last_access = self._tick()
                if not nxt.children:
                    self._push(nxt)
                node = nxt
                continue
            b = int(block_ids[i])
            if b in self._by_block:
                break
            try:
                self.allocator.incref([b])
            except Exception as e:  # the allocator's AllocationError: a free block is not published
                if type(e).__name__ != "AllocationError":
                    raise
                break
            child = RadixNode(key, b, node, self._tick(), node.depth + 1)
            node.children[key] = child
            self._nodes.add(child)
            self._by_block[b] = child
            self._push(child)
            created += 1
            node = child
        self.stats.inserts += created
        self._enforce_budget()
        return created

    # -- eviction ---------------------------------------------------------------------
    def _remove(self, node: RadixNode) -> None:
        if node.children:
            raise AssertionError(f"attempted to evict internal node at depth {node.depth} with "
                                 f"{len(node.children)} children")
        if self._users(node) != 0:
            raise AssertionError(f"attempted to evict block {node.block_id} with {self._users(node)} live users")
        parent = node.parent
        if parent is not None:
            parent.children.pop(node.key, None)
        node.resident = False
        self._nodes.discard(node)
        self._by_block.pop(node.block_id, None)
        self.allocator.free([node.block_id])
        self.stats.evictions += 1
        if parent is not None and parent is not self.root and not parent.children:
            self._push(parent)  # the parent is a leaf now

    def _evict_one(self) -> bool:
        """Evict the least-recently-accessed leaf no live sequence holds; False
        when there is none."""
        heap, held = self._heap, []
        victim = None
        while heap:
            stamp, _, node = heap[0]
            if not node.resident or node.children or stamp != node.last_access:
                heapq.heappop(heap)  # stale: touched, grew a child, or gone
                continue
            if self._users(node) > 0:
                heapq.heappop(heap)
                if not self._notified:
                    held.append((stamp, node))  # evictable again once released: keep it
                continue
            victim = node
            heapq.heappop(heap)
            break
        for stamp, node in held:
            self._seq += 1
            heapq.heappush(heap, (stamp, self._seq, node))
        if victim is None:
            return False
        self._remove(victim)
        return True

    def evict(self, n_blocks: int) -> int:
        if n_blocks <= 0:
            return 0
        freed = 0
        while freed < n_blocks and self._evict_one():
            freed += 1
        return freed

    def reserve(self, n_blocks: int, *, watermark: bool = True) -> bool:
        """Evict unused cached blocks until ``n_blocks`` can be allocated
        (admission's watermark rule when ``watermark``)."""
        a = self.allocator

        def ok() -> bool:
            return a.can_allocate(n_blocks) if watermark else a.num_free >= n_blocks

        while not ok():
            if not self._evict_one():
                return False
        return True

    def _enforce_budget(self) -> None:
        if self.max_cached_blocks is None:
            return
        while self.cached_blocks > self.max_cached_blocks:
            if not self._evict_one():
                break

    def clear(self) -> int:
        freed = 0
        while self._evict_one():
            freed += 1
        return freed

    # -- copy-on-write ------------------------------------------------------------------
    def ensure_writable(self, seq: Any, block_index: int) -> int:
        """The block to write at ``block_index`` (the sequence's last): the same
        block for its sole owner, else a fresh copy made through ``block_copy``."""
        if not 0 <= block_index < len(seq.block_ids):
            raise IndexError(f"block_index {block_index} outside sequence's {len(seq.block_ids)} blocks")
        if block_index != len(seq.block_ids) - 1:
            raise ValueError(
                f"copy-on-write requested for block {block_index} of {len(seq.block_ids)}, which is not "
                "the sequence's last block; only the last, partially filled block of a shared prefix "
                "is ever written.")
        old = seq.block_ids[block_index]
        if self.allocator.refcount(old) == 1:
            return old
        if self._block_copy is None:
            raise RuntimeError(
                f"block {old} needs copy-on-write (refcount {self.allocator.refcount(old)}) but no "
                "block_copy callable was supplied; repointing without a copy would leave the prefix unwritten.")
        new = self.allocator.allocate(1)[0]
        self._block_copy(old, new)
        self.allocator.free([old])
        seq.block_ids[block_index] = new
        self.stats.cow_copies += 1
        return new

    # -- reporting -------------------------------------------------------------------------
    def snapshot(self) -> dict[str, Any]:
        st = self.stats
        return {
            "enabled": self.enabled,
            "block_size": self.block_size,
            "lookups": st.lookups,
            "requests_with_a_hit": st.hits,
            "request_hit_rate": st.request_hit_rate,
            "blocks_reused": st.blocks_reused,
            "blocks_required": st.blocks_required,
            "block_hit_rate": st.hit_rate,
            "mean_partial_hit_depth": st.mean_partial_hit_depth,
            "max_partial_hit_depth": max(st.partial_hit_depths, default=0),
            "partial_block_truncations": st.partial_block_truncations,
            "tokens_matched_but_recomputed": st.truncated_tokens,
            "inserts": st.inserts,
            "evictions": st.evictions,
            "cow_copies": st.cow_copies,
            "node_count": self.num_nodes,
            "max_node_depth": self.max_depth,
            "cached_blocks": self.cached_blocks,
            "shared_blocks_refcount_gt_1": self.shared_blocks,
            "definitions": {
                "block_hit_rate": "blocks_reused / blocks_required at prefill",
                "partial_hit_depth": "blocks matched before divergence, per request",
                "shared_blocks_refcount_gt_1": "cached blocks also held by at least one live sequence",
            },
        }

    def check_invariants(self) -> None:
        """Every resident node reachable from its resident parent, one block per
        edge, depth = parent depth + 1, its block referenced and mapped 1:1."""
        for node in self._nodes:
            p = node.parent
            if p is None:
                raise AssertionError(f"node at depth {node.depth} has no parent")
            if p.children.get(node.key) is not node:
                raise AssertionError(f"node at depth {node.depth} is not reachable from its parent")
            if p is not self.root and p not in self._nodes:
                raise AssertionError("node's parent is not resident")
            if node.depth != p.depth + 1:
                raise AssertionError("depth is not parent.depth + 1")
            if len(node.key) != self.block_size:
                raise AssertionError(f"node key spans {len(node.key)} tokens, not one block ({self.block_size})")
            if self.allocator.refcount(node.block_id) < 1:
                raise AssertionError(f"cached block {node.block_id} has lost the cache's reference")
            if self._by_block.get(node.block_id) is not node:
                raise AssertionError(f"block {node.block_id} is not mapped 1:1 to its node")
        if len(self._by_block) != len(self._nodes):
            raise AssertionError(f"{len(self._by_block)} blocks mapped but {len(self._nodes)} nodes resident")


def attach_prefix(seq: Any, block_ids: Sequence[int], n_tokens: int) -> None:
    """Put acquired cached blocks (whose references ``seq`` now owns) at the
    front of an empty sequence's table."""
    if seq.is_freed:
        raise RuntimeError("cannot attach a cached prefix to a freed sequence")
    if seq.block_ids or seq.num_tokens:
        raise ValueError(f"sequence {seq.seq_id} already holds {len(seq.block_ids)} blocks / {seq.num_tokens} "
                         "tokens; a cached prefix is attached before anything is allocated")
    if n_tokens != len(block_ids) * seq.block_size:
        raise ValueError(f"cached prefix claims {n_tokens} tokens over {len(block_ids)} blocks of "
                         f"{seq.block_size}; reuse is only ever a WHOLE number of blocks")
    seq.block_ids.extend(block_ids)
    seq.num_tokens = n_tokens
