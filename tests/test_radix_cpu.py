"""
``llm_serving_layer_b200.radix`` — the block allocator and radix prefix cache
with logarithmic eviction — against the reference's own ``BlockAllocator`` /
``RadixCache`` (serving/memory/allocator.py, serving/cache/radix.py).

* Golden replay: ``tests/golden/radix_ops.json.gz`` holds ~3800 operations a
  scheduler performs (admissions with prefix lookups, growth, publication,
  retirement, eviction, reserve with and without the watermark, clear,
  copy-on-write, invariant checks), run on the reference's classes by
  ``tests/golden/make_radix_golden.py`` with every result and a digest of the
  allocator's free list and refcounts and the cache's resident blocks, shape and
  statistics after each. The same operations on this module must give the same
  results and digests — the same victims in the same order, the same free-list
  order, the same statistics.
* Behaviour the reference's tests pin (restated): LRU leaf-first eviction that
  never takes a block a live sequence holds, parents becoming evictable after
  their children, the last-token rule, partial-block truncation statistics,
  copy-on-write rules and errors, attach_prefix errors, allocator errors and the
  three corruptions ``check_invariants`` must catch.
* Cost: evicting every block of a 20 000-node cache takes far less time than the
  reference's scan would (bounded work per eviction).
"""

from __future__ import annotations

import gzip
import hashlib
import json
import time
from pathlib import Path

import pytest

from llm_serving_layer_b200.radix import AllocationError, BlockAllocator, RadixCache, attach_prefix

GOLD = Path(__file__).resolve().parent / "golden" / "radix_ops.json.gz"


class Seq:
    """The two SequenceBlocks operations the trace uses (serving/memory/block_table.py:
    append allocates ceil(total / block_size) - held blocks, free releases them all)."""

    def __init__(self, alloc, seq_id=0):
        self.alloc, self.seq_id, self.block_size = alloc, seq_id, alloc.block_size
        self.block_ids, self.num_tokens, self.is_freed = [], 0, False

    def blocks_needed_for(self, n):
        return max(0, (self.num_tokens + n + self.block_size - 1) // self.block_size - len(self.block_ids))

    def append(self, n):
        if n == 0:
            return
        need = self.blocks_needed_for(n)
        if need:
            self.block_ids.extend(self.alloc.allocate(need))
        self.num_tokens += n

    def free(self):
        if self.is_freed:
            return
        if self.block_ids:
            self.alloc.free(self.block_ids)
        self.block_ids, self.num_tokens, self.is_freed = [], 0, True


def digest(alloc, cache) -> str:
    st = cache.stats
    state = [list(alloc._free), list(alloc._refcount), sorted(cache._by_block), cache.num_nodes, cache.max_depth,
             cache.shared_blocks, [st.lookups, st.hits, st.blocks_reused, st.blocks_required,
                                   st.partial_block_truncations, st.truncated_tokens, st.inserts, st.evictions,
                                   st.cow_copies, len(st.partial_hit_depths), sum(st.partial_hit_depths)],
             alloc.total_allocated, alloc.total_freed, alloc.peak_used]
    return hashlib.sha1(json.dumps(state, separators=(",", ":")).encode()).hexdigest()[:16]


class UnhookedAllocator(BlockAllocator):
    """An allocator that does not report releases (as the reference's does not):
    the cache then keeps held leaves aside during a search instead."""

    add_release_listener = None


def replay(params, ops, alloc_cls=BlockAllocator):
    alloc = alloc_cls(num_blocks=params["num_blocks"], block_size=params["bs"], watermark_blocks=2)
    copies = []
    cache = RadixCache(alloc, max_cached_blocks=params["budget"], block_copy=lambda a, b: copies.append((a, b)))
    running, holders, next_id = [], [], 0
    for n, o in enumerate(ops):
        op = o["op"]
        if op == "admit":
            tokens = o["tokens"]
            seq = Seq(alloc, next_id)
            next_id += 1
            res = cache.acquire(tokens)
            if res.block_ids:
                attach_prefix(seq, res.block_ids, res.n_tokens)
            ok_res = cache.reserve(seq.blocks_needed_for(len(tokens) - res.n_tokens), watermark=False)
            try:
                seq.append(len(tokens) - res.n_tokens)
                ok = True
            except AllocationError:
                ok = False
            if ok:
                running.append((seq, list(tokens)))
            else:
                seq.free()
            ret = [res.block_ids, res.n_tokens, res.depth, res.blocks_required, res.truncated_partial_block,
                   res.truncated_tokens, ok_res, ok]
        elif op == "grow":
            seq, tokens = running[o["i"]]
            extra = o["extra"]
            ok_res = cache.reserve(seq.blocks_needed_for(len(extra)), watermark=False)
            try:
                seq.append(len(extra))
                tokens.extend(extra)
                ok = True
            except AllocationError:
                ok = False
            ret = [ok_res, ok]
        elif op == "publish":
            seq, tokens = running[o["i"]]
            ret = cache.insert(tokens[:seq.num_tokens], seq.block_ids)
        elif op == "retire":
            seq, tokens = running.pop(o["i"])
            ret = cache.insert(tokens[:seq.num_tokens], seq.block_ids)
            seq.free()
        elif op == "evict":
            ret = cache.evict(o["k"])
        elif op == "reserve":
            ret = cache.reserve(o["k"], watermark=o["wm"])
        elif op == "cow":
            seq, _ = running[o["i"]]
            last = seq.block_ids[-1]
            alloc.incref([last])
            holders.append(last)
            try:
                new = cache.ensure_writable(seq, len(seq.block_ids) - 1)
                ret = [new, list(copies[-1]) if copies else None]
            except AllocationError:
                ret = ["full"]
        elif op == "unhold":
            alloc.free([holders.pop(o["j"])])
            ret = None
        elif op == "clear":
            ret = cache.clear()
        else:
            alloc.check_invariants()
            alloc.check_invariants(full=False)
            cache.check_invariants()
            ret = None
        want = o["ret"]
        assert json.loads(json.dumps(ret)) == want, f"op {n} ({op}): got {ret}, reference {want}"
        assert digest(alloc, cache) == o["d"], f"op {n} ({op}): state differs from the reference's"


@pytest.mark.parametrize("alloc_cls", [BlockAllocator, UnhookedAllocator])
def test_replays_the_reference_allocator_and_radix_trace(alloc_cls):
    with gzip.open(GOLD, "rt") as f:
        runs = json.load(f)
    assert len(runs) == 3 and sum(len(r["ops"]) for r in runs) > 3700
    kinds = set()
    for r in runs:
        replay(r["params"], r["ops"], alloc_cls)
        kinds |= {o["op"] for o in r["ops"]}
    assert kinds == {"admit", "grow", "publish", "retire", "evict", "reserve", "cow", "unhold", "clear", "check"}


def _cache(num_blocks=64, bs=4, **kw):
    alloc = BlockAllocator(num_blocks=num_blocks, block_size=bs)
    return alloc, RadixCache(alloc, **kw)


def _published(alloc, cache, tokens):
    s = Seq(alloc)
    s.append(len(tokens))
    cache.insert(tokens, s.block_ids)
    return s


def test_eviction_is_lru_among_leaves_no_sequence_holds():
    alloc, cache = _cache()
    a = _published(alloc, cache, list(range(12)))          # 3 blocks, chain
    b = _published(alloc, cache, [50 + t for t in range(8)])  # 2 blocks, another chain
    a.free()
    b.free()
    cache.acquire(list(range(12)) + [99])                   # touches all of a's path (and holds it)
    held = cache.acquire(list(range(12)) + [98])
    assert cache.evict(1) == 1                              # b's leaf: a's chain is held
    assert cache.cached_blocks == 4
    assert all(alloc.refcount(x) > 1 for x in held.block_ids)
    assert cache.evict(10) == 1                             # b's root block became a leaf; a's chain stays
    assert cache.cached_blocks == 3 and cache.num_nodes == 3
    cache.check_invariants()
    alloc.check_invariants()


def test_parent_becomes_evictable_after_its_child_and_clear_empties_the_cache():
    alloc, cache = _cache()
    s = _published(alloc, cache, list(range(16)))
    s.free()
    assert cache.num_nodes == 4 and cache.max_depth == 4
    assert cache.clear() == 4
    assert cache.num_nodes == 0 and alloc.num_free == alloc.num_blocks
    alloc.check_invariants()


def test_lookup_never_returns_the_whole_prompt_and_reports_partial_blocks():
    alloc, cache = _cache()
    _published(alloc, cache, list(range(8)))
    r = cache.match(list(range(8)))
    assert r.n_tokens == 4 and r.depth == 1                 # one block left to compute
    r = cache.match([0, 1, 2, 3, 4, 5, 7, 7, 9])
    assert r.n_tokens == 4 and r.truncated_partial_block and r.truncated_tokens == 2
    assert cache.match([]).n_tokens == 0


def test_copy_on_write_rules():
    alloc = BlockAllocator(num_blocks=32, block_size=4)
    copies = []
    cache = RadixCache(alloc, block_copy=lambda a, b: copies.append((a, b)))
    s = Seq(alloc)
    s.append(6)
    assert cache.ensure_writable(s, 1) == s.block_ids[1] and not copies  # sole owner
    with pytest.raises(ValueError, match="not the sequence's last block"):
        cache.ensure_writable(s, 0)
    old = s.block_ids[1]
    alloc.incref([old])
    new = cache.ensure_writable(s, 1)
    assert new != old and copies == [(old, new)] and alloc.refcount(old) == 1 and cache.stats.cow_copies == 1
    nocopy = RadixCache(alloc)
    alloc.incref([new])
    with pytest.raises(RuntimeError, match="copy-on-write"):
        nocopy.ensure_writable(s, 1)


def test_attach_prefix_errors():
    alloc = BlockAllocator(num_blocks=8, block_size=4)
    s = Seq(alloc)
    with pytest.raises(ValueError, match="WHOLE number of blocks"):
        attach_prefix(s, [1], 3)
    s.append(2)
    with pytest.raises(ValueError, match="already holds"):
        attach_prefix(s, [1], 4)


def test_allocator_errors_and_corruptions():
    with pytest.raises(ValueError):
        BlockAllocator(num_blocks=0)
    with pytest.raises(ValueError):
        BlockAllocator(num_blocks=4, watermark_blocks=4)
    a = BlockAllocator(num_blocks=4, block_size=4)
    with pytest.raises(ValueError, match="non-negative"):
        a.allocate(-1)
    with pytest.raises(AllocationError, match="Cannot allocate"):
        a.allocate(5)
    (b,) = a.allocate(1)
    a.free([b])
    with pytest.raises(AllocationError, match="Double free"):
        a.free([b])
    with pytest.raises(AllocationError, match="refcount is 0"):
        a.incref([b])
    with pytest.raises(ValueError, match="out of range"):
        a.refcount(4)
    for corrupt, needle in ((lambda x, y: x._free.append(y), "second owner"),
                            (lambda x, y: x._refcount.__setitem__(y, 0), "leaked")):
        x = BlockAllocator(num_blocks=4, block_size=4)
        (y,) = x.allocate(1)
        corrupt(x, y)
        with pytest.raises(AssertionError, match=needle):
            x.check_invariants()
    x = BlockAllocator(num_blocks=4, block_size=4)
    x._free.append(2)
    with pytest.raises(AssertionError, match="duplicate"):
        x.check_invariants()


def test_eviction_work_is_bounded_per_block():
    """Evicting all blocks of a 20 000-leaf cache, one at a time, stays far below
    the reference's O(nodes) scan per eviction (~2e8 node visits here)."""
    n = 20000
    alloc = BlockAllocator(num_blocks=n + 16, block_size=1)
    cache = RadixCache(alloc)
    for i in range(n):
        s = Seq(alloc)
        s.append(1)
        cache.insert([i], s.block_ids)
        s.free()
    t0 = time.perf_counter()
    assert cache.evict(n) == n
    dt = time.perf_counter() - t0
    assert cache.num_nodes == 0 and alloc.num_free == alloc.num_blocks
    assert dt < 5.0, f"evicting {n} blocks took {dt:.2f} s"
