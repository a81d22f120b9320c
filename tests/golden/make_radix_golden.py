"""
Golden trace of the REFERENCE's block allocator and radix prefix cache
(``serving/memory/allocator.py``, ``serving/cache/radix.py``, with its
``SequenceBlocks`` from ``serving/memory/block_table.py``) under a seeded random
mix of the operations a scheduler performs: admissions that look a prompt up
(``acquire`` + ``attach_prefix``) and allocate the rest, growth, publication
(``insert``), retirement (publish, then free), eviction (``evict``, ``reserve``
with and without the watermark, ``clear``), copy-on-write of a shared last
block (``ensure_writable``) and the invariant checks. Every operation's result
and a digest of the allocator's free list and refcounts, the cache's resident
blocks, node count, depth, shared blocks and statistics are recorded;
``tests/test_radix_cpu.py`` replays the same operations on
``llm_serving_layer_b200.radix`` and requires the same results and digests.

    python tests/golden/make_radix_golden.py /path/to/llm_serving_layer
"""

from __future__ import annotations

import gzip
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
OUT = HERE / "radix_ops.json.gz"


def digest(alloc, cache) -> str:
    st = cache.stats
    state = [list(alloc._free), list(alloc._refcount), sorted(cache._by_block), cache.num_nodes, cache.max_depth,
             cache.shared_blocks, [st.lookups, st.hits, st.blocks_reused, st.blocks_required,
                                   st.partial_block_truncations, st.truncated_tokens, st.inserts, st.evictions,
                                   st.cow_copies, len(st.partial_hit_depths), sum(st.partial_hit_depths)],
             alloc.total_allocated, alloc.total_freed, alloc.peak_used]
    return hashlib.sha1(json.dumps(state, separators=(",", ":")).encode()).hexdigest()[:16]


def run(ref_root: str, seed: int, n_ops: int, num_blocks: int, bs: int, budget):
    sys.path.insert(0, ref_root)
    from serving.cache.radix import RadixCache, attach_prefix
    from serving.memory.allocator import AllocationError, BlockAllocator
    from serving.memory.block_table import SequenceBlocks

    rs = np.random.RandomState(seed)
    alloc = BlockAllocator(num_blocks=num_blocks, block_size=bs, watermark_blocks=2)
    copies = []
    cache = RadixCache(alloc, max_cached_blocks=budget, block_copy=lambda a, b: copies.append((a, b)))
    fams = [[int(x) for x in rs.randint(0, 6, size=int(rs.randint(8, 40)))] for _ in range(6)]
    running, holders, next_id = [], [], 0
    ops = []

    def rec(op, ret, **kw):
        ops.append({"op": op, **kw, "ret": ret, "d": digest(alloc, cache)})

    for _ in range(n_ops):
        u = rs.rand()
        if u < 0.22 or not running:
            f = fams[rs.randint(len(fams))]
            cut = int(rs.randint(1, len(f) + 1))
            tokens = f[:cut] + [int(x) for x in rs.randint(0, 6, size=int(rs.randint(0, 12)))]
            if not tokens:
                tokens = [int(rs.randint(0, 6))]
            seq = SequenceBlocks(alloc, seq_id=next_id)
            next_id += 1
            res = cache.acquire(tokens)
            if res.block_ids:
                attach_prefix(seq, res.block_ids, res.n_tokens)
            need = seq.blocks_needed_for(len(tokens) - res.n_tokens)
            ok_res = cache.reserve(need, watermark=False)
            try:
                seq.append(len(tokens) - res.n_tokens)
                ok = True
            except AllocationError:
                ok = False
            if ok:
                running.append((seq, tokens))
            else:
                seq.free()
            rec("admit", [res.block_ids, res.n_tokens, res.depth, res.blocks_required, res.truncated_partial_block,
                          res.truncated_tokens, ok_res, ok], tokens=list(tokens))
        elif u < 0.42:
            i = int(rs.randint(len(running)))
            seq, tokens = running[i]
            n = int(rs.randint(1, 6))
            extra = [int(x) for x in rs.randint(0, 6, size=n)]
            ok_res = cache.reserve(seq.blocks_needed_for(n), watermark=False)
            try:
                seq.append(n)
                tokens.extend(extra)
                ok = True
            except AllocationError:
                ok = False
            rec("grow", [ok_res, ok], i=i, extra=extra)
        elif u < 0.55:
            i = int(rs.randint(len(running)))
            seq, tokens = running[i]
            rec("publish", cache.insert(tokens[:seq.num_tokens], seq.block_ids), i=i)
        elif u < 0.70:
            i = int(rs.randint(len(running)))
            seq, tokens = running.pop(i)
            n = cache.insert(tokens[:seq.num_tokens], seq.block_ids)
            seq.free()
            rec("retire", n, i=i)
        elif u < 0.77:
            k = int(rs.randint(1, 6))
            rec("evict", cache.evict(k), k=k)
        elif u < 0.84:
            k = int(rs.randint(0, 12))
            wm = bool(rs.rand() < 0.5)
            rec("reserve", cache.reserve(k, watermark=wm), k=k, wm=wm)
        elif u < 0.90:
            cands = [j for j, (s, _) in enumerate(running) if s.num_tokens % bs and s.block_ids]
            if not cands:
                continue
            i = cands[int(rs.randint(len(cands)))]
            seq, _ = running[i]
            last = seq.block_ids[-1]
            alloc.incref([last])
            holders.append(last)
            try:
                new = cache.ensure_writable(seq, len(seq.block_ids) - 1)
                ret = [new, copies[-1] if copies else None]
            except AllocationError:
                ret = ["full"]
            rec("cow", ret, i=i)
        elif u < 0.94 and holders:
            j = int(rs.randint(len(holders)))
            alloc.free([holders.pop(j)])
            rec("unhold", None, j=j)
        elif u < 0.96:
            rec("clear", cache.clear())
        else:
            alloc.check_invariants()
            cache.check_invariants()
            rec("check", None)
    return ops


def main(ref_root: str) -> None:
    runs = [
        {"seed": 1, "n_ops": 1500, "num_blocks": 96, "bs": 4, "budget": None},
        {"seed": 2, "n_ops": 1500, "num_blocks": 64, "bs": 4, "budget": 24},
        {"seed": 3, "n_ops": 800, "num_blocks": 200, "bs": 2, "budget": None},
    ]
    out = []
    for r in runs:
        ops = run(ref_root, **r)
        kinds = {}
        for o in ops:
            kinds[o["op"]] = kinds.get(o["op"], 0) + 1
        print(r, kinds)
        out.append({"params": r, "ops": ops})
    with gzip.open(OUT, "wt") as f:
        json.dump(out, f, separators=(",", ":"))
    print(f"wrote {OUT} ({OUT.stat().st_size / 1e3:.0f} kB)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_radix_golden.py /path/to/reference/checkout")
    main(sys.argv[1])
