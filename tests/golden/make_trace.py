"""
Record a trace of the REFERENCE's own serving stack driving its paged backend:
the unmodified ``Scheduler`` (serving/scheduler/scheduler.py) with a
``RadixCache`` whose ``block_copy`` is the backend's ``copy_block`` (as
``build_default_app`` wires it, serving/server/app.py:1245-1252), SWAP
preemption through ``KVSwapSpace`` (serving/scheduler/preemption.py), and
``PagedTorchBackend`` (serving/backends/paged_torch.py) on CPU tensors, in fp16,
at Llama-3.2-1B's attention geometry (32 query heads, 8 KV heads, head_dim 64,
16-token blocks), 2 layers.

The model is a ``forward_varlen`` in the pattern of the reference's own
``TinyPagedModel`` (tests/test_preemption.py:105-147): embed, per layer project
Q/K/V, rotate q and k at ``meta.positions``, ``append_kv``, ``attend``,
residual, logits at ``meta.last_token_ix`` — so every token depends on the
whole paged history and the scheduler's greedy choices come from the backend.

Workload: requests in three prompt families arriving over several steps, so
later arrivals hit the radix cache on their family's published blocks; chunked
prefill (``max_prefill_tokens`` 32) mixed with decodes; a pool small enough
that the running batch exhausts it and the scheduler preempts by swapping a
victim out and resuming it later; and one copy-on-write, made the way the
reference's own COW test makes it (tests/test_radix.py:475-507: a second
holder takes a reference on a running sequence's partially filled last block,
then ``RadixCache.ensure_writable`` gives the writer a private copy through
``block_copy``). The reference scheduler never calls ``ensure_writable``
itself (block-granular reuse never needs it), so the harness does, between
two steps.

Every backend call is recorded in order — ``append_kv`` / ``attend`` inputs
and outputs with their ``BatchMeta`` fields, ``copy_block`` pairs, and the
swap space's ``swap_out`` (block ids, token count, the host K/V it produced),
``swap_in`` (the fresh block ids) and ``release`` — together with a SHA-256 of
the K/V pools after every scheduler step. ``tests/test_gpu_trace.py`` replays
it against ``B200PagedBackend`` / ``B200SwapSpace``.

Run in a container where the reference checkout exists (the fixture travels,
the reference does not):

    python tests/golden/make_trace.py /path/to/llm_serving_layer
"""

from __future__ import annotations

import hashlib
import math
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

import llm_serving_layer_b200.meta as meta_mod  # noqa: E402

OUT = HERE / "scheduler_trace.npz"

L, P, HKV, HQ, D = 2, 16, 8, 32, 64
NUM_BLOCKS = 9
VOCAB, DM = 64, 128
SCALE = 1.0 / math.sqrt(D)
META_FIELDS = ("query_lens", "cu_query_lens", "kv_lens", "positions", "last_token_ix", "kv_indptr",
               "kv_indices", "kv_last_page_len", "batch_indices", "slot_mapping")
KIND = {"append": 0, "attend": 1, "copy": 2, "swap_out": 3, "swap_in": 4, "release": 5, "step": 6}


def import_reference(ref_root: str):
    eng = types.ModuleType("engine")
    eng.attention_backend = meta_mod
    sys.modules["engine"] = eng
    sys.modules["engine.attention_backend"] = meta_mod
    sys.path.insert(0, ref_root)
    from serving.backends.paged_torch import PagedTorchBackend
    from serving.cache.radix import RadixCache
    from serving.memory.allocator import BlockAllocator
    from serving.scheduler.preemption import KVSwapSpace, PreemptionPolicy
    from serving.scheduler.scheduler import Request, Scheduler, SchedulerConfig

    return types.SimpleNamespace(**locals())


def rope(t: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    """Rotary embedding over (tokens, heads, D) at absolute positions, the
    formula of the reference's paged-model tests (halves a, b -> a cos - b sin,
    a sin + b cos), float32, base 500000 (Llama-3's)."""
    half = t.shape[-1] // 2
    inv = 500000.0 ** (-torch.arange(half, dtype=torch.float32) / half)
    ang = positions.to(torch.float32)[:, None] * inv[None, :]
    cos, sin = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
    a, b = t[..., :half], t[..., half:]
    return torch.cat([a * cos - b * sin, a * sin + b * cos], dim=-1)


class TraceModel:
    """A ``forward_varlen`` model over a paged backend: random float32 weights,
    fp16 q/k/v at the backend boundary (the pool's dtype)."""

    def __init__(self, seed: int = 20261202):
        g = torch.Generator().manual_seed(seed)

        def rand(*shape, std=1.0):
            return torch.randn(*shape, generator=g, dtype=torch.float32) * std

        self.device = torch.device("cpu")
        self.emb = rand(VOCAB, DM)
        self.wq = [rand(DM, HQ * D, std=DM ** -0.5) for _ in range(L)]
        self.wk = [rand(DM, HKV * D, std=DM ** -0.5) for _ in range(L)]
        self.wv = [rand(DM, HKV * D, std=DM ** -0.5) for _ in range(L)]
        self.wo = [rand(HQ * D, DM, std=(HQ * D) ** -0.5) for _ in range(L)]
        self.head = rand(DM, VOCAB, std=DM ** -0.5)

    def forward_varlen(self, tokens: torch.Tensor, meta, backend) -> torch.Tensor:
        t = tokens.shape[0]
        x = self.emb[tokens]
        pos = meta.positions
        for layer in range(L):
            q = rope((x @ self.wq[layer]).view(t, HQ, D), pos).half()
            k = rope((x @ self.wk[layer]).view(t, HKV, D), pos).half()
            v = (x @ self.wv[layer]).view(t, HKV, D).half()
            backend.append_kv(layer, k, v, meta)
            o = backend.attend(q, layer, SCALE, meta)
            x = x + o.float().reshape(t, HQ * D) @ self.wo[layer]
        return x[meta.last_token_ix.long()] @ self.head


class Trace:
    def __init__(self):
        self.ev: list[tuple[int, int, int, int, int, int]] = []
        self.step = 0
        self.metas: list = []
        self._meta_ix: dict[int, int] = {}
        self.k, self.v, self.q, self.out = [], [], [], []
        self.n_app = self.n_att = 0
        self.swap_blocks: list[int] = []
        self.swap_ntok: list[int] = []
        self.swap_nb: list[int] = []
        self.swap_k, self.swap_v = [], []
        self.swapin_blocks: list[int] = []
        self.pool_sha: list[str] = []

    def meta_index(self, meta) -> int:
        key = id(meta)
        if key not in self._meta_ix:
            self._meta_ix[key] = len(self.metas)
            self.metas.append(meta)  # the reference keeps the id alive
        return self._meta_ix[key]


class RecordingBackend:
    """Passes every call to the reference backend and records it."""

    def __init__(self, inner, trace: Trace):
        self._inner, self._t = inner, trace

    def __getattr__(self, name):
        return getattr(self._inner, name)

    def append_kv(self, layer_idx, k, v, meta):
        t = self._t
        t.ev.append((KIND["append"], t.step, layer_idx, t.meta_index(meta), t.n_app, k.shape[0]))
        t.k.append(k.numpy().copy())
        t.v.append(v.numpy().copy())
        t.n_app += k.shape[0]
        self._inner.append_kv(layer_idx, k, v, meta)

    def attend(self, q, layer_idx, scale, meta):
        assert scale == SCALE
        out = self._inner.attend(q, layer_idx, scale, meta)
        t = self._t
        t.ev.append((KIND["attend"], t.step, layer_idx, t.meta_index(meta), t.n_att, q.shape[0]))
        t.q.append(q.numpy().copy())
        t.out.append(out.numpy().copy())
        t.n_att += q.shape[0]
        return out

    def copy_block(self, src, dst):
        t = self._t
        t.ev.append((KIND["copy"], t.step, -1, -1, int(src), int(dst)))
        self._inner.copy_block(src, dst)


class RecordingSwap:
    """Passes every call to the reference ``KVSwapSpace`` and records it."""

    def __init__(self, inner, trace: Trace):
        self._inner, self._t = inner, trace
        self._hid: dict[int, int] = {}

    def __getattr__(self, name):
        return getattr(self._inner, name)

    def swap_out(self, request_id, blocks):
        h = self._inner.swap_out(request_id, blocks)
        t = self._t
        hid = len(t.swap_nb)
        self._hid[id(h)] = hid
        t.ev.append((KIND["swap_out"], t.step, -1, -1, hid, len(t.swap_blocks)))
        t.swap_blocks += [int(b) for b in blocks.block_ids]
        t.swap_nb.append(len(blocks.block_ids))
        t.swap_ntok.append(int(blocks.num_tokens))
        t.swap_k.append(h.k.numpy().copy())
        t.swap_v.append(h.v.numpy().copy())
        return h

    def swap_in(self, handle, blocks):
        t = self._t
        t.ev.append((KIND["swap_in"], t.step, -1, -1, self._hid[id(handle)], len(t.swapin_blocks)))
        t.swapin_blocks += [int(b) for b in blocks.block_ids]
        return self._inner.swap_in(handle, blocks)

    def release(self, handle):
        t = self._t
        if id(handle) in self._hid:
            t.ev.append((KIND["release"], t.step, -1, -1, self._hid[id(handle)], 0))
        return self._inner.release(handle)


def pool_digest(backend) -> str:
    h = hashlib.sha256()
    for layer in range(L):
        h.update(backend.k_pool[layer].numpy().tobytes())
        h.update(backend.v_pool[layer].numpy().tobytes())
    return h.hexdigest()


def workload(rs: np.random.RandomState):
    """(arrival step, request id, prompt, max_tokens): three families with a
    shared prefix each; later members arrive after the first has published
    whole blocks of the prefix."""
    fam = {f: list(rs.randint(0, VOCAB, size=n)) for f, n in (("a", 48), ("b", 40), ("c", 32))}
    reqs = [
        (0, "a0", fam["a"][:44], 9),
        (0, "b0", fam["b"][:38], 10),
        (0, "c0", fam["c"][:30], 8),
        (6, "a1", fam["a"][:32] + list(rs.randint(0, VOCAB, size=11)), 8),
        (8, "b1", fam["b"][:16] + list(rs.randint(0, VOCAB, size=9)), 9),
        (10, "c1", fam["c"][:16] + list(rs.randint(0, VOCAB, size=5)), 7),
    ]
    return [(s, rid, [int(x) for x in p], m) for s, rid, p, m in reqs]


def main(ref_root: str) -> None:
    torch.set_num_threads(1)
    ref = import_reference(ref_root)
    rs = np.random.RandomState(7)
    trace = Trace()
    alloc = ref.BlockAllocator(num_blocks=NUM_BLOCKS, block_size=P)
    inner = ref.PagedTorchBackend(num_layers=L, num_blocks=NUM_BLOCKS, block_size=P, n_kv_heads=HKV,
                                  n_heads=HQ, head_dim=D, device="cpu", dtype=torch.float16)
    backend = RecordingBackend(inner, trace)
    cache = ref.RadixCache(alloc, block_copy=backend.copy_block)
    sched = ref.Scheduler(TraceModel(), backend, alloc,
                          ref.SchedulerConfig(max_prefill_tokens=32,
                                              preemption_policy=ref.PreemptionPolicy.SWAP),
                          prefix_cache=cache)
    sched._swap = RecordingSwap(ref.KVSwapSpace(inner), trace)  # the scheduler's swap-space slot

    arrivals = workload(rs)
    reader = None  # (block id) held by the copy-on-write harness's second holder
    cow_done = False
    steps = 0
    while steps < 400 and (arrivals or sched.has_work):
        for a in [a for a in arrivals if a[0] <= steps]:
            sched.add_request(ref.Request(request_id=a[1], prompt_ids=a[2], max_tokens=a[3], ignore_eos=True))
            arrivals.remove(a)
        if not cow_done and steps >= 4:
            # a second holder of a running sequence's partial last block, then
            # the writer's copy-on-write (tests/test_radix.py:475-507)
            for req in sched.running:
                nb = len(req.blocks.block_ids) if req.blocks is not None else 0
                if nb and req.prefill_done and req.blocks.num_tokens % P and alloc.num_free >= 1:
                    old = req.blocks.block_ids[-1]
                    alloc.incref([old])
                    new = cache.ensure_writable(req.blocks, nb - 1)
                    assert new != old and req.blocks.block_ids[-1] == new
                    reader, cow_done, cow_step = old, True, steps
                    break
        if reader is not None and steps >= cow_step + 3:
            alloc.free([reader])  # the second holder lets go
            reader = None
        trace.step = steps
        sched.step()
        steps += 1
        trace.ev.append((KIND["step"], steps - 1, -1, -1, len(trace.pool_sha), 0))
        trace.pool_sha.append(pool_digest(inner))
        alloc.check_invariants()
    assert not sched.has_work and reader is None
    finished = {r.request_id: list(r.output_ids) for r in sched.finished}

    ev = np.asarray(trace.ev, dtype=np.int64)
    kinds = ev[:, 0]
    stats = {
        "steps": steps,
        "copy_block": int((kinds == KIND["copy"]).sum()),
        "swap_out": int((kinds == KIND["swap_out"]).sum()),
        "swap_in": int((kinds == KIND["swap_in"]).sum()),
        "blocks_reused": int(cache.stats.blocks_reused) if hasattr(cache.stats, "blocks_reused") else -1,
        "cow_copies": int(cache.stats.cow_copies),
        "preemptions": int(sched.preemption.total),
    }
    metas = trace.metas
    qmax = [int(m.query_lens.max()) for m in metas]
    stats["decode_steps"] = sum(1 for x in qmax if x == 1)
    stats["mixed_steps"] = sum(1 for m, x in zip(metas, qmax) if x > 1 and int(m.query_lens.min()) == 1)
    print(stats)
    assert stats["copy_block"] == 1 and stats["cow_copies"] == 1
    assert stats["swap_out"] >= 1 and stats["swap_in"] >= 1
    assert stats["blocks_reused"] > 0
    assert stats["decode_steps"] > 0 and stats["mixed_steps"] > 0

    arrays = {
        "geometry": np.asarray([L, NUM_BLOCKS, P, HKV, HQ, D], dtype=np.int64),
        "scale": np.asarray(SCALE, dtype=np.float64),
        "events": ev,
        "k": np.concatenate(trace.k), "v": np.concatenate(trace.v),
        "q": np.concatenate(trace.q), "out": np.concatenate(trace.out),
        "swap_blocks": np.asarray(trace.swap_blocks, dtype=np.int32),
        "swap_nb": np.asarray(trace.swap_nb, dtype=np.int64),
        "swap_ntok": np.asarray(trace.swap_ntok, dtype=np.int64),
        "swap_k": np.concatenate(trace.swap_k, axis=1), "swap_v": np.concatenate(trace.swap_v, axis=1),
        "swapin_blocks": np.asarray(trace.swapin_blocks, dtype=np.int32),
        "pool_sha": np.asarray(trace.pool_sha),
        "meta_is_prefill": np.asarray([bool(m.is_prefill) for m in metas]),
        "stats": np.asarray([stats[k] for k in sorted(stats)], dtype=np.int64),
        "stats_keys": np.asarray(sorted(stats)),
        "outputs": np.asarray([" ".join(f"{rid}:{','.join(map(str, toks))}" for rid, toks in sorted(finished.items()))]),
    }
    for f in META_FIELDS:
        parts = [getattr(m, f).numpy() for m in metas]
        arrays[f"meta_{f}"] = np.concatenate(parts).astype(np.int64)
        arrays[f"meta_{f}_off"] = np.cumsum([0] + [p.shape[0] for p in parts]).astype(np.int64)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1e6:.2f} MB): {len(ev)} events, {len(metas)} steps with a "
          f"forward pass, {arrays['q'].shape[0]} attended rows per layer-pass in total")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_trace.py /path/to/reference/checkout")
    main(sys.argv[1])
