"""
Generate the golden fixtures in this folder by running the REFERENCE's own code.

Run in a container where the reference checkout exists (it does not travel to
the GPU box; the fixtures do):

    python tests/golden/make_golden.py /path/to/llm_serving_layer

The reference's engine submodule (which defines ``BatchMeta``) is not vendored,
so ``engine.attention_backend`` is provided by this package's field-compatible
``llm_serving_layer_b200.meta`` before the reference is imported. Everything
computed here is the reference's: ``PagedTorchBackend.append_kv/attend/
copy_block`` (serving/backends/paged_torch.py), ``KVSwapSpace.swap_out/swap_in``
(serving/scheduler/preemption.py) and ``build_batch_meta``
(serving/engine_iface/batch.py).
"""

from __future__ import annotations

import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

from cases import (  # noqa: E402
    COPY_OPS,
    SWAP_GEOM,
    SWAP_TOKENS,
    attn_cases,
    copy_block_pool,
)

import llm_serving_layer_b200.meta as meta_mod  # noqa: E402


def import_reference(ref_root: str):
    eng = types.ModuleType("engine")
    eng.attention_backend = meta_mod
    sys.modules["engine"] = eng
    sys.modules["engine.attention_backend"] = meta_mod
    sys.path.insert(0, ref_root)
    from serving.backends.paged_torch import PagedTorchBackend
    from serving.engine_iface.batch import ScheduledSeq, build_batch_meta
    from serving.memory.allocator import BlockAllocator
    from serving.memory.block_table import SequenceBlocks
    from serving.scheduler.preemption import KVSwapSpace

    return types.SimpleNamespace(
        PagedTorchBackend=PagedTorchBackend, ScheduledSeq=ScheduledSeq,
        build_batch_meta=build_batch_meta, BlockAllocator=BlockAllocator,
        SequenceBlocks=SequenceBlocks, KVSwapSpace=KVSwapSpace,
    )


TORCH_DT = {"float16": torch.float16, "float32": torch.float32, "float64": torch.float64}


def gen_attention(ref) -> None:
    for c in attn_cases():
        c.materialise()
        dt = TORCH_DT[c.dtype]
        bk = ref.PagedTorchBackend(1, c.num_blocks, c.block_size, c.n_kv_heads,
                                   c.n_heads, c.head_dim, device="cpu", dtype=dt)
        if c.poison is not None:
            bk.k_pool[0].fill_(c.poison)
            bk.v_pool[0].fill_(c.poison)
        hist_slots = c.slots("hist")
        if hist_slots.size:
            hm = types.SimpleNamespace(slot_mapping=torch.from_numpy(hist_slots).to(torch.int32))
            bk.append_kv(0, torch.from_numpy(c.k_hist), torch.from_numpy(c.v_hist), hm)
        m = meta_mod.build_meta(c.tables, c.kv_lens, c.qlens, c.block_size)
        bk.append_kv(0, torch.from_numpy(c.k_new), torch.from_numpy(c.v_new), m)
        out = bk.attend(torch.from_numpy(c.q), 0, c.scale, m)
        np.savez(HERE / f"{c.name}.npz", out=out.numpy(), checksum=c.checksum(),
                 k_pool=bk.k_pool[0].numpy() if c.num_blocks * c.block_size <= 256 else np.zeros(0),
                 v_pool=bk.v_pool[0].numpy() if c.num_blocks * c.block_size <= 256 else np.zeros(0))
        print(f"{c.name}: out {tuple(out.shape)} {out.dtype}")


def gen_copy(ref) -> None:
    k, v = copy_block_pool()
    L, NB, P, H, D = k.shape
    bk = ref.PagedTorchBackend(L, NB, P, H, 2 * H, D, device="cpu", dtype=torch.float32)
    for l in range(L):
        bk.k_pool[l].copy_(torch.from_numpy(k[l]))
        bk.v_pool[l].copy_(torch.from_numpy(v[l]))
    for s, d in COPY_OPS:
        bk.copy_block(s, d)
    raised = []
    for s, d in [(-1, 0), (0, -1), (NB, 0), (0, NB)]:
        try:
            bk.copy_block(s, d)
        except IndexError:
            raised.append(1)
    np.savez(HERE / "copy_block.npz",
             k=np.stack([t.numpy() for t in bk.k_pool]),
             v=np.stack([t.numpy() for t in bk.v_pool]),
             raised=np.asarray(raised))
    print("copy_block: ok")


def gen_swap(ref) -> None:
    g = SWAP_GEOM
    bk = ref.PagedTorchBackend(g["num_layers"], g["num_blocks"], g["block_size"],
                               g["n_kv_heads"], 2 * g["n_kv_heads"], g["head_dim"],
                               device="cpu", dtype=torch.float64)
    alloc = ref.BlockAllocator(num_blocks=g["num_blocks"], block_size=g["block_size"])
    # fragment: take everything, hand back a scattered, non-monotonic set
    held = alloc.allocate(g["num_blocks"])
    alloc.free([held[i] for i in (11, 2, 7, 14, 0, 9, 5, 12, 3, 15, 1, 6, 8, 13, 10, 4)])
    src = ref.SequenceBlocks(alloc, seq_id=1)
    src.append(SWAP_TOKENS)
    for layer in range(bk.num_layers):
        for i, b in enumerate(src.block_ids):
            bk.k_pool[layer][b] = 7.0 + layer * 100 + i + torch.arange(
                g["block_size"] * g["n_kv_heads"] * g["head_dim"], dtype=torch.float64
            ).view(g["block_size"], g["n_kv_heads"], g["head_dim"]) / 1000
            bk.v_pool[layer][b] = -(7.0 + layer * 100 + i)
    swap = ref.KVSwapSpace(bk)
    src_ids = list(src.block_ids)
    handle = swap.swap_out("r", src)
    src.free()
    decoy = ref.SequenceBlocks(alloc, seq_id=2)
    decoy.append(SWAP_TOKENS)
    for layer in range(bk.num_layers):
        for b in decoy.block_ids:
            bk.k_pool[layer][b] = -99.0
            bk.v_pool[layer][b] = -99.0
    dst = ref.SequenceBlocks(alloc, seq_id=3)
    dst.append(handle.num_tokens)
    swap.swap_in(handle, dst)
    np.savez(HERE / "swap_roundtrip.npz",
             src_ids=np.asarray(src_ids), decoy_ids=np.asarray(decoy.block_ids),
             dst_ids=np.asarray(dst.block_ids),
             k_host=handle.k.numpy(), v_host=handle.v.numpy(),
             k_pool=np.stack([t.numpy() for t in bk.k_pool]),
             v_pool=np.stack([t.numpy() for t in bk.v_pool]),
             nbytes=np.asarray(handle.nbytes))
    print(f"swap: {src_ids} -> {dst.block_ids}")


def gen_batch(ref) -> None:
    alloc = ref.BlockAllocator(num_blocks=64, block_size=16)
    held = alloc.allocate(64)
    rs = np.random.RandomState(7)
    alloc.free([held[i] for i in rs.permutation(64)])
    lens_hist = [20, 0, 16, 47, 1]
    qlens = [1, 33, 1, 17, 1]
    seqs = []
    for i, (h, q) in enumerate(zip(lens_hist, qlens)):
        s = ref.SequenceBlocks(alloc, seq_id=i)
        if h:
            s.append(h)
        s.append(q)
        seqs.append(ref.ScheduledSeq(s, list(range(q))))
    m = ref.build_batch_meta(seqs, "cpu", 16)
    fields = {f: getattr(m, f).numpy() for f in (
        "query_lens", "cu_query_lens", "kv_lens", "positions", "last_token_ix",
        "kv_indptr", "kv_indices", "kv_last_page_len", "batch_indices", "slot_mapping")}
    tables = [s.blocks.block_ids for s in seqs]
    flat = np.concatenate([np.asarray(t) for t in tables])
    lens = np.asarray([len(t) for t in tables])
    np.savez(HERE / "batch_assembly.npz", tables_flat=flat, tables_len=lens,
             hist=np.asarray(lens_hist), qlens=np.asarray(qlens),
             is_prefill=np.asarray(m.is_prefill), **fields)
    print("batch_assembly: ok")


def gen_rope(ref_root: str) -> None:
    """The reference's own rotary embedding (``_rope`` of its paged-model tests,
    tests/test_preemption.py:85-102, float64, theta 10000) on seeded inputs;
    the positions include 0 and values past 2^11."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("ref_test_preemption", Path(ref_root, "tests/test_preemption.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    g = torch.Generator().manual_seed(11)
    T, H, D = 37, 3, 64
    x = torch.randn(T, H, D, generator=g, dtype=torch.float64)
    positions = torch.randint(0, 5000, (T,), generator=g, dtype=torch.int64)
    positions[:3] = torch.tensor([0, 1, 4097])
    out = mod._rope(x, positions)
    np.savez(HERE / "rope.npz", x=x.numpy(), positions=positions.numpy(), out=out.numpy(), theta=10000.0)
    print("rope: ok")


def main() -> None:
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LLM_SERVING_LAYER_REF", "")
    if not ref_root or not Path(ref_root, "serving").is_dir():
        raise SystemExit("usage: make_golden.py <reference checkout>")
    torch.set_num_threads(1)
    ref = import_reference(ref_root)
    gen_attention(ref)
    gen_copy(ref)
    gen_swap(ref)
    gen_batch(ref)
    gen_rope(ref_root)


if __name__ == "__main__":
    main()
