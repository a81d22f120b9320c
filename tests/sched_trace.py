"""
Loader of ``tests/golden/scheduler_trace.npz``: the backend and swap-space calls
the reference's own ``Scheduler`` + ``RadixCache`` + ``KVSwapSpace`` made on its
``PagedTorchBackend`` (recorded by ``tests/golden/make_trace.py``), in order.

``load()`` returns a ``SchedulerTrace`` whose ``events()`` yields one tuple per
recorded call:

* ``("append", step, layer, meta_ix, k, v)``
* ``("attend", step, layer, meta_ix, q, out)`` — ``out`` is the reference's output
* ``("copy", step, src, dst)``
* ``("swap_out", step, handle_id, block_ids, num_tokens, k_host, v_host)``
* ``("swap_in", step, handle_id, block_ids)``
* ``("release", step, handle_id)``
* ``("step", step, pool_sha256)`` — after each scheduler step, the SHA-256 of
  the reference's K then V pools, layer by layer (``[NB,16,8,64]`` fp16 each)

and ``meta(i)`` the fields of the ``BatchMeta`` the reference built for a step.
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np

PATH = Path(__file__).resolve().parent / "golden" / "scheduler_trace.npz"
META_FIELDS = ("query_lens", "cu_query_lens", "kv_lens", "positions", "last_token_ix", "kv_indptr",
               "kv_indices", "kv_last_page_len", "batch_indices", "slot_mapping")
KINDS = ("append", "attend", "copy", "swap_out", "swap_in", "release", "step")


class SchedulerTrace:
    def __init__(self, path: Path = PATH):
        z = np.load(path)
        self.z = {k: z[k] for k in z.files}
        self.num_layers, self.num_blocks, self.block_size, self.n_kv_heads, self.n_heads, self.head_dim = (
            int(x) for x in self.z["geometry"])
        self.scale = float(self.z["scale"])
        self.stats = dict(zip(self.z["stats_keys"].tolist(), self.z["stats"].tolist()))
        self.n_metas = int(self.z["meta_query_lens_off"].shape[0] - 1)

    def meta(self, i: int) -> dict:
        out = {}
        for f in META_FIELDS:
            off = self.z[f"meta_{f}_off"]
            out[f] = self.z[f"meta_{f}"][off[i]:off[i + 1]]
        out["is_prefill"] = bool(self.z["meta_is_prefill"][i])
        return out

    def events(self):
        z = self.z
        swap_off = np.concatenate([[0], np.cumsum(z["swap_nb"])])
        for kind, step, layer, mi, a, b in z["events"].tolist():
            name = KINDS[kind]
            if name == "append":
                yield name, step, layer, mi, z["k"][a:a + b], z["v"][a:a + b]
            elif name == "attend":
                yield name, step, layer, mi, z["q"][a:a + b], z["out"][a:a + b]
            elif name == "copy":
                yield name, step, a, b
            elif name == "swap_out":
                nb = int(z["swap_nb"][a])
                yield (name, step, a, z["swap_blocks"][b:b + nb].tolist(), int(z["swap_ntok"][a]),
                       z["swap_k"][:, swap_off[a]:swap_off[a] + nb], z["swap_v"][:, swap_off[a]:swap_off[a] + nb])
            elif name == "swap_in":
                nb = int(z["swap_nb"][a])
                yield name, step, a, z["swapin_blocks"][b:b + nb].tolist()
            elif name == "release":
                yield name, step, a
            else:
                yield name, step, str(z["pool_sha"][a])


def load() -> SchedulerTrace:
    return SchedulerTrace()


def pool_sha(k_pools, v_pools) -> str:
    """SHA-256 of per-layer K then V pools given as numpy arrays, the digest the
    trace records after every step."""
    h = hashlib.sha256()
    for k, v in zip(k_pools, v_pools):
        h.update(np.ascontiguousarray(k).tobytes())
        h.update(np.ascontiguousarray(v).tobytes())
    return h.hexdigest()


class Blocks:
    """The two ``SequenceBlocks`` attributes a swap space reads, plus the ones
    its checks look at."""

    def __init__(self, ids, n, seq_id=0):
        self.block_ids, self.num_tokens, self.seq_id, self.is_freed = list(ids), n, seq_id, False
