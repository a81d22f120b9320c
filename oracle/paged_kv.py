"""
CPU ORACLE — TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

numpy restatement of the reference's paged-KV path. Every function cites the
reference file:line whose algorithm it follows; the steps, their order and the
precision of each step are the reference's.

Pool layout (as the reference's): per layer, K and V are separate arrays of
shape ``[num_blocks, block_size, n_kv_heads, head_dim]``; a flat slot
``s = block * block_size + offset`` addresses one ``[n_kv_heads, head_dim]``
token row.
"""

from __future__ import annotations

from typing import Any, Mapping, Sequence

import numpy as np

__all__ = [
    "slot_for",
    "last_page_len",
    "build_csr",
    "meta_arrays",
    "attend_reference",
    "attend_exact",
    "rope",
    "OraclePool",
]


# ---------------------------------------------------------------------------
# block-table arithmetic — serving/memory/block_table.py
# ---------------------------------------------------------------------------


def slot_for(block_ids: Sequence[int], position: int, block_size: int) -> int:
    """Physical slot of a logical position (``block_table.py:100-109``)."""
    if not 0 <= position < len(block_ids) * block_size:
        raise IndexError(f"position {position} outside table of {len(block_ids)} blocks")
    return int(block_ids[position // block_size]) * block_size + position % block_size


def last_page_len(num_tokens: int, block_size: int) -> int:
    """Occupancy of the final block, in [1, block_size] (``block_table.py:124-138``)."""
    if num_tokens <= 0:
        raise ValueError("last_page_len is undefined for an empty sequence")
    rem = num_tokens % block_size
    return rem if rem else block_size


def build_csr(
    tables: Sequence[Sequence[int]], num_tokens: Sequence[int], block_size: int
) -> tuple[list[int], list[int], list[int]]:
    """Concatenate block tables into (kv_indptr, kv_indices, kv_last_page_len)
    (``block_table.py:184-208``)."""
    indptr, indices, last = [0], [], []
    for ids, n in zip(tables, num_tokens):
        indices.extend(int(b) for b in ids)
        indptr.append(len(indices))
        last.append(last_page_len(int(n), block_size))
    return indptr, indices, last


def meta_arrays(meta: Any) -> dict[str, np.ndarray]:
    """Pull a BatchMeta-like object's fields to host numpy int64 arrays."""
    out: dict[str, np.ndarray] = {}
    for name in (
        "query_lens", "cu_query_lens", "kv_lens", "positions", "kv_indptr",
        "kv_indices", "kv_last_page_len", "batch_indices", "slot_mapping",
    ):
        v = meta[name] if isinstance(meta, Mapping) else getattr(meta, name, None)
        if v is None:
            out[name] = None  # type: ignore[assignment]
            continue
        if hasattr(v, "detach"):
            v = v.detach().cpu().numpy()
        out[name] = np.asarray(v, dtype=np.int64)
    return out


# ---------------------------------------------------------------------------
# attention — serving/backends/paged_torch.py:280-485
# ---------------------------------------------------------------------------


def _gather(pool_l: np.ndarray, pages: np.ndarray, kv_len: int, last: int) -> np.ndarray:
    """Dense ``(kv_len, H, D)`` history of one sequence (``paged_torch.py:348-398``):
    checks page count and last-page length, gathers pages in listed order,
    truncates to ``kv_len`` so the unwritten tail of the last page is never read."""
    bs = pool_l.shape[1]
    need = (kv_len + bs - 1) // bs
    if pages.shape[0] != need:
        raise ValueError(f"{pages.shape[0]} pages supplied but kv_len={kv_len} needs {need}")
    tail = kv_len - (pages.shape[0] - 1) * bs
    if last != tail:
        raise ValueError(f"kv_last_page_len={last} but kv_len={kv_len} implies {tail}")
    return pool_l[pages].reshape(-1, pool_l.shape[2], pool_l.shape[3])[:kv_len]


def _softmax_f32(x: np.ndarray) -> np.ndarray:
    m = np.max(x, axis=-1, keepdims=True)
    e = np.exp(x - m, dtype=np.float32)
    return (e / np.sum(e, axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)


def attend_reference(
    q: np.ndarray, k_pool_l: np.ndarray, v_pool_l: np.ndarray, scale: float, meta: Any
) -> np.ndarray:
    """The reference's attention, step for step (``paged_torch.py:280-346,400-485``).

    Per sequence: gather its pages, query head ``h`` reads KV head
    ``h // groups`` (the ``repeat_interleave`` mapping, done here by grouping
    the query heads of one KV head instead of copying K/V), scores ``q·kᵀ`` in
    float32 times ``scale``, bottom-right causal mask ``triu(kv_len - q_len + 1)``
    when ``q_len > 1``, float32 softmax, probabilities cast to the pool dtype,
    then ``probs @ v`` in the pool dtype. Returns ``(tokens, n_heads, head_dim)``
    in the pool dtype.
    """
    m = meta_arrays(meta)
    dt = k_pool_l.dtype
    T, Hq, D = q.shape
    Hkv = k_pool_l.shape[2]
    g = Hq // Hkv
    out = np.zeros((T, Hq, D), dtype=dt)
    cu, ql, kl = m["cu_query_lens"], m["query_lens"], m["kv_lens"]
    ip, idx, lp = m["kv_indptr"], m["kv_indices"], m["kv_last_page_len"]
    for i in range(ql.shape[0]):
        q_len, kv_len = int(ql[i]), int(kl[i])
        if q_len == 0:
            continue
        pages = idx[ip[i]: ip[i + 1]]
        k = _gather(k_pool_l, pages, kv_len, int(lp[i]))  # (kv, Hkv, D)
        v = _gather(v_pool_l, pages, kv_len, int(lp[i]))
        # (q_len, Hq, D) -> (Hkv, g*q_len, D): row (j, t) of KV head c is query head c*g + j
        qg = q[cu[i]: cu[i + 1]].reshape(q_len, Hkv, g, D).transpose(1, 2, 0, 3).reshape(Hkv, g * q_len, D)
        scores = np.matmul(qg.astype(np.float32), k.astype(np.float32).transpose(1, 2, 0))
        scores = (scores * np.float32(scale)).reshape(Hkv, g, q_len, kv_len)
        if q_len > 1:
            off = kv_len - q_len
            mask = np.triu(np.full((q_len, kv_len), -np.inf, dtype=np.float32), k=off + 1)
            scores = scores + mask
        probs = _softmax_f32(scores).astype(dt).reshape(Hkv, g * q_len, kv_len)
        o = np.matmul(probs, v.transpose(1, 0, 2)).astype(dt)  # pool dtype
        out[cu[i]: cu[i + 1]] = o.reshape(Hkv, g, q_len, D).transpose(2, 0, 1, 3).reshape(q_len, Hq, D)
    return out


def attend_exact(
    q: np.ndarray, k_pool_l: np.ndarray, v_pool_l: np.ndarray, scale: float, meta: Any
) -> np.ndarray:
    """The same attention evaluated in float64 with no intermediate rounding:
    the "contiguous softmax(q·kᵀ·scale)·v" the tolerance is measured against.
    Same gather, GQA mapping and bottom-right causal rule as ``attend_reference``."""
    m = meta_arrays(meta)
    T, Hq, D = q.shape
    Hkv = k_pool_l.shape[2]
    groups = Hq // Hkv
    out = np.zeros((T, Hq, D), dtype=np.float64)
    cu, ql, kl = m["cu_query_lens"], m["query_lens"], m["kv_lens"]
    ip, idx, lp = m["kv_indptr"], m["kv_indices"], m["kv_last_page_len"]
    for i in range(ql.shape[0]):
        q_len, kv_len = int(ql[i]), int(kl[i])
        if q_len == 0:
            continue
        pages = idx[ip[i]: ip[i + 1]]
        k = _gather(k_pool_l, pages, kv_len, int(lp[i])).astype(np.float64)
        v = _gather(v_pool_l, pages, kv_len, int(lp[i])).astype(np.float64)
        k = np.repeat(k, groups, axis=1).transpose(1, 0, 2)
        v = np.repeat(v, groups, axis=1).transpose(1, 0, 2)
        qh = q[cu[i]: cu[i + 1]].astype(np.float64).transpose(1, 0, 2)
        s = np.matmul(qh, k.transpose(0, 2, 1)) * float(scale)
        if q_len > 1:
            off = kv_len - q_len
            s = s + np.triu(np.full((q_len, kv_len), -np.inf), k=off + 1)[None]
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=-1, keepdims=True)
        out[cu[i]: cu[i + 1]] = np.matmul(p, v).transpose(1, 0, 2)
    return out


# ---------------------------------------------------------------------------
# rotary embedding — the engine step before append_kv / attend
# ---------------------------------------------------------------------------

def rope(x: np.ndarray, positions, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Rotary embedding of ``x`` ``(tokens, heads, head_dim)`` at each token's
    absolute position, with cosine / sine tables ``[max_pos, head_dim // 2]``.

    The formula is the one of the reference's own paged model
    (``tests/test_preemption.py:85-102``: the two halves a = x[..., :D/2],
    b = x[..., D/2:] become ``a*cos - b*sin`` and ``a*sin + b*cos``) and of the
    engine it stands in for, which indexes precomputed tables by
    ``meta.positions`` (``docs/ENGINE_INTEGRATION.md:108``: ``cos[positions]``
    applied to q and k). Arithmetic in the tables' dtype, every product and
    sum rounded on its own (numpy evaluates each operation separately), then
    cast to ``x``'s dtype (round to nearest even)."""
    pos = np.asarray(positions, dtype=np.int64)
    c = cos[pos][:, None, :]
    s = sin[pos][:, None, :]
    half = x.shape[-1] // 2
    a = x[..., :half].astype(cos.dtype)
    b = x[..., half:].astype(cos.dtype)
    return np.concatenate([a * c - b * s, a * s + b * c], axis=-1).astype(x.dtype)


# ---------------------------------------------------------------------------
# the pool: append, copy_block, swap — paged_torch.py / preemption.py
# ---------------------------------------------------------------------------


class OraclePool:
    """Per-layer K/V pools with the reference's write-side operations."""

    def __init__(self, num_layers: int, num_blocks: int, block_size: int,
                 n_kv_heads: int, head_dim: int, dtype=np.float16):
        shape = (num_blocks, block_size, n_kv_heads, head_dim)
        self.num_layers = num_layers
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.k = [np.zeros(shape, dtype=dtype) for _ in range(num_layers)]
        self.v = [np.zeros(shape, dtype=dtype) for _ in range(num_layers)]

    def append_kv(self, layer: int, k: np.ndarray, v: np.ndarray, slot_mapping) -> None:
        """Indexed scatter ``pool.view(-1,H,D)[slots] = k`` (``paged_torch.py:270-276``).
        For duplicate slots the later token wins, as with sequential assignment."""
        slots = np.asarray(slot_mapping, dtype=np.int64)
        H, D = self.k[layer].shape[2:]
        kf = self.k[layer].reshape(-1, H, D)
        vf = self.v[layer].reshape(-1, H, D)
        kf[slots] = k.astype(kf.dtype)
        vf[slots] = v.astype(vf.dtype)

    def copy_block(self, src: int, dst: int) -> None:
        """Duplicate one block across every layer, K and V (``paged_torch.py:181-207``);
        ``IndexError`` out of range, no-op when ``src == dst``."""
        if not (0 <= src < self.num_blocks and 0 <= dst < self.num_blocks):
            raise IndexError(f"copy_block({src} -> {dst}) outside [0, {self.num_blocks})")
        if src == dst:
            return
        for layer in range(self.num_layers):
            self.k[layer][dst] = self.k[layer][src]
            self.v[layer][dst] = self.v[layer][src]

    def swap_out(self, block_ids: Sequence[int]) -> tuple[np.ndarray, np.ndarray]:
        """Gather a sequence's blocks, every layer, into ``(L, nb, P, H, D)`` host
        arrays in logical block order (``preemption.py:490-509``)."""
        idx = np.asarray(block_ids, dtype=np.int64)
        k = np.stack([self.k[l][idx] for l in range(self.num_layers)])
        v = np.stack([self.v[l][idx] for l in range(self.num_layers)])
        return k, v

    def swap_in(self, k_host: np.ndarray, v_host: np.ndarray, block_ids: Sequence[int]) -> None:
        """Scatter host block ``i`` to ``block_ids[i]`` for every layer
        (``preemption.py:511-523``)."""
        idx = np.asarray(block_ids, dtype=np.int64)
        if k_host.shape[1] != idx.shape[0]:
            raise RuntimeError(
                f"resume mismatch: {idx.shape[0]} blocks allocated, {k_host.shape[1]} swapped out"
            )
        for l in range(self.num_layers):
            self.k[l][idx] = k_host[l]
            self.v[l][idx] = v_host[l]

    def attend(self, q: np.ndarray, layer: int, scale: float, meta: Any, exact: bool = False):
        f = attend_exact if exact else attend_reference
        return f(q, self.k[layer], self.v[layer], scale, meta)
