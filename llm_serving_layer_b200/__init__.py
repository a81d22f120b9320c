"""
llm_serving_layer_b200 — B200-native (sm_100a) paged-KV hot path for the
``llm_serving_layer`` serving system.

Drop-ins behind the reference's own interfaces:

* ``B200PagedBackend`` — attention backend (``append_kv`` / ``attend`` /
  ``copy_block``), replacing ``serving.backends.paged_torch.PagedTorchBackend``
  and ``serving.backends.flashinfer_backend.FlashInferBackend``;
* ``B200SwapSpace`` — preemption swap engine, replacing
  ``serving.scheduler.preemption.KVSwapSpace``;
* ``BatchMeta`` / ``build_meta`` — the engine's step descriptor (field-for-field)
  and a vectorised host assembler;
* ``DeviceBlockTables`` — block tables kept on the device and each step's
  ``BatchMeta`` assembled there, replacing the engine's ``build_batch_meta``;
* ``BlockAllocator`` / ``RadixCache`` / ``attach_prefix`` (``radix``) — the
  block manager and prefix cache the scheduler drives, with eviction in
  O(log nodes) and an O(1) invariant check, replacing
  ``serving.memory.allocator`` / ``serving.cache.radix``;
* ``sample_greedy`` / ``TokenReadback`` — greedy sampling on the device into a
  device token table, with the host reading the tokens a step later,
  replacing the scheduler's ``torch.argmax(logits).tolist()``.

All compute runs in ``_lib/libpkv.so`` (hand-written CUDA, C ABI in
``include/pkv.h``); build it with ``python -m llm_serving_layer_b200.build``.
"""

from .backend import B200PagedBackend
from .meta import AttentionBackend, BatchMeta, build_meta
from .radix import BlockAllocator, RadixCache, attach_prefix
from .sampling import TokenReadback, sample_greedy
from .swap import B200SwapSpace, SwapHandle, SwapSpaceFull
from .tables import DeviceBlockTables

__all__ = [
    "B200PagedBackend",
    "B200SwapSpace",
    "SwapHandle",
    "SwapSpaceFull",
    "BatchMeta",
    "AttentionBackend",
    "build_meta",
    "DeviceBlockTables",
    "BlockAllocator",
    "RadixCache",
    "attach_prefix",
    "sample_greedy",
    "TokenReadback",
]
