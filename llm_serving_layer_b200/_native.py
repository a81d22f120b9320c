"""
ctypes binding of ``libpkv.so`` (the C ABI declared in ``include/pkv.h``).

The library is built in-tree (``python -m llm_serving_layer_b200.build``) and
loaded from ``llm_serving_layer_b200/_lib/libpkv.so``. There is no fallback: if
the library is missing or does not load, every entry point raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libpkv.so"

PKV_OK, PKV_ERR_ARG, PKV_ERR_UNSUPPORTED, PKV_ERR_CUDA, PKV_ERR_DEVICE = 0, 1, 2, 3, 4
PKV_KERNEL_GENERIC, PKV_KERNEL_DECODE, PKV_KERNEL_PREFILL = 0, 1, 2
KERNEL_NAMES = {PKV_KERNEL_GENERIC: "generic", PKV_KERNEL_DECODE: "decode", PKV_KERNEL_PREFILL: "prefill"}
DEV_SLOT_OOB, DEV_META_BAD, DEV_QLEN_BAD, DEV_WAIT_TIMEOUT, DEV_WORKSPACE = 0x1, 0x2, 0x4, 0x8, 0x10

DTYPE_CODE = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2, torch.float64: 3}

c_i32, c_i64, c_u64, c_size, c_vp, c_float = (
    ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_float)


class PoolDesc(ctypes.Structure):
    _fields_ = [("base", c_vp), ("num_blocks", c_i64), ("num_layers", c_i32),
                ("block_size", c_i32), ("n_kv_heads", c_i32), ("head_dim", c_i32),
                ("dtype", c_i32), ("reserved", c_i32)]


class BatchDesc(ctypes.Structure):
    _fields_ = [("n_seqs", c_i32), ("n_tokens", c_i32), ("total_pages", c_i64),
                ("cu_query_lens", c_vp), ("kv_lens", c_vp), ("kv_indptr", c_vp),
                ("kv_indices", c_vp), ("kv_last_page_len", c_vp), ("dev_status", c_vp)]


class BlockTablesDesc(ctypes.Structure):
    _fields_ = [("table", c_vp), ("max_seqs", c_i32), ("max_pages", c_i32), ("block_size", c_i32),
                ("reserved", c_i32)]


class MetaOutDesc(ctypes.Structure):
    _fields_ = [("query_lens", c_vp), ("cu_query_lens", c_vp), ("kv_lens", c_vp), ("positions", c_vp),
                ("last_token_ix", c_vp), ("kv_indptr", c_vp), ("kv_indices", c_vp),
                ("kv_last_page_len", c_vp), ("batch_indices", c_vp), ("slot_mapping", c_vp),
                ("seqs_cap", c_i32), ("reserved", c_i32), ("tokens_cap", c_i64), ("pages_cap", c_i64)]


P_POOL = ctypes.POINTER(PoolDesc)
P_BATCH = ctypes.POINTER(BatchDesc)
P_TABLES = ctypes.POINTER(BlockTablesDesc)
P_META_OUT = ctypes.POINTER(MetaOutDesc)

# name -> (restype, argtypes); every symbol include/pkv.h declares
SIGNATURES = {
    "pkv_version": (c_i32, []),
    "pkv_last_error": (ctypes.c_char_p, []),
    "pkv_append_kv": (c_i32, [P_POOL, c_i32, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp]),
    "pkv_attend_workspace_size": (c_size, [P_POOL, c_i32, c_i32, c_i64, c_i32]),
    "pkv_attend": (c_i32, [P_POOL, c_i32, c_i32, c_vp, c_vp, c_float, P_BATCH, c_i32, c_vp, c_size, c_vp]),
    "pkv_plan": (c_i32, [P_POOL, c_i32, P_BATCH, c_vp, c_size, c_vp]),
    "pkv_attend_planned": (c_i32, [P_POOL, c_i32, c_i32, c_vp, c_vp, c_float, P_BATCH, c_i32, c_vp, c_size, c_vp]),
    "pkv_attend_kernel": (c_i32, [P_POOL, c_i32, c_i32, c_i32, c_i32]),
    "pkv_append_attend_planned": (c_i32, [P_POOL, c_i32, c_i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_float, P_BATCH,
                                          c_i32, c_vp, c_size, c_vp]),
    "pkv_rope": (c_i32, [c_i32, c_vp, c_vp, c_i32, c_vp, c_vp, c_i32, c_i64, c_i32, c_vp, c_vp, c_vp, c_i64, c_vp,
                         c_vp]),
    "pkv_append_attend_rope_planned": (c_i32, [P_POOL, c_i32, c_i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_float, P_BATCH,
                                               c_i32, c_vp, c_size, c_vp, c_vp, c_vp, c_i64, c_vp]),
    "pkv_attend_decode_noalloc": (c_i32, [P_POOL, c_i32, c_i32, c_vp, c_vp, c_float, P_BATCH, c_vp]),
    "pkv_wait_probe": (c_i32, [c_vp, c_vp, c_vp, c_vp]),
    "pkv_sample_greedy": (c_i32, [c_i32, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_i64, c_vp, c_vp, c_vp]),
    "pkv_copy_blocks": (c_i32, [P_POOL, c_vp, c_vp, c_i64, c_vp, c_vp]),
    "pkv_copy_block": (c_i32, [P_POOL, c_i64, c_i64, c_vp]),
    "pkv_build_batch_meta": (c_i32, [P_TABLES, c_vp, c_vp, c_i32, c_i32, P_META_OUT, c_vp, c_vp]),
    "pkv_swap_gather": (c_i32, [P_POOL, c_vp, c_i64, c_vp, c_vp, c_vp]),
    "pkv_swap_scatter": (c_i32, [P_POOL, c_vp, c_i64, c_vp, c_vp, c_vp]),
    "pkv_swapper_create": (c_i32, [c_vp, c_size, ctypes.POINTER(c_vp)]),
    "pkv_swapper_destroy": (c_i32, [c_vp]),
    "pkv_swap_out": (c_i32, [c_vp, P_POOL, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, ctypes.POINTER(c_u64)]),
    "pkv_swap_in": (c_i32, [c_vp, P_POOL, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, ctypes.POINTER(c_u64)]),
    "pkv_swapper_wait": (c_i32, [c_vp, c_u64]),
    "pkv_swapper_done": (c_i32, [c_vp, c_u64]),
}

_lib: ctypes.CDLL | None = None


class PkvError(RuntimeError):
    """A libpkv call failed; ``code`` is the PKV_ERR_* status."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def lib() -> ctypes.CDLL:
    """Load libpkv.so once. Raises if it is missing: there is no CPU path."""
    global _lib
    if _lib is None:
        path = Path(os.environ.get("PKV_LIB", LIB_PATH))
        if not path.exists():
            raise RuntimeError(
                f"libpkv.so not found at {path}; build it with "
                "`python -m llm_serving_layer_b200.build` (nvcc, sm_100a)")
        l = ctypes.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def check(rc: int, what: str, arg_exc: type[Exception] = ValueError) -> None:
    """Raise for a non-OK status: argument errors as ``arg_exc`` (ValueError by
    default, matching the reference's validation errors), others as PkvError."""
    if rc == PKV_OK:
        return
    msg = lib().pkv_last_error().decode(errors="replace")
    if rc == PKV_ERR_ARG:
        raise arg_exc(f"{what}: {msg}")
    raise PkvError(rc, f"{what} failed ({rc}): {msg}")


def describe_status(bits: int) -> str:
    names = []
    for bit, name in ((DEV_SLOT_OOB, "slot or block id outside the pool"),
                      (DEV_META_BAD, "page table inconsistent with kv_lens / kv_last_page_len"),
                      (DEV_QLEN_BAD, "decode kernel given a query length != 1"),
                      (DEV_WAIT_TIMEOUT, "a bounded device wait timed out"),
                      (DEV_WORKSPACE, "workspace too small")):
        if bits & bit:
            names.append(name)
    return "; ".join(names) or "ok"


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def raw_stream(device_index: int) -> int:
    """cudaStream_t of torch's current stream on `device_index` (the handle
    torch.cuda.current_stream(device).cuda_stream returns, without building a
    Stream object on every call)."""
    if _raw_stream is not None:
        return _raw_stream(device_index)
    return torch.cuda.current_stream(device_index).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()
