"""
The tcgen05 prefill kernels against each other's paths and the oracle.

Launches of more than one wave of CTAs (more than two tiles x KV heads per SM)
run a persistent kernel — by default the lean one (three CTAs per SM), with
``PKV_PREFILL_LEAN=0`` the two-CTA one — and smaller launches one CTA per
tile. The environment variables (read once per process) move the lines:
``PKV_PREFILL_PERSISTENT=2`` sends every launch to the two-CTA persistent
kernel, ``PKV_PREFILL_PERSISTENT=0`` none; ``PKV_PREFILL_LEAN=2`` every launch
to the lean kernel; one-CTA-per-tile launches split each tile's key blocks
over two groups of the CTA when they have at most one CTA per SM
(``PKV_PREFILL_SPLIT=2``: every such launch, ``0``: none). Here the whole prefill suite and the reference-scheduler
trace replay run again in child processes under each setting, so each kernel
meets every case (chunks after long prefixes, tile and page edges, every GQA
group size, bf16, NaN-poisoned page tails, radix sharing with copy-on-write,
mixed batches), and a large batch — persistent CTAs walking several tiles
each — with one sequence whose page table points outside the pool and one
whose lengths disagree checks that only those sequences are affected: the
first gets zero rows and ``PKV_DEV_SLOT_OOB``, the second no rows written and
``PKV_DEV_META_BAD``, and every other row is within the fp16 tolerance of the
float64 evaluation (in this process with the default kernel, and in a child
process with the two-CTA persistent kernel).
"""

from __future__ import annotations

import dataclasses
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from llm_serving_layer_b200 import _native as N
from test_gpu_prefill import build_step, exact

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


KERNELS = {
    "persistent": {"PKV_PREFILL_PERSISTENT": "2", "PKV_PREFILL_LEAN": "0"},
    "lean": {"PKV_PREFILL_LEAN": "2"},
    "per_tile": {"PKV_PREFILL_PERSISTENT": "0", "PKV_PREFILL_LEAN": "0", "PKV_PREFILL_SPLIT": "0"},
    "per_tile_split": {"PKV_PREFILL_PERSISTENT": "0", "PKV_PREFILL_LEAN": "0", "PKV_PREFILL_SPLIT": "2"},
}


def _child(env_over, *targets):
    env = dict(os.environ, **env_over)
    r = subprocess.run([sys.executable, "-m", "pytest", "-x", "-q", "-m", "gpu", "-p", "no:cacheprovider", *targets],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


@pytest.mark.parametrize("kernel", sorted(KERNELS))
def test_prefill_suite_under_each_kernel(kernel):
    _child(KERNELS[kernel], "tests/test_gpu_prefill.py", "tests/test_gpu_trace.py")


def test_two_cta_persistent_kernel_isolates_bad_sequences():
    if os.environ.get("PKV_PREFILL_LEAN") == "0":
        pytest.skip("this process already runs the two-CTA persistent kernel")
    _child({"PKV_PREFILL_LEAN": "0"},
           "tests/test_gpu_prefill_persistent.py::test_persistent_kernel_isolates_bad_sequences")


def test_persistent_kernel_isolates_bad_sequences():
    rs = np.random.RandomState(21)
    specs = [(int(rs.randint(0, 300)), int(rs.randint(20, 90))) for _ in range(90)]
    bk, seqs, m, q = build_step(21, specs, 4096, validate="device")
    n_items = sum((ql + 31) // 32 for _, ql in specs) * 8
    assert n_items > 2 * torch.cuda.get_device_properties(0).multi_processor_count  # persistent launch
    want = exact(bk, q, m, 0.125)
    # sequence 7: a page id outside the pool; sequence 40: last_page_len disagreeing with kv_len
    ip = m.kv_indptr.cpu().numpy()
    idx = m.kv_indices.clone()
    idx[int(ip[7]) + 1] = bk.num_blocks + 5
    lpl = m.kv_last_page_len.clone()
    lpl[40] = (int(lpl[40]) % 16) + 1 if int(lpl[40]) != 16 else 3
    bad = dataclasses.replace(m, kv_indices=idx, kv_last_page_len=lpl)
    out = torch.full((q.shape[0], 32, 64), 7.0, dtype=torch.float16, device="cuda:0")
    bk.attend(q.cuda(), 0, 0.125, bad, out=out)
    torch.cuda.synchronize()
    bits = int(bk._status.item())
    bk._status.zero_()
    assert bits & N.DEV_SLOT_OOB and bits & N.DEV_META_BAD, hex(bits)
    got = out.double().cpu().numpy()
    cu = m.cu_query_lens.cpu().numpy()
    rows = np.ones(q.shape[0], dtype=bool)
    assert (got[cu[7]:cu[8]] == 0).all(), "rows of the sequence with a bad page are not zero"
    assert (got[cu[40]:cu[41]] == 7.0).all(), "rows of the inconsistent sequence were written"
    rows[cu[7]:cu[8]] = False
    rows[cu[40]:cu[41]] = False
    err = np.abs(got[rows] - want[rows]).max()
    assert err <= 2e-3, f"other sequences off by {err}"
