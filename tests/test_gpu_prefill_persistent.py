"""
The two tcgen05 prefill kernels against each other's paths and the oracle.

Launches of more than one wave of CTAs (more than two tiles x KV heads per SM)
run the persistent kernel, smaller ones one CTA per tile. The environment
variable ``PKV_PREFILL_PERSISTENT`` (read once per process) moves the line:
``2`` sends every launch to the persistent kernel, ``0`` none. Here the whole
prefill suite and the reference-scheduler trace replay run again in child
processes under both settings, so each kernel meets every case (chunks after
long prefixes, tile and page edges, every GQA group size, bf16, NaN-poisoned
page tails, radix sharing with copy-on-write, mixed batches), and a large
batch — persistent CTAs walking several tiles each — with one sequence whose
page table points outside the pool and one whose lengths disagree checks that
only those sequences are affected: the first gets zero rows and
``PKV_DEV_SLOT_OOB``, the second no rows written and ``PKV_DEV_META_BAD``, and
every other row is within the fp16 tolerance of the float64 evaluation.
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


@pytest.mark.parametrize("mode", ["2", "0"])
def test_prefill_suite_under_each_kernel(mode):
    env = dict(os.environ, PKV_PREFILL_PERSISTENT=mode)
    r = subprocess.run([sys.executable, "-m", "pytest", "-x", "-q", "-m", "gpu", "-p", "no:cacheprovider",
                        "tests/test_gpu_prefill.py", "tests/test_gpu_trace.py"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


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
