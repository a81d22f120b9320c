"""
CPU ORACLE — TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's paged-KV hot path
(``serving/backends/paged_torch.py``, ``serving/scheduler/preemption.py``,
``serving/memory/block_table.py``), used as the checker for the CUDA path.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg (and its ``--impl reference`` arm) may import this package, and only to
check or to time the CPU baseline. The product (``llm_serving_layer_b200``)
never imports it and has no CPU fallback.

Pinning: ``tests/test_oracle_golden.py`` checks every function here against
golden vectors produced by running the reference's own code in the build
container (``tests/golden/make_golden.py``) and against the known-answer
scenarios of the reference's tests (``tests/test_paged_torch.py``,
``tests/test_copy_block.py``, ``tests/test_preemption.py``).
"""

from .paged_kv import (  # noqa: F401
    OraclePool,
    attend_exact,
    attend_reference,
    build_csr,
    last_page_len,
    rope,
    slot_for,
)
