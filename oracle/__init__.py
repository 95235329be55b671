"""CPU oracle for the paged decode-attention path -- TEST INFRASTRUCTURE ONLY.

This package restates, in NumPy, the reference project's CPU model of paged
single-query attention (``src/paged_decode/reference.py``), its split-KV
protocols (``kernels.py``, ``matched_splitkv.py``) and its static partition
plan (``splitkv_plan.py``).  Every function cites the reference file:line it
follows.

Who may use it: ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
``cpu_baseline`` leg / ``--impl reference`` arm, and only as the checker or
the timed CPU baseline.  The product package (``paged-decode-lab_b200/``)
never imports it; the CUDA path fails loudly instead of falling back here.

Parity is pinned: ``tests/test_oracle_golden.py`` checks this restatement
against golden vectors that ``tests/golden/make_golden.py`` produced by
importing the reference's own NumPy code, and against the reference's
known-answer plan fixtures (``tests/test_splitkv_plan.py:7-30``).
"""
from .reference import (  # noqa: F401
    bf16_bits, bits_to_f32, round_bf16,
    validate_metadata, gather_kv, dense_reference, partial, merge_partials,
    streaming_reference, partition_bounds, normalized_partitions, lse_merge,
    unnormalized_partitions, merge_unnormalized, matched_reference, score_magnitudes,
    balanced_span,
)
from .plan import OraclePlan, make_splitkv_plan, spec_geometry  # noqa: F401
