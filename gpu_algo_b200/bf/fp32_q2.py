"""Drop-in for bf/fp32_q2.py (run_bf_fp32_q2, bf/fp32_q2.py:140-177).

The reference shares each database row between two queries of a block; the
B200 engines share every database tile between whole query tiles, so this
runner calls the same engine.  Output is sorted (the reference's q2 output is
unsorted, bf/fp32_q2.py:101-135; the set of results is the same).
"""
from __future__ import annotations

from .fp32 import _engine_attrs, _finish, _make_runner


def run_bf_fp32_q2(Q_gpu, X_gpu, k: int, reps: int = 10) -> dict:
    Q, X, fn, out_ids, out_dists = _make_runner(Q_gpu, X_gpu, k)
    fn()
    block, smem, attrs = _engine_attrs(Q, X, k, "auto", 0, "two_queries_per_block")
    ms, ids, dists = _finish(fn, out_ids, out_dists, reps)
    return {
        "ids": ids,
        "dists": dists,
        "ms": ms,
        "block": block,
        "shared_mem_bytes": smem,
        "kernel_attrs": attrs,
    }
