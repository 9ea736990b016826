"""Drop-in for bf/fp32_heap.py (run_bf_fp32_heap, bf/fp32_heap.py:149-177).

The reference's binary max-heap variant returns the same exact top-k as the
baseline; here it runs the same B200 engine.
"""
from __future__ import annotations

from .fp32 import _engine_attrs, _finish, _make_runner


def run_bf_fp32_heap(Q_gpu, X_gpu, k: int, reps: int = 10) -> dict:
    Q, X, fn, out_ids, out_dists = _make_runner(Q_gpu, X_gpu, k)
    fn()
    block, smem, attrs = _engine_attrs(Q, X, k, "auto", 0, "true_max_heap")
    ms, ids, dists = _finish(fn, out_ids, out_dists, reps)
    return {
        "ids": ids,
        "dists": dists,
        "ms": ms,
        "block": block,
        "shared_mem_bytes": smem,
        "kernel_attrs": attrs,
    }
