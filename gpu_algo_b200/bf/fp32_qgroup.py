"""Drop-in for bf/fp32_qgroup.py (run_bf_fp32_qgroup, bf/fp32_qgroup.py:228-291).

The reference keeps ``qpb`` queries per block so each database element is
loaded once per group (bf/fp32_qgroup.py:93-102).  The B200 engines take that
idea to whole query tiles (32 queries per SIMT block, 128 per tensor-core
tile), so ``qpb`` is accepted and reported but does not change the launch.
"""
from __future__ import annotations

from .fp32 import _engine_attrs, _finish, _make_runner, _merge_report


def choose_qgroup_block(k: int, d: int, qpb: int) -> int:
    """The reference's heuristic (bf/fp32_qgroup.py:217-225), kept for callers."""
    limit = 47 * 1024
    reg_cap = max(32, 65536 // max(64, qpb * (d + k) + 10))
    for b in [128, 64, 32]:
        if b > reg_cap:
            continue
        if (qpb * d + 2 * b * k) * 4 < limit:
            return b
    return 32


def run_bf_fp32_qgroup(Q_gpu, X_gpu, k: int, qpb: int, reps: int = 8) -> dict:
    if qpb <= 0:
        raise ValueError("qpb must be positive")
    m = X_gpu.shape[0]
    n_tiles = qpb
    tile_size = (m + n_tiles - 1) // n_tiles
    Q, X, fn, out_ids, out_dists = _make_runner(Q_gpu, X_gpu, k)
    fn()
    block, smem, attrs = _engine_attrs(Q, X, k, "auto", 0, f"q{qpb}")
    merge_smem, merge_attrs = _merge_report(Q, X, k, "auto", 0, "qgroup_merge")
    ms, ids, dists = _finish(fn, out_ids, out_dists, reps)
    return {
        "ids": ids,
        "dists": dists,
        "ms": ms,
        "block": block,
        "qpb": qpb,
        "qpb_note": "qpb is reported only: the engine's own query tiles (32 or 128 queries) "
                    "set the launch, so it does not change the work or the results",
        "tile_size": tile_size,
        "n_tiles": n_tiles,
        "partial_shared_mem_bytes": smem,
        "merge_shared_mem_bytes": merge_smem,
        "partial_kernel_attrs": attrs,
        "merge_kernel_attrs": merge_attrs,
    }
