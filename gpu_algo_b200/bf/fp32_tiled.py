"""Drop-in for bf/fp32_tiled.py (run_bf_fp32_tiled, bf/fp32_tiled.py:182-239).

The reference splits the database into tiles of ``tile_size`` rows, writes a
partial top-k per (query, tile) to HBM and merges them in a second kernel.
Here ``tile_size`` sets the number of database slices of the engine
(ceil(m / tile_size)); the per-slice results are merged on the device by the
merge kernel of ``bfk_merge``.  Output is sorted (the reference's is not,
bf/fp32_tiled.py:172-177; the set of results is the same).
"""
from __future__ import annotations

from .fp32 import _engine_attrs, _finish, _make_runner, _merge_report


def run_bf_fp32_tiled(Q_gpu, X_gpu, k: int, tile_size: int = 125_000, reps: int = 10) -> dict:
    if tile_size <= 0:
        raise ValueError("tile_size must be positive")
    m = X_gpu.shape[0]
    n_tiles = (m + tile_size - 1) // tile_size
    slices = max(1, min(n_tiles, 65535))
    Q, X, fn, out_ids, out_dists = _make_runner(Q_gpu, X_gpu, k, engine="direct", slices=slices)
    fn()
    block, smem, attrs = _engine_attrs(Q, X, k, "direct", slices, "tiled_partial")
    merge_smem, merge_attrs = _merge_report(Q, X, k, "direct", slices, "tiled_merge")
    ms, ids, dists = _finish(fn, out_ids, out_dists, reps)
    return {
        "ids": ids,
        "dists": dists,
        "ms": ms,
        "block": block,
        "tile_size": tile_size,
        "n_tiles": n_tiles,
        "partial_shared_mem_bytes": smem,
        "merge_shared_mem_bytes": merge_smem,
        "partial_kernel_attrs": attrs,
        "merge_kernel_attrs": merge_attrs,
    }
