"""Generate the golden fixtures in tests/golden/ from the C oracle.

    python tests/golden/make_golden.py

Writes:
  plumbing_k10.npz   exact top-10 of the plumbing workload (N=65,536 x d=128
                     N(0,1) seed 0, Q=1,024 seed 1) -- every query;
  edges.npz          expected outputs of small edge cases (m < k, exact ties
                     from duplicate rows, a query equal to a row, ragged d,
                     k in {1,2,31,32,33,100,256}, a NaN row, a single query,
                     integer-valued data, distances that overflow to +inf,
                     subnormal distances); their inputs come from
                     ``edge_cases()`` (seeded) and are pinned by SHA-256;
  inputs.json        SHA-256 of the generated inputs, to catch generator drift.

The inputs are regenerated from their seeds by the tests; only the expected
outputs (and the small edge-case inputs) are stored.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from gpu_algo_b200 import data  # noqa: E402
from oracle import oracle_knn  # noqa: E402


def edge_cases() -> dict[str, tuple[np.ndarray, np.ndarray, int]]:
    """name -> (Q, X, k); deterministic."""
    rng = np.random.Generator(np.random.PCG64(12345))
    cases = {}
    # fewer rows than k: padding
    cases["m_lt_k"] = (rng.standard_normal((9, 16), dtype=np.float32),
                       rng.standard_normal((5, 16), dtype=np.float32), 8)
    # exact ties: every row appears 3 times
    base = rng.standard_normal((40, 24), dtype=np.float32)
    X = np.repeat(base, 3, axis=0)
    perm = rng.permutation(X.shape[0])
    cases["ties"] = (rng.standard_normal((17, 24), dtype=np.float32), X[perm].copy(), 10)
    # queries equal to rows: distance 0 must come first
    X = rng.standard_normal((500, 32), dtype=np.float32)
    cases["self_match"] = (X[[3, 77, 499, 250]].copy(), X, 5)
    # ragged dimensions
    for d in (1, 7, 33, 130):
        cases[f"ragged_d{d}"] = (rng.standard_normal((37, d), dtype=np.float32),
                                 rng.standard_normal((1000, d), dtype=np.float32), 10)
    # k sweep over odd and boundary values
    Xk = rng.standard_normal((3000, 64), dtype=np.float32)
    Qk = rng.standard_normal((70, 64), dtype=np.float32)
    for k in (1, 2, 31, 32, 33, 100, 256):
        cases[f"k{k}"] = (Qk, Xk, k)
    # a NaN row is never returned
    X = rng.standard_normal((300, 16), dtype=np.float32)
    X[17, 5] = np.nan
    cases["nan_row"] = (rng.standard_normal((11, 16), dtype=np.float32), X, 300)
    # one query
    cases["single_query"] = (rng.standard_normal((1, 128), dtype=np.float32),
                             rng.standard_normal((20000, 128), dtype=np.float32), 10)
    # integer-valued data: many exact distance ties across different rows
    cases["int_grid"] = (rng.integers(-2, 3, size=(50, 8)).astype(np.float32),
                         rng.integers(-2, 3, size=(4000, 8)).astype(np.float32), 20)
    # norms of 1.2e19: finite squared norms, distances that overflow to +inf; with k = m
    # the rows at +inf come last, ordered by index
    def at_norm(a, norm):
        return (a / np.linalg.norm(a, axis=1, keepdims=True) * np.float32(norm)).astype(np.float32)
    cases["inf_dists"] = (at_norm(rng.standard_normal((11, 16), dtype=np.float32), 1.2e19),
                          at_norm(rng.standard_normal((300, 16), dtype=np.float32), 1.2e19), 300)
    # norms near 1e-19: subnormal distances
    cases["tiny_norms"] = ((rng.standard_normal((37, 32)) * 1e-20).astype(np.float32),
                           (rng.standard_normal((3000, 32)) * 1e-20).astype(np.float32), 10)
    return cases


def main() -> int:
    X, Q = data.workload_arrays("plumbing")
    d_, i_ = oracle_knn(Q, X, 10)
    np.savez_compressed(os.path.join(HERE, "plumbing_k10.npz"), dists=d_, ids=i_)
    shas = {"plumbing.X": data.sha256(X), "plumbing.Q": data.sha256(Q)}
    # small prefixes of the large workloads, to pin the generators
    for name in ("mixture-k-sweep", "unit-10m", "highdim-960", "stream-100m", "published-d8"):
        Xs, Qs = data.workload_arrays(name, n_rows=2048, n_queries=64)
        shas[f"{name}.X[:2048]"] = data.sha256(Xs)
        shas[f"{name}.Q[:64]"] = data.sha256(Qs)
    with open(os.path.join(HERE, "inputs.json"), "w") as f:
        json.dump(shas, f, indent=1, sort_keys=True)
    arrays = {}
    for name, (Qe, Xe, k) in edge_cases().items():
        de, ie = oracle_knn(Qe, Xe, k)
        shas[f"edge.{name}.Q"] = data.sha256(Qe)
        shas[f"edge.{name}.X"] = data.sha256(Xe)
        arrays[f"{name}.dists"] = de
        arrays[f"{name}.ids"] = ie
    np.savez_compressed(os.path.join(HERE, "edges.npz"), **arrays)
    with open(os.path.join(HERE, "inputs.json"), "w") as f:
        json.dump(shas, f, indent=1, sort_keys=True)
    print("wrote plumbing_k10.npz, edges.npz, inputs.json")
    return 0


if __name__ == "__main__":
    sys.exit(main())
