"""CPU oracle for exact brute-force k-NN -- TEST INFRASTRUCTURE ONLY.

This package is the checker.  Only ``tests/``, ``__graft_entry__.smoke()`` and
the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it,
and only to check or to time the CPU baseline.  The product path
(``gpu_algo_b200``) never imports it and has no CPU fallback.

Contents
--------
``knn_oracle.c``      plain-C restatement of the reference kernels' arithmetic
                      (bf/fp32.py:74-82), bit-faithful, OpenMP over queries.
``oracle.py``         ctypes binding, NumPy BLAS CPU baseline, parity checker.
``build_ref.py``      compiles the reference's own CUDA kernel strings (read
                      from the reference checkout) into ``oracle/_ref/`` for the
                      GPU-side pin of the oracle.
"""
from .oracle import (  # noqa: F401
    build_oracle,
    oracle_knn,
    oracle_merge,
    oracle_all_dists,
    oracle_ref_dist,
    numpy_knn,
    check_parity,
    PAD_DIST,
)
