"""Seeded synthetic inputs for the exact k-NN workloads.

The reference draws its database and then its queries from one CuPy generator
(bf/bench_fp32.py:35-37, bf/bench_fp32_variant_repeat_over_n.py:97-106).  That
stream cannot be reproduced without CuPy, and the workloads here name one seed
per array, so every array comes from NumPy's PCG64 instead:

* rows are generated in fixed chunks of ``CHUNK_ROWS`` rows, chunk ``c`` of
  seed ``s`` drawn from ``SeedSequence([s, c + 1])``, so any row range (a
  shard of a multi-GPU run) is generated without touching the other rows and
  the data does not depend on the GPU count;
* ``normal``    -- i.i.d. N(0, 1) float32;
* ``unit``      -- i.i.d. U[0, 1) float32, each row divided by its L2 norm
  (computed in float64, then rounded once to float32);
* ``mixture``   -- 256 centres drawn once from ``SeedSequence([centre_seed, 0])``
  as 2 * N(0, 1) (variance 4), each row = centre[label] + N(0, 1) with a uniform
  label; queries reuse the database's centres (``centre_seed``) with labels and
  noise from their own seed.
"""
from __future__ import annotations

import hashlib
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

CHUNK_ROWS = 1 << 20
MIXTURE_COMPONENTS = 256


def _chunk_rng(seed: int, chunk: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, chunk + 1])))


def _centres(centre_seed: int, d: int) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([centre_seed, 0])))
    return (rng.standard_normal((MIXTURE_COMPONENTS, d), dtype=np.float32) * np.float32(2.0))


def _gen_chunk(kind: str, seed: int, chunk: int, rows: int, d: int,
               centre_seed: int | None) -> np.ndarray:
    rng = _chunk_rng(seed, chunk)
    if kind == "normal":
        return rng.standard_normal((rows, d), dtype=np.float32)
    if kind == "unit":
        x = rng.random((rows, d), dtype=np.float32)
        nrm = np.sqrt(np.einsum("ij,ij->i", x.astype(np.float64), x.astype(np.float64)))
        nrm[nrm == 0] = 1.0
        return (x / nrm[:, None]).astype(np.float32)
    if kind == "mixture":
        cs = seed if centre_seed is None else centre_seed
        centres = _centres(cs, d)
        # labels and noise come from separate streams so that a prefix of a
        # chunk does not depend on how many rows were asked for
        lab_rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, chunk + 1, 1])))
        labels = lab_rng.integers(0, MIXTURE_COMPONENTS, size=rows)
        noise = rng.standard_normal((rows, d), dtype=np.float32)
        return centres[labels] + noise
    raise ValueError(f"unknown distribution {kind!r}")


def generate(kind: str, seed: int, d: int, row_begin: int, row_end: int,
             centre_seed: int | None = None, out: np.ndarray | None = None,
             threads: int | None = None) -> np.ndarray:
    """Rows [row_begin, row_end) of the seeded array (float32, C-contiguous)."""
    rows = row_end - row_begin
    if out is None:
        out = np.empty((rows, d), np.float32)
    pieces = []  # (chunk, lo, hi, pos): rows [lo, hi) of chunk land at out[pos:]
    pos = 0
    c = row_begin // CHUNK_ROWS
    while pos < rows:
        c0 = c * CHUNK_ROWS
        lo = row_begin + pos - c0
        hi = min(CHUNK_ROWS, row_end - c0)
        pieces.append((c, lo, hi, pos))
        pos += hi - lo
        c += 1

    def one(piece):
        c, lo, hi, pos = piece
        # every generator consumes its stream row by row, so the first `hi` rows
        # of a chunk are the same whatever range was asked for
        chunk = _gen_chunk(kind, seed, c, hi, d, centre_seed)
        out[pos:pos + (hi - lo)] = chunk[lo:hi]

    nthreads = threads if threads is not None else min(len(pieces), os.cpu_count() or 1, 16)
    if nthreads <= 1 or len(pieces) == 1:
        for p in pieces:
            one(p)
    else:
        with ThreadPoolExecutor(nthreads) as ex:
            list(ex.map(one, pieces))
    return out


def sha256(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# The five workloads: (database kind, db seed, queries kind, query seed, N, Q, d, ks)
WORKLOADS = {
    "plumbing": dict(kind="normal", db_seed=0, q_seed=1, N=65_536, Q=1_024, d=128, ks=(10,)),
    "mixture-k-sweep": dict(kind="mixture", db_seed=2, q_seed=3, N=1_000_000, Q=10_000, d=128,
                            ks=(1, 10, 32, 100, 256)),
    "unit-10m": dict(kind="unit", db_seed=4, q_seed=5, N=10_000_000, Q=10_000, d=128, ks=(100,)),
    "highdim-960": dict(kind="normal", db_seed=6, q_seed=7, N=2_000_000, Q=1_000, d=960, ks=(100,)),
    "stream-100m": dict(kind="normal", db_seed=8, q_seed=9, N=100_000_000, Q=128, d=96, ks=(10,)),
    # the shape of the reference's only published results (1M rows, d=8, k=1, up to 128k
    # queries, Gaussian data); the seeds are this package's own
    "published-d8": dict(kind="normal", db_seed=10, q_seed=11, N=1_000_000, Q=128_000, d=8, ks=(1,)),
}


def workload_arrays(name: str, n_rows: int | None = None, n_queries: int | None = None,
                    row_begin: int = 0):
    """(database rows, queries) for a named workload; optionally truncated."""
    w = WORKLOADS[name]
    N = w["N"] if n_rows is None else n_rows
    Qn = w["Q"] if n_queries is None else n_queries
    cs = w["db_seed"] if w["kind"] == "mixture" else None
    X = generate(w["kind"], w["db_seed"], w["d"], row_begin, row_begin + N, centre_seed=cs)
    Q = generate(w["kind"], w["q_seed"], w["d"], 0, Qn, centre_seed=cs)
    return X, Q
