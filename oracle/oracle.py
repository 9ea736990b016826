"""ctypes binding to the C oracle, the NumPy CPU baseline, and the parity rule.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "knn_oracle.c")
LIB = os.path.join(HERE, "libknn_oracle.so")
PAD_DIST = np.float32(3.402823e38)

_lock = threading.Lock()
_lib = None


def build_oracle(force: bool = False) -> str:
    """Compile ``knn_oracle.c`` into ``oracle/libknn_oracle.so``.

    ``-ffp-contract=off`` keeps gcc from fusing anything the C source does not
    fuse explicitly; the only fused operation is the explicit ``fmaf`` that
    mirrors the reference kernel's contracted ``dist += dif*dif``.
    """
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cmd = [
        "gcc", "-O3", "-mavx2", "-mfma", "-ffp-contract=off", "-fno-fast-math",
        "-fopenmp", "-shared", "-fPIC", SRC, "-o", LIB + ".tmp", "-lm",
    ]
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


def _load():
    global _lib
    with _lock:
        if _lib is None:
            build_oracle()
            lib = ctypes.CDLL(LIB)
            f32p = ctypes.POINTER(ctypes.c_float)
            i32p = ctypes.POINTER(ctypes.c_int32)
            lib.oracle_ref_dist.restype = ctypes.c_float
            lib.oracle_ref_dist.argtypes = [f32p, f32p, ctypes.c_int32]
            lib.oracle_all_dists.restype = None
            lib.oracle_all_dists.argtypes = [f32p, ctypes.c_int64, f32p, ctypes.c_int64,
                                             ctypes.c_int32, f32p]
            lib.oracle_knn.restype = ctypes.c_int
            lib.oracle_knn.argtypes = [f32p, ctypes.c_int64, f32p, ctypes.c_int64, ctypes.c_int32,
                                       ctypes.c_int32, ctypes.c_int64, f32p, i32p, ctypes.c_int32]
            lib.oracle_merge.restype = ctypes.c_int
            lib.oracle_merge.argtypes = [f32p, i32p, ctypes.c_int64, ctypes.c_int32,
                                         ctypes.c_int32, f32p, i32p]
            _lib = lib
    return _lib


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _i32(a):
    a = np.ascontiguousarray(a, dtype=np.int32)
    return a, a.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))


def oracle_ref_dist(q: np.ndarray, x: np.ndarray) -> np.float32:
    """One distance in the reference kernel's operation order (bf/fp32.py:80)."""
    q, qp = _f32(q)
    x, xp = _f32(x)
    return np.float32(_load().oracle_ref_dist(qp, xp, q.shape[-1]))


def oracle_all_dists(Q: np.ndarray, X: np.ndarray) -> np.ndarray:
    Q, qp = _f32(Q)
    X, xp = _f32(X)
    out = np.empty((Q.shape[0], X.shape[0]), np.float32)
    _load().oracle_all_dists(qp, Q.shape[0], xp, X.shape[0], Q.shape[1],
                             out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return out


def oracle_knn(Q: np.ndarray, X: np.ndarray, k: int, id_offset: int = 0,
               nthreads: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """Exact top-k (distances ascending, ties by lower index), padded (3.4e38, -1)."""
    Q, qp = _f32(Q)
    X, xp = _f32(X)
    if Q.ndim != 2 or X.ndim != 2 or (X.shape[0] and Q.shape[1] != X.shape[1]):
        raise ValueError("Q (n,d) and X (m,d) must share d")
    n, d = Q.shape
    m = X.shape[0]
    out_d = np.empty((n, k), np.float32)
    out_i = np.empty((n, k), np.int32)
    rc = _load().oracle_knn(qp, n, xp, m, d, k, id_offset,
                            out_d.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                            out_i.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), nthreads)
    if rc != 0:
        raise ValueError("oracle_knn: bad arguments")
    return out_d, out_i


def oracle_merge(cand_d: np.ndarray, cand_i: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """Merge sorted lists laid out (lists, n, k) into the k best per query."""
    cand_d, dp = _f32(cand_d)
    cand_i, ip = _i32(cand_i)
    lists, n, kk = cand_d.shape
    if kk != k:
        raise ValueError("list length must equal k")
    out_d = np.empty((n, k), np.float32)
    out_i = np.empty((n, k), np.int32)
    rc = _load().oracle_merge(dp, ip, n, lists, k,
                              out_d.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                              out_i.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)))
    if rc != 0:
        raise ValueError("oracle_merge: bad arguments")
    return out_d, out_i


def numpy_knn(Q: np.ndarray, X: np.ndarray, k: int, qblock: int = 256,
              rblock: int = 1 << 20) -> tuple[np.ndarray, np.ndarray]:
    """Blocked CPU brute force with OpenBLAS sgemm (the timed CPU baseline).

    ||q||^2 + ||x||^2 - 2 q.X^T per (query block, row block), argpartition,
    a running top-k per query, then a sort by (distance, index).  It is not
    bit-faithful to the reference's direct differences (the C oracle is); it
    is the fast CPU comparison point the workloads name.
    """
    Q = np.ascontiguousarray(Q, np.float32)
    X = np.ascontiguousarray(X, np.float32)
    n = Q.shape[0]
    m = X.shape[0]
    out_d = np.full((n, k), PAD_DIST, np.float32)
    out_i = np.full((n, k), -1, np.int32)
    for q0 in range(0, n, qblock):
        qb = Q[q0:q0 + qblock]
        qn = np.einsum("ij,ij->i", qb, qb)[:, None]
        best_d = np.empty((qb.shape[0], 0), np.float32)
        best_i = np.empty((qb.shape[0], 0), np.int64)
        for r0 in range(0, m, rblock):
            xb = X[r0:r0 + rblock]
            dist = np.einsum("ij,ij->i", xb, xb)[None, :] - 2.0 * (qb @ xb.T)
            dist += qn
            kk = min(k, xb.shape[0])
            if kk < xb.shape[0]:
                part = np.argpartition(dist, kk - 1, axis=1)[:, :kk]
            else:
                part = np.broadcast_to(np.arange(xb.shape[0]), dist.shape)
            cd = np.concatenate([best_d, np.take_along_axis(dist, part, axis=1)], axis=1)
            ci = np.concatenate([best_i, part + r0], axis=1)
            order = np.lexsort((ci, cd), axis=1)[:, :k]
            best_d = np.take_along_axis(cd, order, axis=1)
            best_i = np.take_along_axis(ci, order, axis=1)
        kk = best_d.shape[1]
        out_d[q0:q0 + qblock, :kk] = best_d
        out_i[q0:q0 + qblock, :kk] = best_i
    return out_d, out_i


def check_parity(got_d: np.ndarray, got_i: np.ndarray, ref_d: np.ndarray, ref_i: np.ndarray,
                 k: int, rel_tie: float = 1e-5, rel_dist: float = 1e-4,
                 abs_floor: float = 1e-6) -> list[str]:
    """The acceptance rule for results against the oracle.

    ``ref_d``/``ref_i`` hold the oracle's top-(k+1) (or top-k when the
    database has only k rows).  Per query:
      * if d[k] - d[k-1] >= rel_tie * d[k-1] the index sets must be equal;
      * otherwise every oracle index with d < d[k-1]*(1-rel_tie) must be
        present, and every returned index must have an oracle distance
        <= d[k-1]*(1+rel_tie);
      * sorted distances must agree within rel_dist relative (abs_floor
        absolute near zero).
    Returns a list of human-readable failures (empty == pass).
    """
    fails: list[str] = []
    n = got_d.shape[0]
    for qi in range(n):
        gi = got_i[qi, :k]
        gd = got_d[qi, :k]
        ri = ref_i[qi]
        rd = ref_d[qi]
        valid = ri[:k] >= 0
        nk = int(valid.sum())
        ref_set = set(int(v) for v in ri[:k][valid])
        got_set = set(int(v) for v in gi[gi >= 0])
        if nk == 0:
            if got_set:
                fails.append(f"q{qi}: expected no results, got {len(got_set)}")
            continue
        dk = float(rd[nk - 1])
        has_next = ref_d.shape[1] > k and ri[k] >= 0
        gap_ok = (not has_next) or (float(rd[k]) - dk >= rel_tie * abs(dk))
        if gap_ok:
            if ref_set != got_set:
                fails.append(f"q{qi}: index sets differ ({len(ref_set ^ got_set)} symmetric)")
        else:
            lo = dk * (1 - rel_tie)
            must = set(int(v) for v, dd in zip(ri[:k], rd[:k]) if v >= 0 and dd < lo)
            if not must <= got_set:
                fails.append(f"q{qi}: missing strict neighbours {sorted(must - got_set)[:5]}")
            if len(got_set) != nk:
                fails.append(f"q{qi}: returned {len(got_set)} valid ids, expected {nk}")
            if np.any(gd[gi >= 0] > dk * (1 + rel_tie) + abs_floor):
                fails.append(f"q{qi}: a returned distance exceeds the k-th by > {rel_tie}")
        gdv = gd[gi >= 0]
        rdv = rd[:k][valid]
        if gdv.shape != rdv.shape or not np.all(
                np.abs(gdv - rdv) <= rel_dist * np.abs(rdv) + abs_floor):
            fails.append(f"q{qi}: distances differ beyond {rel_dist} relative")
    return fails
