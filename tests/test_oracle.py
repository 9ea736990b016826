"""The CPU oracle against exact arithmetic, the golden fixtures and itself."""
import json
import os
from fractions import Fraction

import numpy as np
import pytest

from gpu_algo_b200 import data
from oracle import (check_parity, numpy_knn, oracle_all_dists, oracle_knn, oracle_merge,
                    oracle_ref_dist)

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _round_f32(x: Fraction) -> np.float32:
    """Correctly rounded (nearest-even) float32 of an exact rational."""
    f = np.float32(float(x))
    lo = f if Fraction(float(f)) <= x else np.nextafter(f, np.float32(-np.inf))
    hi = np.nextafter(lo, np.float32(np.inf))
    dl, dh = x - Fraction(float(lo)), Fraction(float(hi)) - x
    if dl < dh:
        return lo
    if dh < dl:
        return hi
    return lo if (lo.view(np.uint32) & 1) == 0 else hi


def _exact_ref(q, x):
    """bf/fp32.py:80 with fmad contraction: dif = fl(q-x); acc = fl(dif*dif + acc)."""
    acc = np.float32(0)
    for a, b in zip(q, x):
        dif = np.float32(a) - np.float32(b)  # one float32 rounding
        acc = _round_f32(Fraction(float(dif)) ** 2 + Fraction(float(acc)))
    return acc


@pytest.mark.parametrize("d", [1, 7, 33, 128])
def test_ref_dist_is_fused_sequential(d):
    rng = np.random.Generator(np.random.PCG64(d))
    for _ in range(20):
        q = rng.standard_normal(d, dtype=np.float32) * np.float32(rng.uniform(0.01, 100))
        x = rng.standard_normal(d, dtype=np.float32)
        assert oracle_ref_dist(q, x) == _exact_ref(q, x)


def test_knn_matches_all_dists_sort():
    rng = np.random.Generator(np.random.PCG64(7))
    X = rng.integers(-3, 4, size=(700, 5)).astype(np.float32)  # many exact ties
    Q = rng.integers(-3, 4, size=(23, 5)).astype(np.float32)
    k = 17
    D = oracle_all_dists(Q, X)
    got_d, got_i = oracle_knn(Q, X, k)
    for qi in range(Q.shape[0]):
        order = np.lexsort((np.arange(X.shape[0]), D[qi]))[:k]
        np.testing.assert_array_equal(got_i[qi], order)
        np.testing.assert_array_equal(got_d[qi], D[qi, order])


def test_inputs_match_pinned_hashes():
    with open(os.path.join(GOLDEN, "inputs.json")) as f:
        shas = json.load(f)
    X, Q = data.workload_arrays("plumbing")
    assert data.sha256(X) == shas["plumbing.X"]
    assert data.sha256(Q) == shas["plumbing.Q"]
    for name in ("mixture-k-sweep", "unit-10m", "highdim-960", "stream-100m", "published-d8"):
        Xs, Qs = data.workload_arrays(name, n_rows=2048, n_queries=64)
        assert data.sha256(Xs) == shas[f"{name}.X[:2048]"]
        assert data.sha256(Qs) == shas[f"{name}.Q[:64]"]


def test_shard_generation_is_range_independent():
    a = data.generate("normal", 8, 12, data.CHUNK_ROWS - 3, data.CHUNK_ROWS + 3)
    b = data.generate("normal", 8, 12, 0, data.CHUNK_ROWS + 3)
    np.testing.assert_array_equal(a, b[-6:])


def test_oracle_reproduces_plumbing_golden(plumbing):
    X, Q, gd, gi = plumbing
    d_, i_ = oracle_knn(Q[:256], X, 10)
    np.testing.assert_array_equal(i_, gi[:256])
    np.testing.assert_array_equal(d_, gd[:256])


def test_oracle_reproduces_edge_goldens(edges):
    with open(os.path.join(GOLDEN, "inputs.json")) as f:
        shas = json.load(f)
    for name, (Q, X, k, gd, gi) in edges.items():
        assert data.sha256(Q) == shas[f"edge.{name}.Q"], name
        assert data.sha256(X) == shas[f"edge.{name}.X"], name
        d_, i_ = oracle_knn(Q, X, k)
        np.testing.assert_array_equal(i_, gi, err_msg=name)
        np.testing.assert_array_equal(d_, gd, err_msg=name)


def test_edge_semantics(edges):
    Q, X, k, gd, gi = edges["m_lt_k"]
    assert (gi[:, 5:] == -1).all() and (gd[:, 5:] == np.float32(3.402823e38)).all()
    Q, X, k, gd, gi = edges["self_match"]
    assert (gd[:, 0] == 0).all() and list(gi[:, 0]) == [3, 77, 499, 250]
    Q, X, k, gd, gi = edges["nan_row"]
    assert 17 not in set(gi.ravel()) and (gi[:, -1] == -1).all()
    Q, X, k, gd, gi = edges["ties"]
    for qi in range(Q.shape[0]):  # equal distances are ordered by index
        for a in range(k - 1):
            assert (gd[qi, a], gi[qi, a]) < (gd[qi, a + 1], gi[qi, a + 1])
    # rows at +inf are returned (k = m), last, by index
    Q, X, k, gd, gi = edges["inf_dists"]
    assert np.isinf(gd).any() and (gi >= 0).all()
    for qi in range(Q.shape[0]):
        inf = np.isinf(gd[qi])
        assert (np.diff(inf.astype(int)) >= 0).all()  # after every finite distance
        assert (np.diff(gi[qi][inf]) > 0).all()
    # subnormal distances keep their order
    Q, X, k, gd, gi = edges["tiny_norms"]
    assert (gd < np.finfo(np.float32).tiny).all() and (gd > 0).all()
    assert (np.diff(gd, axis=1) >= 0).all()


def test_merge_of_shards_equals_whole(plumbing):
    X, Q, gd, gi = plumbing
    k = 10
    parts_d, parts_i = [], []
    bounds = [0, 10_000, 30_001, 65_536]
    for a, b in zip(bounds[:-1], bounds[1:]):
        d_, i_ = oracle_knn(Q[:128], X[a:b], k, id_offset=a)
        parts_d.append(d_)
        parts_i.append(i_)
    md, mi = oracle_merge(np.stack(parts_d), np.stack(parts_i), k)
    np.testing.assert_array_equal(mi, gi[:128])
    np.testing.assert_array_equal(md, gd[:128])


def test_numpy_baseline_meets_parity_rule(plumbing):
    X, Q, gd, gi = plumbing
    k = 10
    nd, ni = numpy_knn(Q[:200], X, k)
    rd, ri = oracle_knn(Q[:200], X, k + 1)
    assert check_parity(nd, ni, rd, ri, k) == []


def test_parity_rule_catches_planted_mistakes(plumbing):
    X, Q, gd, gi = plumbing
    k = 10
    rd, ri = oracle_knn(Q[:50], X, k + 1)
    good_d, good_i = rd[:, :k].copy(), ri[:, :k].copy()
    assert check_parity(good_d, good_i, rd, ri, k) == []
    bad_i = good_i.copy()
    bad_i[3, 4] = 65_535 if bad_i[3, 4] != 65_535 else 0  # a wrong neighbour
    assert check_parity(good_d, bad_i, rd, ri, k)
    bad_d = good_d.copy()
    bad_d[7, 2] *= np.float32(1.001)  # a distance off by 1e-3
    assert check_parity(bad_d, good_i, rd, ri, k)
