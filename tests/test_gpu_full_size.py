"""The bench workload at full size: 10M unit rows x d=128, all 10,000 queries, k=100
(B200 only).

The oracle cannot check 10,000 queries against 10M rows in a test's time, so the
full result is checked through properties that do not depend on size, and a sample
of it exactly:
* every list is sorted by (distance, index), with distinct in-range ids;
* sampled entries carry the reference arithmetic's distance to their row, bit for bit;
* sampled queries' lists equal the oracle's exact top-k.
"""
import numpy as np
import pytest
import torch

from gpu_algo_b200 import data, engine
from oracle import oracle_knn, oracle_ref_dist

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def unit10m():
    X, Q = data.workload_arrays("unit-10m")
    Xd, Qd = torch.from_numpy(X).cuda(), torch.from_numpy(Q).cuda()
    d_, i_ = engine.search(Qd, Xd, 100)
    torch.cuda.synchronize()
    return X, Q, d_.cpu().numpy(), i_.cpu().numpy()


def test_full_size_lists_are_sorted_and_distinct(unit10m):
    X, Q, dd, ii = unit10m
    m = X.shape[0]
    assert dd.shape == (Q.shape[0], 100) and ii.dtype == np.int32
    assert ((ii >= 0) & (ii < m)).all()
    s = np.sort(ii, axis=1)
    assert (s[:, 1:] != s[:, :-1]).all()
    # ascending by (distance, index)
    assert ((dd[:, 1:] > dd[:, :-1]) | ((dd[:, 1:] == dd[:, :-1]) & (ii[:, 1:] > ii[:, :-1]))).all()


def test_full_size_sampled_distances_and_lists_are_exact(unit10m):
    X, Q, dd, ii = unit10m
    rng = np.random.Generator(np.random.PCG64(41))
    for q, r in zip(rng.integers(0, Q.shape[0], 256), rng.integers(0, 100, 256)):
        assert dd[q, r] == oracle_ref_dist(Q[q], X[ii[q, r]])
    sel = rng.choice(Q.shape[0], size=8, replace=False)
    ed, ei = oracle_knn(Q[sel], X, 100)
    np.testing.assert_array_equal(ii[sel], ei)
    np.testing.assert_array_equal(dd[sel], ed)


def test_full_size_every_query_equals_the_simt_engine(unit10m):
    """All 10,000 lists against the exact SIMT engine, an independent full scan with the
    reference arithmetic (pinned to the oracle by the parity tests): distances and ids
    equal, every query."""
    X, Q, dd, ii = unit10m
    Xd, Qd = torch.from_numpy(X).cuda(), torch.from_numpy(Q).cuda()
    sd, si = engine.search(Qd, Xd, 100, engine="direct")
    torch.cuda.synchronize()
    np.testing.assert_array_equal(sd.cpu().numpy(), dd)
    np.testing.assert_array_equal(si.cpu().numpy(), ii)
