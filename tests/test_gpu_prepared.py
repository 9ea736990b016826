"""Prepared databases (bfk_prepare / bfk_search_prepared), B200 only.

A search over prepared rows must return exactly what the search over the raw
rows returns (the oracle's lists), before and after the buffer's bytes go to
a file and back; a buffer made for other rows is rejected.
"""
import numpy as np
import pytest
import torch

from gpu_algo_b200 import _lib, engine
from oracle import oracle_knn

pytestmark = pytest.mark.gpu


def _data(m, n, d, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    return (rng.standard_normal((m, d), dtype=np.float32),
            rng.standard_normal((n, d), dtype=np.float32))


@pytest.mark.parametrize("m,d,k", [(50_000, 128, 10), (30_001, 96, 100), (20_000, 300, 32)])
def test_prepared_search_is_exact(tmp_path, m, d, k):
    X, Q = _data(m, 257, d, m + d)
    Xd, Qd = torch.from_numpy(X).cuda(), torch.from_numpy(Q).cuda()
    ed, ei = oracle_knn(Q, X, k)
    prep = engine.PreparedRows.prepare(Xd)
    for rows in (prep, None):
        d_, i_ = engine.search(Qd, Xd, k, engine="tc_f16", prepared=rows)
        np.testing.assert_array_equal(i_.cpu().numpy(), ei)
        np.testing.assert_array_equal(d_.cpu().numpy(), ed)
    path = tmp_path / "rows.bin"
    prep.save(path)
    back = engine.PreparedRows.load(path, Xd.device)
    assert torch.equal(back.buffer, prep.buffer)
    d_, i_ = engine.search(Qd, Xd, k, engine="tc_f16", prepared=back)
    np.testing.assert_array_equal(i_.cpu().numpy(), ei)
    st = engine.last_stats(Qd, Xd, k, engine="tc_f16", prepared=True)
    assert st["engine"] == "tc_f16" and st["device_error"] == 0
    # the rows' norm bound and largest rounding error travel in the buffer, so the margin
    # and the filter's candidates are those of the search that converts the rows itself
    engine.search(Qd, Xd, k, engine="tc_f16")
    sr = engine.last_stats(Qd, Xd, k, engine="tc_f16")
    assert (st["candidates"], st["survivors"]) == (sr["candidates"], sr["survivors"])


def test_prepared_workspace_is_smaller_and_mismatch_is_rejected():
    X, Q = _data(40_000, 64, 128, 7)
    Xd, Qd = torch.from_numpy(X).cuda(), torch.from_numpy(Q).cuda()
    plain = _lib.make_opts("tc_f16")
    prep_opts = _lib.make_opts("tc_f16", flags=_lib.FLAG_PREPARED)
    full = engine.workspace_size(64, 40_000, 128, 10, plain)
    small = engine.workspace_size(64, 40_000, 128, 10, prep_opts)
    assert full - small >= 40_000 * 128 * 2  # the f16 rows are not in it
    other = engine.PreparedRows.prepare(Xd[:30_000])
    with pytest.raises(ValueError):
        engine.search(Qd, Xd, 10, engine="tc_f16", prepared=other)
    # the library checks the buffer's own header too
    forged = engine.PreparedRows(other.buffer, (40_000, 128))
    with pytest.raises(_lib.BfkError) as e:
        engine.search(Qd, Xd, 10, engine="tc_f16", prepared=forged)
    assert e.value.status == 1
