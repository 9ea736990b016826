"""Out-of-core search (gpu_algo_b200.streaming), B200 only.

The database sits in host memory and crosses to the GPU in row chunks; the
running k-th distance bounds later chunks.  The merged lists must equal the
oracle's exact top-k of the whole database, with or without that bound, for
chunk sizes that divide the rows unevenly, and for one chunk larger than the
database.
"""
import numpy as np
import pytest
import torch

from gpu_algo_b200.streaming import streamed_search
from oracle import oracle_knn

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("chunk_rows,share", [(65_536, True), (65_536, False), (1 << 20, True)])
def test_streamed_search_is_exact(chunk_rows, share):
    rng = np.random.Generator(np.random.PCG64(21))
    X = rng.standard_normal((300_001, 64), dtype=np.float32)
    Q = rng.standard_normal((200, 64), dtype=np.float32)
    ed, ei = oracle_knn(Q, X, 32)
    Xh = torch.from_numpy(X).pin_memory()
    d_, i_ = streamed_search(torch.from_numpy(Q).cuda(), Xh, 32, chunk_rows=chunk_rows,
                             share_bound=share)
    np.testing.assert_array_equal(i_.cpu().numpy(), ei)
    np.testing.assert_array_equal(d_.cpu().numpy(), ed)


def test_streamed_search_pageable_host_memory():
    rng = np.random.Generator(np.random.PCG64(22))
    X = rng.standard_normal((90_000, 128), dtype=np.float32)
    Q = rng.standard_normal((130, 128), dtype=np.float32)
    ed, ei = oracle_knn(Q, X, 100)
    d_, i_ = streamed_search(torch.from_numpy(Q).cuda(), torch.from_numpy(X), 100,
                             chunk_rows=40_000)
    np.testing.assert_array_equal(i_.cpu().numpy(), ei)
    np.testing.assert_array_equal(d_.cpu().numpy(), ed)
