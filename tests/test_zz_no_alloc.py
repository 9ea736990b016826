"""bfk_search_noalloc: the search for callers that cannot allocate device memory.

Some callers (code running inside another allocator's callback, real-time
threads that must not block on cudaMalloc, hosts that only hand out fixed
pre-registered buffers) cannot provide a workspace.  The no-allocation entry
point keeps its scratch in a fixed array inside the library.  This file is
collected last so that a run stopping at the first failure has run every
other test first.
"""
import ctypes

import numpy as np
import pytest
import torch

from gpu_algo_b200 import _lib, data
from oracle import oracle_knn

pytestmark = pytest.mark.gpu


def _noalloc(Q, X, k, id_offset=0):
    lib = _lib.load()
    n, d = Q.shape
    m = X.shape[0]
    out_d = torch.empty((n, k), dtype=torch.float32, device=Q.device)
    out_i = torch.empty((n, k), dtype=torch.int32, device=Q.device)
    st = lib.bfk_search_noalloc(Q.data_ptr(), n, X.data_ptr() if m else None, m, d, k,
                                id_offset, out_d.data_ptr(), out_i.data_ptr(),
                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(st, "bfk_search_noalloc")
    torch.cuda.synchronize()
    return out_d.cpu().numpy(), out_i.cpu().numpy()


@pytest.mark.parametrize("q0,q1,k,off", [
    (0, 300, 10, 0),        # about 45 slices: the sorting-network merge
    (300, 600, 37, 1000),   # the same, with ids offset
    (600, 2600, 10, 7),     # about 8 slices: the rank merge
])
def test_noalloc_matches_oracle_twice(q0, q1, k, off):
    X, Q = data.workload_arrays("plumbing", n_rows=50_000, n_queries=2600)
    Xd = torch.from_numpy(X).cuda()
    Qd = torch.from_numpy(Q[q0:q1]).cuda()
    ref_d, ref_i = oracle_knn(Q[q0:q1], X, k)
    # two calls in a row share the scratch: the second must not see the first's lists
    for _ in range(2):
        got_d, got_i = _noalloc(Qd, Xd, k, off)
        np.testing.assert_array_equal(got_i, ref_i + off)
        np.testing.assert_array_equal(got_d, ref_d)


def test_noalloc_without_rows_pads():
    Qd = torch.zeros((5, 8), dtype=torch.float32, device="cuda")
    Xd = torch.zeros((0, 8), dtype=torch.float32, device="cuda")
    got_d, got_i = _noalloc(Qd, Xd, 3)
    np.testing.assert_array_equal(got_i, np.full((5, 3), -1, np.int32))
    np.testing.assert_array_equal(got_d, np.full((5, 3), np.float32(3.402823e38)))


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib = _lib.load()
    # 16 * n * k bytes > 16 MiB, and shapes whose byte count would wrap in 64 bits
    for n, k in ((2048, 1024), (1 << 61, 1), ((1 << 62) + 1, 2), (1 << 20, 2)):
        st = lib.bfk_search_noalloc(None, n, None, 10, 8, k, 0, None, None, None)
        assert st == 2, (n, k)  # BFK_ERR_UNSUPPORTED, before any device work
