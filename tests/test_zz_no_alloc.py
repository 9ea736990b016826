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

from gpu_algo_b200 import _lib, data, engine

pytestmark = pytest.mark.gpu


def _noalloc(Q, X, k, id_offset=0):
    lib = _lib.load()
    n, d = Q.shape
    m = X.shape[0]
    out_d = torch.empty((n, k), dtype=torch.float32, device=Q.device)
    out_i = torch.empty((n, k), dtype=torch.int32, device=Q.device)
    st = lib.bfk_search_noalloc(Q.data_ptr(), n, X.data_ptr(), m, d, k, id_offset,
                                out_d.data_ptr(), out_i.data_ptr(),
                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(st, "bfk_search_noalloc")
    torch.cuda.synchronize()
    return out_d.cpu().numpy(), out_i.cpu().numpy()


def test_noalloc_matches_workspace_entry_point_twice():
    X, Q = data.workload_arrays("plumbing", n_rows=50_000, n_queries=600)
    Xd = torch.from_numpy(X).cuda()
    for (q0, q1, k, off) in ((0, 300, 10, 0), (300, 600, 37, 1000)):
        Qd = torch.from_numpy(Q[q0:q1]).cuda()
        got_d, got_i = _noalloc(Qd, Xd, k, off)  # two calls in a row share the scratch
        ref_d, ref_i = engine.search(Qd, Xd, k, id_offset=off)
        torch.cuda.synchronize()
        # both are exact: the same distances bit for bit, the same ids
        np.testing.assert_array_equal(got_i, ref_i.cpu().numpy())
        np.testing.assert_array_equal(got_d, ref_d.cpu().numpy())


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib = _lib.load()
    n, k = 2048, 1024  # 16 * n * k bytes > 16 MiB
    st = lib.bfk_search_noalloc(None, n, None, 10, 8, k, 0, None, None, None)
    assert st == 2  # BFK_ERR_UNSUPPORTED, before any device work
