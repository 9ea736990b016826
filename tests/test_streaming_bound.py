"""The bound the out-of-core search hands to later chunks (CPU only).

_bound_from_running turns the running k-th exact distance D into a bound on
(k-th distance - ||q||^2).  It must not fall below D - ||q||^2 for the engine's
FP32 ||q||^2 (a sequential FP32 sum of squares) nor for the exact one, and it is
+inf while the running list still holds padding.
"""
import numpy as np
import torch

from gpu_algo_b200.streaming import PAD_DIST, _bound_from_running


def test_bound_is_above_both_norms():
    rng = np.random.Generator(np.random.PCG64(31))
    for d in (8, 128, 960):
        q = rng.standard_normal((64, d)).astype(np.float32) * np.float32(rng.uniform(0.01, 100))
        exact = (q.astype(np.float64) ** 2).sum(1)
        fp32 = np.zeros(64, dtype=np.float32)
        for c in range(d):
            fp32 = np.float32(fp32 + q[:, c] * q[:, c])
        dk = (exact * rng.uniform(0.5, 3.0, 64)).astype(np.float32)
        run_d = np.zeros((64, 5), dtype=np.float32)
        run_d[:, 4] = dk
        run_d[:3, 4] = PAD_DIST
        qn2_low = torch.from_numpy(exact) * (1.0 - (d + 2) * 2.0 ** -23)
        b = _bound_from_running(torch.from_numpy(run_d), qn2_low, 5).numpy()
        assert np.isinf(b[:3]).all()
        assert (b[3:].astype(np.float64) >= dk[3:].astype(np.float64) - exact[3:]).all()
        assert (b[3:].astype(np.float64) >= dk[3:].astype(np.float64) - fp32[3:].astype(np.float64)).all()
