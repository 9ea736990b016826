"""The tensor-core filter's error margin, measured on the device for every pair.

The tensor-core engine is exact only if, for every query q and row x,

    |(||q||^2 + v) - D| <= m_q,

where v is the filter value the kernel computes from the f16 tensor-core dot product
(v = ||x||^2 - 2 q.x), D is the reference's FP32 distance (bf/fp32.py:74-82: direct
differences, fused multiply-adds in dimension order) and m_q the margin the engine
derives for the query.  The derivation assumes how the tensor core accumulates f16
products in FP32.  These tests read v for every (query, row) pair of each case from
the device (``bfk_filter_values``: the engine's own preparation and filter kernel,
one pass with no bound) and check the inequality against the oracle's D, with ||q||^2
taken exactly (float64).  Each case has at least 10^7 pairs; the largest ratio
|(||q||^2 + v) - D| / m_q is printed.

The same data also isolate the one assumption about the hardware: the f16 operands
the kernel feeds the tensor core are rebuilt on the host (the same power-of-two
scales and round-to-nearest f16), their dot products taken in float64, and the
device's v compared with ||x||^2 - 2 q.x of those operands.  What is left is the
tensor core's FP32 accumulation (plus the FP32 norm and the epilogue's one fused
step), which the margin allows (d_pad + 16) * 2^-22 * ||q|| * max ||x|| for, per
dot product; the largest share of that allowance used is printed and asserted.
"""
import zlib

import numpy as np
import pytest
import torch

from gpu_algo_b200 import data, engine
from oracle import oracle_all_dists

pytestmark = pytest.mark.gpu


def _rng(seed):
    return np.random.default_rng(np.random.PCG64(seed))


def _unit(n, m, d, seed):
    X, Q = data.workload_arrays("unit-10m", n_rows=m, n_queries=n)
    return Q, X


def _mixture(n, m, d, seed):
    X, Q = data.workload_arrays("mixture-k-sweep", n_rows=m, n_queries=n)
    return Q, X


def _near_duplicates(n, m, d, seed):
    # rows and queries within 1e-3 of one centre of norm ~1100: the largest
    # cancellation between ||q||^2 + ||x||^2 and 2 q.x
    g = _rng(seed)
    c = (100.0 * g.standard_normal(d)).astype(np.float32)
    X = (c + 1e-3 * g.standard_normal((m, d))).astype(np.float32)
    Q = (c + 1e-3 * g.standard_normal((n, d))).astype(np.float32)
    return Q, X


def _large_row_in_group(n, m, d, seed):
    # one row of norm ~1e3 in every 64-row scale group of rows of norm ~0.1: the
    # group's power-of-two scale follows the large row, the small rows keep few
    # f16 bits (some elements become subnormal or zero)
    g = _rng(seed)
    X = (0.01 * g.standard_normal((m, d))).astype(np.float32)
    X[17::64] *= np.float32(1e4)
    Q = (0.01 * g.standard_normal((n, d))).astype(np.float32)
    Q[::7] *= np.float32(300.0)
    return Q, X


def _mixed_query_scales(n, m, d, seed):
    g = _rng(seed)
    X = g.standard_normal((m, d)).astype(np.float32)
    scale = (10.0 ** g.uniform(-3, 3, size=(n, 1))).astype(np.float32)
    Q = (g.standard_normal((n, d)) * scale).astype(np.float32)
    return Q, X


def _halves_long(n, m, d, seed):
    # d = 1024, products positive over the first half of the dimensions and negative
    # over the second: the partial sums grow to ~d/2 * 9 and cancel to about 0 (the
    # longest accumulation with the largest cancellation)
    g = _rng(seed)
    sign = np.where(np.arange(d) < d // 2, 1.0, -1.0)
    X = (3.0 * sign + 0.05 * g.standard_normal((m, d))).astype(np.float32)
    Q = (3.0 + 0.05 * g.standard_normal((n, d))).astype(np.float32)
    return Q, X


def _gaussian_long(n, m, d, seed):
    g = _rng(seed)
    return (g.standard_normal((n, d)).astype(np.float32),
            g.standard_normal((m, d)).astype(np.float32))


def _pow2_scale(maxabs):
    """The engine's power-of-two scale: maxabs * scale in [2^13, 2^14)."""
    maxabs = np.asarray(maxabs, np.float64)
    _, e = np.frexp(maxabs)
    p = np.clip(14 - e, -126, 126)
    ok = (maxabs > 0) & np.isfinite(maxabs)
    return np.where(ok, np.ldexp(1.0, p), 1.0)


def _f16_dot(Q, X):
    """Dot products of the f16 operands the kernel multiplies, exactly, in real units."""
    sq = float(_pow2_scale(np.abs(Q).max()))
    gmax = np.abs(X).reshape(-1, 64, X.shape[1]).max(axis=(1, 2)) if X.shape[0] % 64 == 0 \
        else None
    assert gmax is not None, "row count must be a multiple of the 64-row scale group"
    sx = np.repeat(_pow2_scale(gmax), 64)
    qh = (Q * np.float32(sq)).astype(np.float16).astype(np.float64) / sq
    xh = (X * sx[:, None].astype(np.float32)).astype(np.float16).astype(np.float64) / sx[:, None]
    return qh @ xh.T


CASES = {
    # name: (generator, queries, rows, d)
    "unit-vectors": (_unit, 512, 32_768, 128),
    "mixture": (_mixture, 512, 32_768, 128),
    "near-duplicates": (_near_duplicates, 512, 32_768, 128),
    "large-row-in-group": (_large_row_in_group, 512, 32_768, 128),
    "mixed-query-scales": (_mixed_query_scales, 512, 32_768, 128),
    "gaussian-d1024": (_gaussian_long, 128, 81_920, 1024),
    "cancelling-halves-d1024": (_halves_long, 128, 81_920, 1024),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_filter_values_stay_within_the_margin(name):
    gen, n, m, d = CASES[name]
    Q, X = gen(n, m, d, seed=zlib.crc32(name.encode()))
    assert n * m >= 10_000_000
    v, qinfo, exact_only = engine.filter_values(torch.from_numpy(Q).cuda(),
                                                torch.from_numpy(X).cuda())
    torch.cuda.synchronize()
    assert not exact_only, "inside the margin's range: the filter must be used"
    v = v.cpu().numpy().astype(np.float64)
    margin = qinfo[:, 1].cpu().numpy().astype(np.float64)
    assert np.all(np.isfinite(v)), "every pair of finite inputs has a finite filter value"
    assert np.all(np.isfinite(margin)) and np.all(margin > 0)
    D = oracle_all_dists(Q, X).astype(np.float64)
    qn2 = np.einsum("ij,ij->i", Q.astype(np.float64), Q.astype(np.float64))
    ratio = np.abs(qn2[:, None] + v - D) / margin[:, None]
    worst = np.unravel_index(int(np.argmax(ratio)), ratio.shape)
    print(f"\nmargin audit {name}: {n * m} pairs, d={d}: max |(||q||^2+v)-D|/margin = "
          f"{ratio.max():.4f} (query {worst[0]}, row {worst[1]}), "
          f"99.99th percentile {np.percentile(ratio, 99.99):.4f}, "
          f"median margin {np.median(margin):.4g}, median D {np.median(D):.4g}")
    assert ratio.max() <= 1.0

    # the tensor core's accumulation alone
    d_pad = -(-d // 64) * 64
    xn2 = np.einsum("ij,ij->i", X.astype(np.float64), X.astype(np.float64))
    qn = np.sqrt(qn2)
    rx = np.sqrt(xn2.max())
    model = xn2[None, :] - 2.0 * _f16_dot(Q, X)
    acc_term = 2.0 * (d_pad + 16) * 2.0 ** -22 * qn[:, None] * rx
    fp32_terms = 2.0 ** -23 * (np.abs(v) + xn2[None, :]) + d * 2.0 ** -24 * xn2[None, :]
    used = np.abs(v - model) / (acc_term + fp32_terms)
    print(f"margin audit {name}: accumulation uses at most {used.max():.4f} of its allowance "
          f"(99.99th percentile {np.percentile(used, 99.99):.4f})")
    assert used.max() <= 1.0
