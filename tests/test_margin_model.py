"""The tensor-core filter's error margin, checked on CPU against the oracle's reference
distances (no GPU).

The filter value of row j for query q is v = fma(c, acc, ||x_j||^2) in FP32, where acc
is the dot product of the f16 forms of q and x_j (q scaled by one power of two per
batch, rows by one per 64-row group, each max |value| into [2^13, 2^14)) and
c = -2 / (s_q s_x).  tc_prep_q_kernel bounds |(||q||^2 + v) - D_j| by a per-query
margin, D_j being the reference kernel's FP32 distance.  This restates that arithmetic
in NumPy (the tensor core modelled as an exact sum rounded once to FP32; the margin's
accumulation term covers the rest; the f16 rounding errors of q and of the rows measured
as the prep kernels measure them) and checks:
* the bound holds, with room, from data scales of 1e6 down to norms near 2^-48;
* below that it fails (c underflows to zero, FP32 rounding goes subnormal), and from
  ||q|| + max ||x|| = 2^63 on v can overflow to +inf, so that the filter never keeps a
  row that the exact search returns with an infinite distance.  Outside
  [2^-48, 2^63) every query goes to the exact SIMT engine.
"""
import math

import numpy as np
import pytest

from oracle import oracle_all_dists

# tc_prep_q_kernel: qn + Rx outside [LOW, HIGH) -> exact SIMT engine
LOW, HIGH = 2.0 ** -48, 2.0 ** 63
GROUP_ROWS = 64


def _pow2_scale_for(maxabs) -> np.float32:
    """2^p with maxabs * 2^p in [2^13, 2^14), p clamped to [-126, 126]."""
    mx = float(maxabs)
    if not mx > 0 or not math.isfinite(mx):
        return np.float32(1.0)
    _, e = math.frexp(mx)
    return np.float32(2.0 ** min(126, max(-126, 14 - e)))


def _f32_round_up(x: float) -> np.float32:
    y = np.float32(x)
    return np.nextafter(y, np.float32(np.inf)) if float(y) < x else y


def filter_model(Q: np.ndarray, X: np.ndarray) -> dict:
    """ratio: |(||q||^2 + v) - D| / margin, max over the rows where v and D are finite,
    per query; norms: qn + Rx per query; v and D: (n, m)."""
    n, d = Q.shape
    d_pad = -(-d // 64) * 64
    sq = _pow2_scale_for(np.abs(Q).max())
    qh = (Q * sq).astype(np.float16)
    ssq = np.einsum("ij,ij->i", Q, Q, dtype=np.float32)
    ssx = np.einsum("ij,ij->i", X, X, dtype=np.float32)
    rx = float(np.max(np.sqrt(ssx) * np.float32(1.0 + 2.0 ** -10)))
    xh = np.empty(X.shape, dtype=np.float16)
    xinv = np.empty(X.shape[0], dtype=np.float32)
    for g in range(0, X.shape[0], GROUP_ROWS):
        sc = _pow2_scale_for(np.abs(X[g:g + GROUP_ROWS]).max())
        xh[g:g + GROUP_ROWS] = (X[g:g + GROUP_ROWS] * sc).astype(np.float16)
        xinv[g:g + GROUP_ROWS] = np.float32(1.0) / sc
    # the f16 rounding errors, measured as the prep kernels measure them (v - h / s is
    # exact in FP32), each norm rounded up by (d + 3) 2^-24
    up = 1.0 + (d + 3) * 2.0 ** -24
    dq = Q - qh.astype(np.float32) * (np.float32(1.0) / sq)
    dx = X - xh.astype(np.float32) * xinv[:, None]
    eq = np.sqrt(np.einsum("ij,ij->i", dq, dq, dtype=np.float32).astype(np.float64)) * up
    ex = float(np.sqrt(np.einsum("ij,ij->i", dx, dx, dtype=np.float32).max())) * up
    acc = (qh.astype(np.float64) @ xh.astype(np.float64).T).astype(np.float32)
    c = (np.float32(-2.0) * (np.float32(1.0) / sq)) * xinv  # FP32, may underflow to 0
    with np.errstate(over="ignore"):  # v may overflow to +inf, as in FP32 on the GPU
        v = (c.astype(np.float64)[None, :] * acc.astype(np.float64)
             + ssx.astype(np.float64)[None, :]).astype(np.float32)
    # the margin, as tc_prep_q_kernel forms it
    qn = np.sqrt(ssq.astype(np.float64)) * (1.0 + 2.0 ** -10)
    dotr = eq * rx + qn * ex + eq * ex
    accr = (d_pad + 16) * 2.0 ** -22 * (qn + eq) * (rx + ex)
    f32t = 2.0 * (d + 8) * 2.0 ** -24 * (qn + rx) ** 2
    margin = np.array([_f32_round_up(t * (1 + 1e-6)) for t in 2.0 * (dotr + accr) + f32t],
                      dtype=np.float64)
    nq = (Q.astype(np.float64) ** 2).sum(1)  # any value common to a query's rows works
    D = oracle_all_dists(Q, X)
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        err = np.abs(nq[:, None] + v.astype(np.float64) - D.astype(np.float64))
        ratio = np.where(np.isfinite(err) & (err > 0), err / margin[:, None], 0.0).max(axis=1)
    return {"ratio": ratio, "norms": qn + rx, "v": v, "D": D}


def _data(seed, n, m, d, q_scale, x_scale):
    rng = np.random.Generator(np.random.PCG64(seed))
    return ((rng.standard_normal((n, d)) * q_scale).astype(np.float32),
            (rng.standard_normal((m, d)) * x_scale).astype(np.float32))


@pytest.mark.parametrize("q_scale,x_scale", [(1.0, 1.0), (1e6, 1e6), (1e-6, 1e-6),
                                             (1e-13, 1e-13), (1e-15, 1e-15),
                                             (1.0, 1e-30), (1e-30, 1.0), (1e-20, 1e-10)])
@pytest.mark.parametrize("d", [8, 128, 300])
def test_margin_bounds_the_filter_error(q_scale, x_scale, d):
    Q, X = _data(d, 24, 640, d, q_scale, x_scale)
    f = filter_model(Q, X)
    assert ((f["norms"] >= LOW) & (f["norms"] < HIGH)).all()
    assert np.isfinite(f["v"]).all() and np.isfinite(f["D"]).all()
    assert f["ratio"].max() <= 0.8, f["ratio"].max()


def test_measured_rounding_beats_the_worst_case():
    """The measured f16 rounding errors are well inside the worst case 2^-11 ||.||,
    which is what makes the margin about half the worst-case one on Gaussian data."""
    Q, X = _data(7, 24, 640, 128, 1.0, 1.0)
    qh = (Q * _pow2_scale_for(np.abs(Q).max())).astype(np.float16)
    dq = Q - qh.astype(np.float32) / _pow2_scale_for(np.abs(Q).max())
    ratio = np.linalg.norm(dq, axis=1) / (2.0 ** -11 * np.linalg.norm(Q, axis=1))
    assert ratio.max() < 0.7


def test_rows_of_mixed_scale_in_one_group():
    """Small rows share their group's scale with a large one: their f16 values lose
    precision (down to subnormals), which the margin's Rx terms cover."""
    Q, X = _data(3, 24, 640, 64, 1.0, 1.0)
    X[::64] *= 1e4
    X[1::64] *= 1e-8
    f = filter_model(Q, X)
    assert f["ratio"].max() <= 0.8, f["ratio"].max()


@pytest.mark.parametrize("scale", [1e-20, 1e-22])
def test_margin_fails_below_the_guard(scale):
    """Below the guard the bound does not hold, so those inputs must not be filtered."""
    Q, X = _data(5, 24, 640, 64, scale, scale)
    f = filter_model(Q, X)
    assert (f["norms"] < LOW).all()
    assert f["ratio"].max() > 1.0


def test_filter_drops_infinite_distances_above_the_guard():
    """From the upper guard on, v overflows to +inf for rows that the exact search returns
    (with an infinite distance, when fewer than k rows have a finite one)."""
    Q, X = _data(6, 24, 640, 8, 1.0, 1.0)
    # every norm 1.2e19: the squared norms stay finite in FP32, their sums do not
    Q = (Q / np.linalg.norm(Q, axis=1, keepdims=True) * np.float32(1.2e19)).astype(np.float32)
    X = (X / np.linalg.norm(X, axis=1, keepdims=True) * np.float32(1.2e19)).astype(np.float32)
    assert np.isfinite(np.einsum("ij,ij->i", X, X, dtype=np.float32)).all()
    f = filter_model(Q, X)
    assert (f["norms"] >= HIGH).all()
    lost = np.isinf(f["v"])
    assert lost.any() and np.isinf(f["D"][lost]).all()
    from oracle import oracle_knn
    _, ids = oracle_knn(Q, X, X.shape[0])
    q = int(np.argmax(lost.any(axis=1)))
    assert np.isin(np.flatnonzero(lost[q]), ids[q]).all()  # returned by the exact search


# ---------------------------------------------------------------------------
# The filter kernel's chunk test (knn_tc_filter_kernel): a 16-column chunk is skipped
# when its largest accumulator is <= T = rd(ru(succ(theta) - min ||x||^2) * (1/c)).
# Skipping must never lose a column whose v = rn(c * acc + ||x||^2) is <= theta.
# Restated here with exact rational arithmetic and the kernel's rounding modes.
# ---------------------------------------------------------------------------
from fractions import Fraction  # noqa: E402

_INF32 = np.float32(np.inf)


def _f32(fr: Fraction, mode: str) -> np.float32:
    """fr rounded to float32: 'rd' down, 'ru' up, 'rn' to nearest (ties to even)."""
    x = np.float32(float(fr))
    while Fraction(float(x)) > fr:
        x = np.nextafter(x, -_INF32)
    while Fraction(float(np.nextafter(x, _INF32))) <= fr:
        x = np.nextafter(x, _INF32)
    lo = x  # the largest float32 <= fr
    if mode == "rd" or Fraction(float(lo)) == fr:
        return lo
    hi = np.nextafter(lo, _INF32)
    if mode == "ru":
        return hi
    dl, dh = fr - Fraction(float(lo)), Fraction(float(hi)) - fr
    if dl != dh:
        return lo if dl < dh else hi
    return lo if (int(lo.view(np.uint32)) & 1) == 0 else hi


def _chunk_skipped(acc, nx, c, theta) -> bool:
    theta2 = np.nextafter(np.float32(theta), _INF32)
    gmin = np.float32(nx.min())
    inv_c = Fraction(1) / Fraction(float(c))  # an exact power of two
    diff = _f32(Fraction(float(theta2)) - Fraction(float(gmin)), "ru")
    T = _f32(Fraction(float(diff)) * inv_c, "rd")
    return bool(np.float32(acc.max()) <= T)


@pytest.mark.parametrize("seed", range(4))
def test_chunk_skip_never_loses_a_kept_column(seed):
    g = np.random.default_rng(seed)
    c = np.float32(-2.0 ** int(g.integers(-30, -10)))
    skipped = kept_in_skipped = 0
    for _ in range(400):
        acc = (g.standard_normal(16) * 2.0 ** int(g.integers(10, 26))).astype(np.float32)
        nx = np.abs(g.standard_normal(16) * 4).astype(np.float32) + np.float32(1.0)
        if g.random() < 0.5:
            nx[:] = nx[0]  # equal norms, as unit vectors have: the tightest case
        v = [_f32(Fraction(float(c)) * Fraction(float(a)) + Fraction(float(x)), "rn")
             for a, x in zip(acc, nx)]
        # theta at, just below or just above the smallest v of the chunk
        vmin = min(v)
        theta = [vmin, np.nextafter(vmin, -_INF32), np.nextafter(vmin, _INF32)][int(g.integers(3))]
        if _chunk_skipped(acc, nx, c, theta):
            skipped += 1
            kept_in_skipped += sum(1 for x in v if x <= theta)
    assert kept_in_skipped == 0
    assert skipped > 0  # the rule does skip (theta just below the chunk's smallest v)
