"""Parity of the CUDA engines with the oracle, through the C ABI (B200 only).

The engines return the reference kernels' exact FP32 distances, so the check
is bit-exact equality with the oracle's (distance, index) lists; the
tolerance rule of check_parity (1e-5 tie window, 1e-4 relative distance) is
asserted as well.
"""
import numpy as np
import pytest
import torch

from gpu_algo_b200 import _lib, engine
from oracle import check_parity, oracle_knn, oracle_merge

pytestmark = pytest.mark.gpu

ENGINES = ["direct", "auto", "tc_f16"]


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run(Q, X, k, **kw):
    d_, i_ = engine.search(dev(Q), dev(X), k, **kw)
    torch.cuda.synchronize()
    return d_.cpu().numpy(), i_.cpu().numpy()


def tc_ok(d, k):
    """Whether the tensor-core engine takes this (d, k) (it rejects, never falls back)."""
    try:
        engine.workspace_size(64, 8192, d, k, _lib.make_opts("tc_f16"))
        return True
    except _lib.BfkError as e:
        assert e.status == 2
        return False


def assert_exact(got_d, got_i, exp_d, exp_i, what=""):
    np.testing.assert_array_equal(got_i, exp_i, err_msg=f"{what}: ids")
    np.testing.assert_array_equal(got_d, exp_d, err_msg=f"{what}: dists")


@pytest.mark.parametrize("eng", ENGINES)
def test_plumbing_bit_exact(plumbing, eng):
    X, Q, gd, gi = plumbing
    d_, i_ = run(Q, X, 10, engine=eng)
    assert_exact(d_, i_, gd, gi, eng)
    rd, ri = oracle_knn(Q[:128], X, 11)
    assert check_parity(d_[:128], i_[:128], rd, ri, 10) == []


@pytest.mark.parametrize("eng", ENGINES)
def test_edge_cases_bit_exact(edges, eng):
    for name, (Q, X, k, gd, gi) in edges.items():
        if eng == "tc_f16" and not tc_ok(Q.shape[1], k):
            continue
        d_, i_ = run(Q, X, k, engine=eng)
        assert_exact(d_, i_, gd, gi, f"{eng}/{name}")


def test_tc_stats_plumbing(plumbing):
    X, Q, gd, gi = plumbing
    Qd, Xd = dev(Q), dev(X)
    engine.search(Qd, Xd, 10, engine="tc_f16")
    st = engine.last_stats(Qd, Xd, 10, engine="tc_f16")
    assert st["engine"] == "tc_f16" and st["device_error"] == 0
    assert st["fallback_queries"] == 0
    assert st["survivors"] >= Q.shape[0] * 10
    assert st["candidates"] >= st["survivors"]


@pytest.mark.parametrize("slices", [1, 2, 5, 64])
def test_tc_slices_agree(plumbing, slices):
    X, Q, gd, gi = plumbing
    d_, i_ = run(Q[:300], X, 10, engine="tc_f16", slices=slices)
    assert_exact(d_, i_, gd[:300], gi[:300], f"tc slices={slices}")


def test_tc_pool_overflow_falls_back_exactly(plumbing):
    X, Q, gd, gi = plumbing
    Qd, Xd = dev(Q[:200]), dev(X)
    d_, i_ = engine.search(Qd, Xd, 10, engine="tc_f16", max_candidates=12)
    st = engine.last_stats(Qd, Xd, 10, engine="tc_f16", max_candidates=12)
    assert st["fallback_queries"] > 0
    assert_exact(d_.cpu().numpy(), i_.cpu().numpy(), gd[:200], gi[:200], "overflow")


def test_tc_nonfinite_rows_use_exact_engine():
    rng = np.random.Generator(np.random.PCG64(5))
    X = rng.standard_normal((9000, 64), dtype=np.float32)
    X[123, 7] = np.nan
    X[4567, 0] = np.inf
    Q = rng.standard_normal((130, 64), dtype=np.float32)
    ed, ei = oracle_knn(Q, X, 16)
    d_, i_ = run(Q, X, 16, engine="tc_f16")
    assert_exact(d_, i_, ed, ei, "nonfinite")


@pytest.mark.parametrize("case", ["tiny", "small", "huge"])
def test_tc_norms_outside_the_margin_guard_use_exact_engine(case):
    """Outside 2^-48 <= ||q|| + max ||x|| < 2^63 the filter cannot be trusted: below,
    its margin does not hold (the scale factor underflows, FP32 rounding goes
    subnormal); above, v and distances overflow to +inf, and rows at +inf are still
    returned when fewer than k rows are finite.  Every query then goes to the exact
    engine.  Inside the range ("small") the filter runs as usual.  All stay bit-exact."""
    rng = np.random.Generator(np.random.PCG64(8))
    m, n, k = (300, 130, 300) if case == "huge" else (9000, 130, 16)
    X = rng.standard_normal((m, 64)).astype(np.float32)
    Q = rng.standard_normal((n, 64)).astype(np.float32)
    if case == "huge":  # norms 1.2e19: finite squared norms, infinite distances
        X = (X / np.linalg.norm(X, axis=1, keepdims=True) * np.float32(1.2e19)).astype(np.float32)
        Q = (Q / np.linalg.norm(Q, axis=1, keepdims=True) * np.float32(1.2e19)).astype(np.float32)
    else:
        scale = np.float32(1e-20 if case == "tiny" else 1e-13)
        X, Q = X * scale, Q * scale
    ed, ei = oracle_knn(Q, X, k)
    if case == "huge":
        assert np.isinf(ed).any() and (ei >= 0).all()
    Qd, Xd = dev(Q), dev(X)
    d_, i_ = engine.search(Qd, Xd, k, engine="tc_f16")
    st = engine.last_stats(Qd, Xd, k, engine="tc_f16")
    assert st["fallback_queries"] == (0 if case == "small" else n)
    assert_exact(d_.cpu().numpy(), i_.cpu().numpy(), ed, ei, case)


@pytest.mark.parametrize("name,n,m,k", [("mixture-k-sweep", 300, 200_000, 32),
                                        ("mixture-k-sweep", 257, 120_000, 100),
                                        ("unit-10m", 256, 300_000, 100),
                                        ("stream-100m", 130, 250_000, 10),
                                        ("mixture-k-sweep", 200, 100_000, 1),
                                        ("published-d8", 300, 1_000_000, 1)])
def test_tc_workload_samples(name, n, m, k):
    from gpu_algo_b200 import data
    X, Q = data.workload_arrays(name, n_rows=m, n_queries=n)
    ed, ei = oracle_knn(Q, X, k)
    d_, i_ = run(Q, X, k, engine="tc_f16")
    assert_exact(d_, i_, ed, ei, f"{name} n={n} m={m} k={k}")


@pytest.mark.parametrize("slices", [1, 3, 17, 64])
def test_direct_slices_agree(plumbing, slices):
    X, Q, gd, gi = plumbing
    d_, i_ = run(Q[:100], X, 10, engine="direct", slices=slices)
    assert_exact(d_, i_, gd[:100], gi[:100], f"slices={slices}")


def test_id_offset_and_empty_inputs(plumbing):
    X, Q, gd, gi = plumbing
    d_, i_ = run(Q[:50], X, 10, id_offset=1_000_000)
    assert_exact(d_, i_, gd[:50], gi[:50] + 1_000_000)
    d_, i_ = run(Q[:5], X[:0], 7)
    assert (i_ == -1).all() and (d_ == np.float32(3.402823e38)).all()
    d_, i_ = run(Q[:0], X, 7)
    assert d_.shape == (0, 7)


def test_merge_kernel_matches_oracle_merge(plumbing):
    X, Q, gd, gi = plumbing
    rng = np.random.Generator(np.random.PCG64(3))
    lists, n, k = 9, 300, 10
    parts = [oracle_knn(Q[:n], X[a:a + 7000], k, id_offset=a)
             for a in rng.integers(0, 58_000, size=lists)]
    cd = np.stack([p[0] for p in parts])
    ci = np.stack([p[1] for p in parts])
    ci[2, :, 6:] = -1  # padding entries are skipped
    cd[2, :, 6:] = np.float32(3.402823e38)
    ed, ei = oracle_merge(cd, ci, k)
    md, mi = engine.merge(dev(cd), dev(ci), k)
    assert_exact(md.cpu().numpy(), mi.cpu().numpy(), ed, ei, "merge")


@pytest.mark.parametrize("lists,k", [(2, 100), (8, 100), (100, 100), (3, 1000)])
def test_merge_rank_and_grouped_paths(lists, k):
    """lists * k <= 8192 merges by rank, larger sets by grouped sorts; ties in
    distance across lists order by index; padding sits at the end of a list."""
    rng = np.random.Generator(np.random.PCG64(lists * 1000 + k))
    n = 64
    cd = np.sort(rng.integers(0, 50, size=(lists, n, k)).astype(np.float32), axis=2)
    ci = rng.permutation(lists * n * k).astype(np.int32).reshape(lists, n, k)
    order = np.lexsort((ci, cd), axis=2)
    cd = np.take_along_axis(cd, order, axis=2)
    ci = np.take_along_axis(ci, order, axis=2)
    cd[0, :, k // 3:] = np.float32(3.402823e38)
    ci[0, :, k // 3:] = -1
    ed, ei = oracle_merge(cd, ci, k)
    md, mi = engine.merge(dev(cd), dev(ci), k)
    assert_exact(md.cpu().numpy(), mi.cpu().numpy(), ed, ei, f"merge {lists}x{k}")


@pytest.mark.parametrize("lists,k", [(2, 10), (8, 100), (40, 100)])
def test_packed_merge_matches_merge(lists, k):
    """The sharded exchange's layout: each list's distances then ids in one int32
    block per list, merged in place (bfk_merge_strided)."""
    from gpu_algo_b200.sharded import pack_lists
    rng = np.random.Generator(np.random.PCG64(lists + 7 * k))
    n = 96
    cd = np.sort(rng.standard_normal((lists, n, k)).astype(np.float32) ** 2, axis=2)
    ci = rng.permutation(lists * n * k).astype(np.int32).reshape(lists, n, k)
    cd[-1, :, k // 2:] = np.float32(3.402823e38)
    ci[-1, :, k // 2:] = -1
    blocks = torch.stack([pack_lists(dev(cd[l]), dev(ci[l])) for l in range(lists)])
    pd, pi = engine.merge_packed(blocks.view(lists, 2, n, k), k)
    md, mi = engine.merge(dev(cd), dev(ci), k)
    ed, ei = oracle_merge(cd, ci, k)
    assert_exact(pd.cpu().numpy(), pi.cpu().numpy(), ed, ei, "packed merge")
    assert_exact(md.cpu().numpy(), mi.cpu().numpy(), ed, ei, "merge")


@pytest.mark.parametrize("n,m,d,k", [(1, 100_000, 96, 10), (3, 50_000, 33, 1), (16, 70_001, 96, 64),
                                     (9, 40_000, 300, 17), (16, 8192, 128, 10)])
def test_small_batch_scan_is_exact(n, m, d, k):
    """n <= 16 queries take the streaming scan (one pass over the rows, warps with
    their own lists, merged per block and then across blocks); with duplicate
    rows (exact ties) and a NaN row."""
    rng = np.random.Generator(np.random.PCG64(n * 7 + d))
    X = rng.standard_normal((m, d), dtype=np.float32)
    X[m // 2: m // 2 + 40] = X[7]       # ties at equal distance: lower index first
    X[m // 3, 0] = np.nan
    Q = rng.standard_normal((n, d), dtype=np.float32)
    Q[0] = X[7] + np.float32(0.001)
    ed, ei = oracle_knn(Q, X, k)
    d_, i_ = run(Q, X, k)
    assert_exact(d_, i_, ed, ei, f"scan n={n} m={m} d={d} k={k}")


def test_large_k_and_high_d():
    rng = np.random.Generator(np.random.PCG64(11))
    X = rng.standard_normal((20_000, 960), dtype=np.float32)
    Q = rng.standard_normal((40, 960), dtype=np.float32)
    for k in (100, 1024):
        ed, ei = oracle_knn(Q, X, k)
        d_, i_ = run(Q, X, k)
        assert_exact(d_, i_, ed, ei, f"d=960 k={k}")


@pytest.mark.parametrize("d", [257, 300, 960, 1024])
def test_tc_streamed_query_tiles_high_d(d):
    """d > 256: the query tile's K chunks stream through the stages with the rows'."""
    rng = np.random.Generator(np.random.PCG64(100 + d))
    X = rng.standard_normal((12_000, d), dtype=np.float32)
    Q = rng.standard_normal((200, d), dtype=np.float32)
    assert tc_ok(d, 100)
    ed, ei = oracle_knn(Q, X, 100)
    for pair in (True, None, False):  # the stats below read the last (single-CTA) search
        d_, i_ = run(Q, X, 100, engine="tc_f16", cta_pair=pair)
        assert_exact(d_, i_, ed, ei, f"tc d={d} pair={pair}")
    st = engine.last_stats(dev(Q), dev(X), 100, engine="tc_f16", cta_pair=False)
    assert st["engine"] == "tc_f16" and st["device_error"] == 0


def test_errors_are_raised():
    Q = torch.zeros((4, 8), device="cuda")
    X = torch.zeros((16, 8), device="cuda")
    with pytest.raises(_lib.BfkError) as e:
        engine.search(Q, X, 5000)
    assert e.value.status == 2
    with pytest.raises(TypeError):
        engine.search(Q.double(), X, 3)
    with pytest.raises(ValueError):
        engine.search(Q, torch.zeros((16, 9), device="cuda"), 3)


def test_main_kernel_timing_after_rejected_and_padding_calls(plumbing):
    """A timed call that is rejected before its kernels run leaves no unrecorded event
    pair behind, and a timed call with no rows times its padding fill. Reading an
    unrecorded pair would fail and leave that error for the next launch check."""
    X, Q, gd, gi = plumbing
    Qd, Xd = dev(Q[:64]), dev(X)
    engine.last_stats(Qd, Xd, 10, engine="tc_f16")  # drain earlier timed calls
    other = engine.PreparedRows.prepare(Xd[:30_000])
    forged = engine.PreparedRows(other.buffer, tuple(Xd.shape))
    with pytest.raises(_lib.BfkError) as e:
        engine.search(Qd, Xd, 10, engine="tc_f16", prepared=forged, time_main=True)
    assert e.value.status == 1
    d_, i_ = engine.search(Qd, Xd[:0], 10, time_main=True)
    assert (i_ == -1).all()
    engine.search(Qd, Xd, 10, engine="tc_f16", time_main=True)
    st = engine.last_stats(Qd, Xd, 10, engine="tc_f16")
    assert st["timed_calls"] == 2 and st["main_kernel_ms"] > 0
    d_, i_ = run(Q[:64], X, 10, engine="direct")
    assert_exact(d_, i_, gd[:64], gi[:64], "after timed calls")


def test_bf_dropin_runners(plumbing):
    from gpu_algo_b200.bf import fp32, fp32_heap, fp32_q2, fp32_qgroup, fp32_tiled
    X, Q, gd, gi = plumbing
    Qd, Xd = dev(Q[:200]), dev(X)
    for res in (fp32.run_bf_fp32(Qd, Xd, 10, reps=2),
                fp32_heap.run_bf_fp32_heap(Qd, Xd, 10, reps=2),
                fp32_q2.run_bf_fp32_q2(Qd, Xd, 10, reps=2),
                fp32_qgroup.run_bf_fp32_qgroup(Qd, Xd, 10, qpb=8, reps=2),
                fp32_tiled.run_bf_fp32_tiled(Qd, Xd, 10, tile_size=20_000, reps=2)):
        np.testing.assert_array_equal(res["ids"], gi[:200])
        np.testing.assert_array_equal(res["dists"], gd[:200])
        assert res["ms"] > 0 and res["block"] > 0
    r = fp32_tiled.run_bf_fp32_tiled(Qd, Xd, 10, tile_size=20_000, reps=1)
    assert r["n_tiles"] == 4 and r["tile_size"] == 20_000
    # the merge the tiled runner reports is the merge kernel that ran: 4 lists of 10
    # go through the rank merge, whose shared memory is the lists' keys
    assert r["merge_shared_mem_bytes"] == 4 * 10 * 8
    assert r["merge_kernel_attrs"]["num_regs"] > 0
    assert r["merge_kernel_attrs"]["kernel_variant"] == "merge of 4 lists"
    assert r["merge_kernel_attrs"] != r["partial_kernel_attrs"]
    g = fp32_qgroup.run_bf_fp32_qgroup(Qd, Xd, 10, qpb=8, reps=1)
    assert "qpb_note" in g
    fn, out_ids, out_dists, block, smem, attrs = fp32.build_bf_fp32_runner(Qd, Xd, 10)
    fn()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out_ids.cpu().numpy(), gi[:200])
    assert attrs["num_regs"] > 0 and "kernel_variant" in attrs


def test_tc_cta_pair_bit_exact(plumbing):
    X, Q, gd, gi = plumbing
    # one CTA per query tile, and the engine's own choice (single CTAs below 4M rows)
    for choice, want in ((False, False), (None, False)):
        d_, i_ = engine.search(dev(Q), dev(X), 10, engine="tc_f16", cta_pair=choice)
        st = engine.last_stats(dev(Q), dev(X), 10, engine="tc_f16", cta_pair=choice)
        assert st["cta_pair"] is want
        assert_exact(d_.cpu().numpy(), i_.cpu().numpy(), gd, gi, f"cta_pair={choice}")
    d_, i_ = engine.search(dev(Q), dev(X), 10, engine="tc_f16", cta_pair=True)
    torch.cuda.synchronize()
    assert_exact(d_.cpu().numpy(), i_.cpu().numpy(), gd, gi, "cta pair")
    # an odd number of query tiles pads the pair with an empty tile
    d_, i_ = engine.search(dev(Q[:300]), dev(X), 10, engine="tc_f16", cta_pair=True)
    torch.cuda.synchronize()
    assert_exact(d_.cpu().numpy(), i_.cpu().numpy(), gd[:300], gi[:300], "cta pair, 3 tiles")


def test_shared_bounds_keep_the_merged_result_exact(plumbing):
    """Emulates a two-shard search on one GPU: shard B filters with the bounds
    shard A found (what the all-reduce MIN hands every shard); the merge of the
    two shards' lists must still be the exact top-k of the union."""
    X, Q, gd, gi = plumbing
    Qd = dev(Q[:512])
    half = X.shape[0] // 2
    XA, XB = dev(X[:half]), dev(X[half:])
    saved = []

    def record(t):
        saved.append(t.clone())

    dA, iA = engine.search(Qd, XA, 10, engine="tc_f16", bound_hook=record, plan_rows=half)
    calls = iter(saved)

    def lower(t):
        torch.minimum(t, next(calls), out=t)

    dB, iB = engine.search(Qd, XB, 10, engine="tc_f16", bound_hook=lower, plan_rows=half,
                           id_offset=half)
    assert len(saved) >= 1  # the sampling levels called the hook
    md, mi = engine.merge(torch.stack([dA, dB]), torch.stack([iA, iB]), 10)
    torch.cuda.synchronize()
    assert_exact(md.cpu().numpy(), mi.cpu().numpy(), gd[:512], gi[:512], "shared bounds")
