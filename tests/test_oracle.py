"""Pins the CPU oracle to the reference's own hand-checked tests.

Each test replays a known-answer or invariant test of the reference
(BleedingDev/ir-multivector-retrieval), cited as path:line. Inputs that the
reference draws from Zig's ``floatNorm`` are drawn from numpy here (the
properties tested do not depend on the particular values).
"""
import math

import numpy as np
import pytest

# ---------------------------------------------------------------- vec.zig


def test_l2sq_hand_checked(orc):
    # src/util/vec.zig:367-372
    assert orc.l2sq([1, 2, 3], [4, 6, 3]) == 25.0
    # :374-377
    a = [0.5, -0.5, 0.25, -0.25, 1.0]
    assert orc.l2sq(a, a) == 0.0
    # :379-388 (tail beyond the SIMD lane)
    assert orc.l2sq(np.arange(9), np.arange(1, 10)) == 9.0
    # :513-519 (dim 4)
    assert orc.l2sq([1, 2, 3, 4], [5, 6, 7, 8]) == 64.0


def test_l2sq_specialisation_parity(orc):
    # src/util/vec.zig:537-550 and :570-583: comptime dims agree with a
    # scalar left fold within 1e-5, and are symmetric.
    i = np.arange(64, dtype=np.float32)
    a = i * np.float32(0.03) - np.float32(0.1)
    b = ((i * 7) % 64) * np.float32(0.005)
    ref = np.float32(0)
    for x, y in zip(a, b):
        d = np.float32(x - y)
        ref = np.float32(ref + np.float32(d * d))
    assert abs(orc.l2sq(a, b) - ref) <= 1e-5
    assert orc.l2sq(a, b) == orc.l2sq(b, a)
    i = np.arange(128, dtype=np.float32)
    a = i * np.float32(0.02)
    b = (127 - i) * np.float32(0.02)
    ref = float(np.sum((a.astype(np.float64) - b) ** 2))
    assert abs(orc.l2sq(a, b) - ref) <= 1e-5 * max(1.0, ref)


def test_l2sq_wide_order_is_four_strided_lanes(orc):
    # vec.zig:142-155: four strided accumulators, then the lane reduction.
    rng = np.random.default_rng(3)
    a = rng.standard_normal(64).astype(np.float32)
    b = rng.standard_normal(64).astype(np.float32)
    acc = [np.float32(0)] * 4
    for q in range(0, 64, 4):
        for l in range(4):
            d = np.float32(a[q + l] - b[q + l])
            acc[l] = np.float32(acc[l] + np.float32(d * d))
    seq = np.float32(np.float32(np.float32(acc[0] + acc[1]) + acc[2]) + acc[3])
    tree = np.float32(np.float32(acc[0] + acc[1]) + np.float32(acc[2] + acc[3]))
    assert orc.l2sq(a, b) == seq
    orc.set_reduce_tree(True)
    try:
        assert orc.l2sq(a, b) == tree
    finally:
        orc.set_reduce_tree(False)


def test_argmin_argmax(orc):
    # src/util/vec.zig:420-438
    assert orc.argmin([3.0, 1.5, 4.0, -2.0, 7.0]) == 3
    assert orc.argmin([1.0, 1.0, 2.0]) == 0  # ties pick first
    assert orc.argmin([]) == -1  # EmptyInput
    assert orc.argmax([-3.0, 1.5, 4.0, -2.0, 7.0]) == 4


# ---------------------------------------------------------------- rng.zig


def test_splitmix_seeding_matches_published_vectors(orc):
    # Rng.init(seed) fills Xoshiro256's state with SplitMix64 outputs; the
    # first three SplitMix64 outputs for seed 0 are the published reference
    # values of the algorithm.
    r = orc.Rng(0)
    assert list(r.state)[:3] == [0xE220A8397B1DCDAF, 0x6E789E6AA1B965F4, 0x06C45D188009454F]


def test_rng_determinism_and_ranges(orc):
    # src/util/rng.zig:104-129
    a, b = orc.Rng(42), orc.Rng(42)
    assert [a.index(1000) for _ in range(32)] == [b.index(1000) for _ in range(32)]
    a, b = orc.Rng(1), orc.Rng(2)
    assert any(a.index(1_000_000) != b.index(1_000_000) for _ in range(16))
    r = orc.Rng(7)
    for _ in range(256):
        x = r.f32()
        assert 0.0 <= x < 1.0
        y = r.f64()
        assert 0.0 <= y < 1.0


def test_weighted_sample(orc):
    # src/util/rng.zig:131-190
    w = [0.1, 0.2, 0.3, 0.4]
    r1, r2 = orc.Rng(123), orc.Rng(123)
    assert [r1.weighted_sample(w) for _ in range(32)] == [r2.weighted_sample(w) for _ in range(32)]
    r = orc.Rng(99)
    assert all(r.weighted_sample([0.0, 1.0, 0.0, 0.0, 2.0]) in (1, 4) for _ in range(256))
    r = orc.Rng(2026)
    counts = np.bincount([r.weighted_sample([0.1, 0.3, 0.6]) for _ in range(10_000)], minlength=3)
    assert 800 < counts[0] < 1200 and 2700 < counts[1] < 3300 and 5600 < counts[2] < 6400
    for bad, code in (([], 8), ([0.0, 0.0, 0.0], 10), ([0.5, -0.1, 0.3], 9), ([0.5, math.nan, 0.3], 9)):
        with pytest.raises(orc.OracleError) as e:
            orc.Rng(0).weighted_sample(bad)
        assert e.value.code == code


# ------------------------------------------------------------- kmeans.zig


def test_kmeans_errors_and_degenerate(orc):
    # src/tac/kmeans.zig:373-407
    for args, code in ((([1, 0, 0, 1], 2, 0), 1), (([], 2, 1), 2), (([1, 2, 3], 2, 1), 3)):
        with pytest.raises(orc.OracleError) as e:
            orc.kmeans_fit(args[0], args[1], args[2], seed=0)
        assert e.value.code == code
    r = orc.kmeans_fit([1, 0, 0, 1], 2, 4, seed=0)
    assert r.wcss == 0.0 and r.iters_run == 0 and list(r.assignments) == [0, 1]
    r = orc.kmeans_fit([1, 0, 0, 1, 1, 1], 2, 3, seed=0)
    assert r.wcss == 0.0 and r.iters_run == 0


def _blobs(centers, offsets):
    pts = []
    for c in centers:
        for o in offsets:
            pts.append((np.float32(c[0]) + np.float32(o[0]), np.float32(c[1]) + np.float32(o[1])))
    return np.array(pts, dtype=np.float32)


OFF6 = [(-0.05, 0.02), (0.03, -0.04), (-0.01, -0.02), (0.02, 0.05), (-0.03, 0.01), (0.04, -0.03)]


def test_kmeans_recovers_blobs(orc):
    # src/tac/kmeans.zig:409-447
    centers = [(0, 0), (10, 0), (0, 10)]
    r = orc.kmeans_fit(_blobs(centers, OFF6), 2, 3, seed=42, max_iters=50)
    c = r.centroids.reshape(3, 2)
    for bc in centers:
        assert min(np.hypot(*(c[j] - bc)) for j in range(3)) < 0.1


def test_kmeans_threads_byte_equal(orc):
    # src/tac/kmeans.zig:449-485 and :628-664
    buf = np.random.default_rng(0xDE7E2).standard_normal(600 * 4).astype(np.float32)
    r1 = orc.kmeans_fit(buf, 4, 32, seed=42, n_threads=1)
    for t in (3, 10, 64, 256):
        rt = orc.kmeans_fit(buf, 4, 32, seed=42, n_threads=t)
        assert rt.centroids.tobytes() == r1.centroids.tobytes()
        assert np.array_equal(rt.assignments, r1.assignments)
        assert rt.wcss == r1.wcss and rt.iters_run == r1.iters_run
    small = buf[: 5 * 4]
    assert orc.kmeans_fit(small, 4, 3, seed=7, n_threads=1).centroids.tobytes() == \
        orc.kmeans_fit(small, 4, 3, seed=7, n_threads=64).centroids.tobytes()


def test_kmeans_deterministic_and_monotone(orc):
    # src/tac/kmeans.zig:487-521
    pts = np.random.default_rng(99).standard_normal(40).astype(np.float32)
    a = orc.kmeans_fit(pts, 2, 4, seed=7, max_iters=30)
    b = orc.kmeans_fit(pts, 2, 4, seed=7, max_iters=30)
    assert a.centroids.tobytes() == b.centroids.tobytes() and a.wcss == b.wcss
    pts = np.random.default_rng(1234).standard_normal(60).astype(np.float32)
    w = [orc.kmeans_fit(pts, 3, 4, seed=111, max_iters=m, tol=0.0).wcss for m in (1, 5, 25)]
    assert w[1] <= w[0] and w[2] <= w[1]


def test_kmeans_assignments_valid_and_reseed(orc):
    # src/tac/kmeans.zig:523-543
    pts = np.random.default_rng(5).standard_normal(50).astype(np.float32)
    r = orc.kmeans_fit(pts, 5, 3, seed=0)
    assert r.assignments.size == 10 and (r.assignments < 3).all()
    r = orc.kmeans_fit([0.0, 0.0, 0.0001, 0.0, 100.0, 0.0], 2, 3, seed=1, max_iters=10)
    assert (r.assignments < 3).all()


def _check_lloyd_invariants(orc, pts, dim, r, k):
    n = pts.size // dim
    x = pts.reshape(n, dim)
    c = r.centroids.reshape(k, dim)
    for i in range(n):
        mine = orc.l2sq(x[i], c[r.assignments[i]])
        assert all(mine <= orc.l2sq(x[i], c[j]) for j in range(k))
    sums = np.zeros((k, dim), dtype=np.float32)
    counts = np.zeros(k, dtype=np.uint32)
    for i in range(n):
        a = r.assignments[i]
        for d in range(dim):
            sums[a, d] = np.float32(sums[a, d] + x[i, d])
        counts[a] += 1
    for j in range(k):
        if counts[j]:
            inv = np.float32(np.float32(1.0) / np.float32(counts[j]))
            assert (sums[j] * inv).astype(np.float32).tobytes() == c[j].tobytes()


def test_kmeans_lloyd_invariants(orc):
    # src/tac/kmeans.zig:545-626 (bit-exact in-order means) and :666-708
    centers = [(0, 0), (50, 0), (0, 50), (-50, 0), (0, -50)]
    off8 = OFF6 + [(0.0, 0.0), (0.01, -0.01)]
    pts = _blobs(centers, off8).reshape(-1)
    r = orc.kmeans_fit(pts, 2, 5, seed=7, max_iters=50)
    _check_lloyd_invariants(orc, pts, 2, r, 5)
    pts = np.array([0.00, 0.00, 0.01, -0.01, -0.02, 0.01, 0.01, 0.02, -0.01, -0.02, 0.00, 0.01,
                    100.0, 100.0, 99.99, 100.01, 100.02, 99.98, 100.01, 99.99, 99.98, 100.02, 100.0,
                    100.0], dtype=np.float32)
    r = orc.kmeans_fit(pts, 2, 2, seed=3, max_iters=25)
    assert r.iters_run <= 5
    _check_lloyd_invariants(orc, pts, 2, r, 2)


# ----------------------------------------------------------------- pq.zig


def test_pq_errors(orc):
    # src/index/pq.zig:357-370
    with pytest.raises(orc.OracleError) as e:
        orc.pq_train(np.zeros(33), 33, 1, pq_m=32)
    assert e.value.code == 4
    with pytest.raises(orc.OracleError) as e:
        orc.pq_train(np.zeros(0), 32, 1, pq_m=32)
    assert e.value.code == 5


def _unit(n, dim, seed, scale=1.0):
    x = np.random.default_rng(seed).standard_normal((n, dim)).astype(np.float32)
    if scale is None:
        return x
    return (x / np.linalg.norm(x, axis=1, keepdims=True)).astype(np.float32)


def test_pq_roundtrip_and_mse(orc):
    # src/index/pq.zig:372-444
    buf = _unit(300, 32, 0x52017)
    cb = orc.pq_train(buf, 32, 17, pq_m=32)
    assert cb.size == 32 * 256
    codes = orc.pq_encode(cb, 32, 32, buf[0])
    dec = np.array([cb[m * 256 + int(codes[0, m])] for m in range(32)], dtype=np.float32)
    assert np.array_equal(orc.pq_encode(cb, 32, 32, dec), codes)
    g = (np.random.default_rng(0xC0DE).standard_normal((1024, 32)) * 0.1).astype(np.float32)
    cb = orc.pq_train(g, 32, 7, pq_m=32)
    codes = orc.pq_encode(cb, 32, 32, g)
    dec = cb.reshape(32, 256)[np.arange(32)[None, :], codes]
    assert float(np.mean((dec - g) ** 2)) < 1e-3


def test_pq_threads_byte_equal(orc):
    # src/index/pq.zig:446-517
    buf = _unit(512, 32, 0xA701C)
    p1 = orc.pq_train(buf, 32, 4242, pq_m=32, n_threads=1)
    for t in (4, 10, 64):
        assert orc.pq_train(buf, 32, 4242, pq_m=32, n_threads=t).tobytes() == p1.tobytes()
    buf = np.random.default_rng(99).standard_normal(300 * 32).astype(np.float32)
    assert orc.pq_train(buf, 32, 1234, pq_m=32).tobytes() == orc.pq_train(buf, 32, 1234, pq_m=32).tobytes()


# ---------------------------------------------------------------- tac.zig


def test_tac_allocate_tail(orc):
    # src/tac/tac.zig:856-880
    k, b = orc.tac_allocate_tail([0, 1, 2, 3, 4, 5, 6, 7], 50, 3, 5)
    assert b == 44 and list(k) == [0, 1, 1, 2, 2, 0, 0, 0]
    with pytest.raises(orc.OracleError) as e:
        orc.tac_allocate_tail([1, 1, 4], 3, 3, 5)
    assert e.value.code == 11
    for mu, tau in ((5, 5), (6, 5), (0, 5)):
        with pytest.raises(orc.OracleError) as e:
            orc.tac_allocate_tail([1], 10, mu, tau)
        assert e.value.code == 13


def test_tac_damped_phase2(orc):
    # src/tac/tac.zig:889-945
    k, f = orc.tac_damped_phase2([9, 16], [2.0, 2.0], [0, 0], 70, 3, 5)
    assert list(k) == [30, 40] and abs(f[0]) < 1e-3 and abs(f[1]) < 1e-3
    k, _ = orc.tac_damped_phase2([25, 25], [1.0, 4.0], [0, 0], 100, 3, 5)
    assert list(k) == [20, 80]
    k, _ = orc.tac_damped_phase2([10, 10, 10], [0.0, 0.0, 0.0], [0, 0, 0], 11, 3, 5)
    assert list(k) == [4, 4, 3]
    k, f = orc.tac_damped_phase2([9, 16], [1.0, 1.0], [0, 0], 10, 3, 5)
    assert list(k) == [4, 5] and abs(f[0] - 0.2857) < 1e-3 and abs(f[1] - 0.7143) < 1e-3


def test_tac_bound_phase3(orc):
    # src/tac/tac.zig:947-980
    assert list(orc.tac_bound_phase3([200], [1], 128, 156, 4, 39)) == [4]
    assert list(orc.tac_bound_phase3([156], [10], 128, 156, 4, 39)) == [4]
    assert list(orc.tac_bound_phase3([50, 200, 500], [1, 2, 1], 128, 256, 4, 39)) == [1, 2, 4]
    with pytest.raises(orc.OracleError) as e:
        orc.tac_bound_phase3([100], [0], 50, 100, 4, 39)
    assert e.value.code == 13


def test_tac_reconcile_phase4(orc):
    # src/tac/tac.zig:982-1039
    assert list(orc.tac_reconcile_phase4([10_000, 10_000], [4, 5], [0.3, 0.8], 12, 3, 5, 4, 39)) == [4, 8]
    assert list(orc.tac_reconcile_phase4([10_000, 10_000], [10, 8], [0.1, 0.6], 14, 3, 5, 4, 39)) == [6, 8]
    assert list(orc.tac_reconcile_phase4([10_000, 10_000], [10, 5], [0.0, 0.9], 8, 3, 5, 4, 39)) == [4, 4]
    with pytest.raises(orc.OracleError) as e:
        orc.tac_reconcile_phase4([156], [4], [0.5], 10, 128, 156, 4, 39)
    assert e.value.code == 12
    assert list(orc.tac_reconcile_phase4([200, 10_000], [2, 4], [0.0, 0.0], 5, 128, 256, 4, 39)) == [1, 4]


def test_tac_allocate_budgets(orc):
    # src/tac/tac.zig:1041-1125
    k = orc.tac_allocate_budgets([0, 2, 4, 20, 20, 20], [0, 0, 0, 1.0, 2.0, 3.0], 18, 3, 5, 4, 1)
    assert list(k) == [0, 1, 2, 4, 4, 7]
    k = orc.tac_allocate_budgets([50, 200, 5000, 5000], [0, 0, 1.0, 2.0], 100)
    assert k.sum() == 100 and k[0] == 1 and k[1] == 2 and 4 <= k[2] <= 128 and 4 <= k[3] <= 128
    assert k[3] >= k[2]
    a = orc.tac_allocate_budgets([0, 100, 250, 1000, 5000], [0, 0, 0, 0.7, 2.3], 50)
    b = orc.tac_allocate_budgets([0, 100, 250, 1000, 5000], [0, 0, 0, 0.7, 2.3], 50)
    assert np.array_equal(a, b)


def test_tac_cluster_flat_tiny(orc):
    # src/tac/tac.zig:1131-1182
    rng = np.random.default_rng(7)
    counts = [10, 10, 6, 4]
    themes = [(1, 0), (0, 1), (-1, 0), (0, -1)]
    ids, vec = [], []
    for tid, c in enumerate(counts):
        for _ in range(c):
            ids.append(tid)
            vec.append([themes[tid][0] + rng.standard_normal() * 0.05, themes[tid][1] + rng.standard_normal() * 0.05])
    r = orc.tac_cluster_flat(ids, np.array(vec, np.float32), 2, 14, 42, mu=3, tau=5, eps=1, theta=1)
    assert r.kappa_per_token.sum() == 14 and r.kappa_per_token[3] == 2
    assert (r.assignments < 14).all() and r.assignments.size == 30 and r.centroids.size == 28
    assert math.isfinite(r.wcss_total) and r.wcss_total >= 0


def test_tac_cluster_flat_absent_token_and_themes(orc):
    # src/tac/tac.zig:1218-1306
    ids = [1, 1, 1, 1, 2, 2, 2, 2, 3, 3, 3, 3]
    v = [0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8, 0.9, 1.0, 1.1, 1.2]
    r = orc.tac_cluster_flat(ids, v, 1, 6, 0, mu=3, tau=5, eps=1, theta=1)
    assert list(r.kappa_per_token) == [0, 2, 2, 2]
    themes = [(10, 0), (0, 10), (-10, 0)]
    rng = np.random.default_rng(99)
    ids, vec = [], []
    for tid, t in enumerate(themes):
        for _ in range(6):
            ids.append(tid)
            vec.append([t[0] + rng.standard_normal() * 0.05, t[1] + rng.standard_normal() * 0.05])
    r = orc.tac_cluster_flat(ids, np.array(vec, np.float32), 2, 3, 0, mu=2, tau=5, eps=1, theta=1)
    assert list(r.kappa_per_token) == [1, 1, 1]
    for j, t in enumerate(themes):
        assert abs(r.centroids[2 * j] - t[0]) < 0.1 and abs(r.centroids[2 * j + 1] - t[1]) < 0.1
    assert list(r.assignments) == ids


def test_tac_cluster_flat_errors(orc):
    # src/tac/tac.zig:1239-1261
    with pytest.raises(orc.OracleError) as e:
        orc.tac_cluster_flat(np.zeros(0, np.uint32), np.zeros(0, np.float32), 2, 1, 0)
    assert e.value.code == 14
    with pytest.raises(orc.OracleError) as e:
        orc.tac_cluster_flat([0, 0], [1, 0, 0, 1], 2, 0, 0)
    assert e.value.code == 11
    with pytest.raises(orc.OracleError) as e:
        orc.tac_cluster_flat([0, 0, 0], [1, 0, 0, 1], 2, 4, 0)
    assert e.value.code == 13


def test_residuals_norms(orc):
    # src/index/storage.zig:255-278
    v = np.array([[3.0, 4.0], [1.0, 1.0]], np.float32)
    c = np.array([[0.0, 0.0], [1.0, 1.0]], np.float32)
    r, n = orc.residuals_norms(v, c, [0, 1], 2)
    assert list(n) == [5.0, 0.0]
    assert abs(r[0] - 0.6) < 1e-6 and abs(r[1] - 0.8) < 1e-6 and r[2] == 0 and r[3] == 0


def test_doc_layouts_round_trip(orc):
    # storage.zig:1116-1194 (round-trip of every section), restated for the
    # per-doc section: parse the index and each [n_d | ids | codes | pad]
    rng = np.random.default_rng(11)
    m = 16
    n_d = [3, 0, 5, 1, 0, 8]
    off = np.concatenate([[0], np.cumsum(n_d)]).astype(np.uint64)
    n = int(off[-1])
    asg = rng.integers(0, 2**32 - 1, size=n, dtype=np.uint64).astype(np.uint32)
    codes = rng.integers(0, 256, size=(n, m), dtype=np.uint8)
    b = orc.write_doc_layouts(off, asg, codes, m)
    nd = len(n_d)
    idx = np.frombuffer(b[: (nd + 1) * 8], dtype=np.uint64)
    base = (nd + 1) * 8
    for d in range(nd):
        p = base + int(idx[d])
        assert p % 8 == 0
        k = int(np.frombuffer(b[p:p + 4], dtype=np.uint32)[0])
        assert k == n_d[d]
        ids = np.frombuffer(b[p + 4:p + 4 + 4 * k], dtype=np.uint32)
        assert np.array_equal(ids, asg[off[d]:off[d + 1]])
        cds = np.frombuffer(b[p + 4 + 4 * k:p + 4 + 4 * k + m * k], dtype=np.uint8)
        assert np.array_equal(cds, codes[off[d]:off[d + 1]].reshape(-1))
        end = base + int(idx[d + 1])
        assert end - p == (4 + k * (4 + m) + 7) // 8 * 8
        assert not any(b[p + 4 + k * (4 + m):end])
    assert len(b) == base + int(idx[nd])


def test_dot_reference_kats(orc):
    # src/util/vec.zig:334-358 and :497-509 (exact where the reference uses
    # expectEqual), :521-575 (ramps, within the reference's 1e-5)
    assert orc.dot([1, 2, 3], [4, -5, 6]) == 12.0
    a = np.arange(1, 18, dtype=np.float32)
    assert orc.dot(a, np.full(17, 2, np.float32)) == 306.0
    assert orc.dot([1, 0, 0, 0], [0, 1, 0, 0]) == 0.0
    assert orc.dot([1, 2], [3, 4]) == 11.0
    assert orc.dot([1, 2, 3, 4], [5, 6, 7, 8]) == 70.0
    i = np.arange(64, dtype=np.float32)
    a, b = i * np.float32(0.01), (63 - i) * np.float32(0.02) + np.float32(0.5)
    assert abs(orc.dot(a, b) - float(np.dot(a.astype(np.float64), b.astype(np.float64)))) < 1e-4
    i = np.arange(128, dtype=np.float32)
    a, b = i * np.float32(0.005) - np.float32(0.3), ((i * 13 + 1) % 128) * np.float32(0.01)
    assert abs(orc.dot(a, b) - float(np.dot(a.astype(np.float64), b.astype(np.float64)))) < 1e-4


def test_distance_table_layout(orc):
    # src/index/pq.zig:344-349, :519-575: table[m][c][i] is the dot product of
    # query token i's sub-vector m with codeword (m, c); bad sizes fail
    rng = np.random.default_rng(1)
    cb = rng.standard_normal(16 * 256 * 4).astype(np.float32)
    q = rng.standard_normal((3, 64)).astype(np.float32)
    t = orc.pq_distance_table(cb, 64, 16, q, 3).reshape(16, 256, 3)
    for m, c, i in [(0, 0, 0), (5, 200, 2), (15, 255, 1)]:
        assert t[m, c, i] == orc.dot(q[i, m * 4:(m + 1) * 4], cb.reshape(16, 256, 4)[m, c])
    with pytest.raises(Exception):
        orc.pq_distance_table(cb, 64, 16, q, 4)
