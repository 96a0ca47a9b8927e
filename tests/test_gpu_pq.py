"""GPU parity of PQ encode / pq.train / kmeans.fit against the CPU oracle.

Bar: bit-exact. Codes and assignments are integers (exact equality); codebooks,
centroids and WCSS are compared byte for byte, which is stricter than the
1e-5 relative tolerance the specification allows for trained codebooks.
"""
import math
import os

import numpy as np
import pytest

from ir_multivector_retrieval_b200 import kmeans, pq, synth
from ir_multivector_retrieval_b200._lib import MvrError

pytestmark = pytest.mark.gpu
THREADS = max(1, os.cpu_count() or 1)


def _rows(n, dim, seed):
    return synth.unit_rows(n, dim, seed)


@pytest.mark.parametrize("dim,m", [(64, 16), (64, 32), (32, 32), (128, 32), (12, 3), (8, 8)])
def test_encode_bitexact(ctx, orc, dim, m):
    rng = np.random.default_rng(dim * 100 + m)
    cb = rng.standard_normal(m * 256 * (dim // m)).astype(np.float32)
    x = _rows(10_007, dim, seed=m)
    p = pq.PQ(dim=dim, sub_dim=dim // m, codebooks=cb, pq_m=m, ctx=ctx)
    got = p.encode_batch(x)
    want = orc.pq_encode(cb, dim, m, x, n_threads=THREADS)
    assert np.array_equal(got, want)
    assert np.array_equal(p.encode(x[5]), want[5])


def test_encode_ties_and_exact_codewords(ctx, orc):
    rng = np.random.default_rng(3)
    cb = rng.standard_normal(16 * 256 * 4).astype(np.float32).reshape(16, 256, 4)
    cb[:, 200] = cb[:, 5]  # duplicate codeword: the first index must win
    cb[:, 17] = cb[:, 16]
    cb = cb.reshape(-1)
    p = pq.PQ(dim=64, sub_dim=4, codebooks=cb, pq_m=16, ctx=ctx)
    codes = rng.integers(0, 256, size=(4096, 16), dtype=np.uint8)
    x = p.decode(codes)
    got = p.encode_batch(x)
    want = orc.pq_encode(cb, 64, 16, x, n_threads=THREADS)
    assert np.array_equal(got, want)
    assert not np.any(got == 200) and not np.any(got == 17)
    # idempotence: encode(decode(c)) == c where codewords are distinct
    assert np.array_equal(p.encode_batch(p.decode(got)), got)


def test_encode_nonfinite_rows(ctx, orc):
    rng = np.random.default_rng(4)
    cb = rng.standard_normal(16 * 256 * 4).astype(np.float32)
    x = _rows(600, 64, 9)
    x[3, 5] = np.nan
    x[7, :] = np.inf
    x[11, 0:4] = -np.inf
    cbn = cb.copy()
    cbn[4 * 3] = np.nan  # codeword 3 of subspace 0 has a NaN
    for c in (cb, cbn):
        got = pq.PQ(dim=64, sub_dim=4, codebooks=c, pq_m=16, ctx=ctx).encode_batch(x)
        assert np.array_equal(got, orc.pq_encode(c, 64, 16, x))


def test_encode_errors(ctx):
    p = pq.PQ(dim=64, sub_dim=4, codebooks=np.zeros(16 * 256 * 4, np.float32), pq_m=16, ctx=ctx)
    with pytest.raises(MvrError) as e:
        p.encode(np.zeros(63, np.float32))
    assert e.value.name == "DimMismatch"
    assert p.encode_batch(np.zeros((0, 64), np.float32)).shape == (0, 16)


@pytest.mark.parametrize("dim,m,n,iters,tol", [
    (64, 16, 6000, 20, -math.inf),
    (64, 16, 6000, 25, 1e-4),
    (64, 32, 5000, 25, 1e-4),
    (32, 32, 3000, 25, 1e-4),
    (128, 32, 2500, 10, -math.inf),
    (12, 3, 4096, 25, 1e-4),
])
def test_pq_train_bitexact(ctx, orc, dim, m, n, iters, tol):
    x = _rows(n, dim, seed=n + m)
    stats = {}
    got = pq.train(x, dim, 0xA1B2C3D4 + 42, 1, pq_m=m, max_iters=iters, tol=tol, ctx=ctx, stats=stats)
    want = orc.pq_train(x, dim, 0xA1B2C3D4 + 42, m, n_threads=THREADS, max_iters=iters, tol=tol)
    assert got.codebooks.tobytes() == want.tobytes()
    assert stats["iters_max"] <= iters
    if tol == -math.inf:
        assert stats["iters_min"] == iters


@pytest.mark.parametrize("n", [1, 200, 256, 257, 300])
def test_pq_train_small_corpora(ctx, orc, n):
    x = _rows(n, 64, seed=n)
    got = pq.train(x, 64, 7, pq_m=16, ctx=ctx)
    assert got.codebooks.tobytes() == orc.pq_train(x, 64, 7, 16).tobytes()


def test_pq_train_errors(ctx):
    for args, name in (((np.zeros(33, np.float32), 33), "DimNotDivisibleByM"),
                       ((np.zeros(0, np.float32), 32), "EmptyCorpus"),
                       ((np.zeros(65, np.float32), 64), "DimMismatch")):
        with pytest.raises(MvrError) as e:
            pq.train(args[0], args[1], 1, pq_m=32 if args[1] != 64 else 16, ctx=ctx)
        assert e.value.name == name
    # fewer distinct sub-vectors than 256 with n > 256: k-means++ runs out of
    # positive weights, weightedSample -> AllZero (src/util/rng.zig:65)
    x = np.tile(_rows(10, 64, 1), (40, 1))
    with pytest.raises(MvrError) as e:
        pq.train(x, 64, 1, pq_m=16, ctx=ctx)
    assert e.value.name == "AllZero"
    x = _rows(400, 64, 2)
    x[17, 3] = np.nan
    with pytest.raises(MvrError) as e:
        pq.train(x, 64, 1, pq_m=16, ctx=ctx)
    assert e.value.name == "NonFinite"


@pytest.mark.parametrize("dim", [1, 2, 4])
@pytest.mark.parametrize("k", [1, 2, 7, 64, 256])
def test_kmeans_fit_bitexact(ctx, orc, dim, k):
    x = np.random.default_rng(dim * 1000 + k).standard_normal(3000 * dim).astype(np.float32)
    for iters, tol in ((25, 1e-4), (12, 0.0), (7, -math.inf)):
        got = kmeans.fit(x, dim, kmeans.KMeansParams(k=k, seed=99 + k, max_iters=iters, tol=tol), ctx=ctx)
        want = orc.kmeans_fit(x, dim, k, 99 + k, max_iters=iters, tol=tol, n_threads=THREADS)
        assert got.centroids.tobytes() == want.centroids.tobytes()
        assert np.array_equal(got.assignments, want.assignments)
        assert got.iters_run == want.iters_run
        assert np.float32(got.wcss).tobytes() == np.float32(want.wcss).tobytes()


def test_kmeans_reference_fixtures(ctx, orc):
    # blobs (src/tac/kmeans.zig:409-447), collinear reseed (:535-543),
    # early break (:666-708), degenerate k >= n (:391-407)
    centers = [(0, 0), (10, 0), (0, 10)]
    off = [(-0.05, 0.02), (0.03, -0.04), (-0.01, -0.02), (0.02, 0.05), (-0.03, 0.01), (0.04, -0.03)]
    pts = np.array([(c[0] + o[0], c[1] + o[1]) for c in centers for o in off], np.float32)
    cases = [(pts, 2, 3, 42, 50), (np.array([0, 0, 0.0001, 0, 100, 0], np.float32), 2, 3, 1, 10),
             (np.array([1, 0, 0, 1], np.float32), 2, 4, 0, 25), (np.array([1, 0, 0, 1, 1, 1], np.float32), 2, 3, 0, 25)]
    for x, dim, k, seed, iters in cases:
        got = kmeans.fit(x, dim, kmeans.KMeansParams(k=k, seed=seed, max_iters=iters), ctx=ctx)
        want = orc.kmeans_fit(x, dim, k, seed, max_iters=iters)
        assert got.centroids.tobytes() == want.centroids.tobytes()
        assert np.array_equal(got.assignments, want.assignments)
        assert got.iters_run == want.iters_run and got.wcss == want.wcss


def test_device_pointer_entry_points(ctx, orc):
    torch = pytest.importorskip("torch")
    import ctypes as C

    from ir_multivector_retrieval_b200._lib import PqTrainStats

    x = _rows(20_000, 64, 5)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        dx = torch.from_numpy(x).cuda()
        dcb = torch.empty(16 * 256 * 4, dtype=torch.float32, device="cuda")
    st = PqTrainStats()
    ctx.set_stream(s.cuda_stream)
    try:
        ctx.check(ctx.lib.mvr_pq_train_device(ctx.handle, C.c_void_p(dx.data_ptr()), x.size, 64, 11, 1, 16,
                                              8, C.c_float(-math.inf), C.c_void_p(dcb.data_ptr()), C.byref(st)))
        with torch.cuda.stream(s):
            codes = torch.empty((20_000, 16), dtype=torch.uint8, device="cuda")
        ctx.check(ctx.lib.mvr_pq_encode_device(ctx.handle, C.c_void_p(dcb.data_ptr()), 64, 16,
                                               C.c_void_p(dx.data_ptr()), 20_000, C.c_void_p(codes.data_ptr())))
        ctx.sync()
    finally:
        ctx.set_stream(None)
    cb = dcb.cpu().numpy()
    want_cb = orc.pq_train(x, 64, 11, 16, n_threads=THREADS, max_iters=8, tol=-math.inf)
    assert cb.tobytes() == want_cb.tobytes()
    assert np.array_equal(codes.cpu().numpy(), orc.pq_encode(cb, 64, 16, x, n_threads=THREADS))
    assert st.iters_max == 8 and st.total_ms > 0


def _seq4(v):
    q = (v.astype(np.float32) ** 2).astype(np.float32)
    return np.float32(np.float32(np.float32(q[0] + q[1]) + q[2]) + q[3])


def test_encode_rounding_order_sensitive_ties(ctx, orc):
    """Codeword pairs whose ranking is decided only by the rounding order of
    the distance sum: for the zero row, c_a = (p,q,r,s) and c_b = (r,s,p,q)
    have the same exact distance and the same pairwise-tree sum, but their
    left-fold sums (the reference order) differ. A kernel that sums in any
    other order, or fuses the squares into FMAs, picks differently."""
    rng = np.random.default_rng(17)
    cases = []
    while len(cases) < 16 * 48:
        a = rng.standard_normal(4).astype(np.float32) * np.float32(rng.choice([1e-3, 1.0, 30.0]))
        b = a[[2, 3, 0, 1]]
        if _seq4(a) != _seq4(b):
            cases.append((a, b))
    x = np.zeros((3, 64), np.float32)
    for call in range(48):
        cb = np.full((16, 256, 4), 1e4, np.float32)
        for m in range(16):
            a, b = cases[call * 16 + m]
            cb[m, 0], cb[m, 1] = a, b
        cb = cb.reshape(-1)
        got = pq.PQ(dim=64, sub_dim=4, codebooks=cb, pq_m=16, ctx=ctx).encode_batch(x)
        want = orc.pq_encode(cb, 64, 16, x)
        assert np.array_equal(got, want)
        assert set(np.unique(want)) <= {0, 1} and len(np.unique(want)) == 2


def test_encode_one_ulp_codewords(ctx, orc):
    """Neighbouring codewords one ulp apart in one coordinate: distances that
    differ only in their last bits."""
    rng = np.random.default_rng(23)
    base = rng.standard_normal((16, 128, 4)).astype(np.float32)
    twin = base.copy()
    k = rng.integers(0, 4, size=(16, 128))
    for m in range(16):
        for c in range(128):
            twin[m, c, k[m, c]] = np.nextafter(twin[m, c, k[m, c]], np.float32(np.inf))
    cb = np.stack([base, twin], axis=2).reshape(-1)  # codeword 2c and 2c+1 are twins
    x = (base[:, rng.integers(0, 128, 50_000)].transpose(1, 0, 2)
         + rng.standard_normal((50_000, 16, 4)).astype(np.float32) * np.float32(1e-3)).reshape(50_000, 64)
    got = pq.PQ(dim=64, sub_dim=4, codebooks=cb, pq_m=16, ctx=ctx).encode_batch(x)
    assert np.array_equal(got, orc.pq_encode(cb, 64, 16, x, n_threads=THREADS))


@pytest.mark.parametrize("trial,S", [(1247, 4), (2902, 2), (612, 1)])
def test_empty_cluster_reseed_matches_oracle(ctx, orc, trial, S):
    """Seeded data whose Lloyd iterations empty a cluster (kmeans.zig:199-211):
    pq.train with pq_m = 1 reseeds it exactly as the oracle does."""
    rng = np.random.default_rng(trial)
    n = int(rng.integers(260, 2000))
    if trial == 612:
        x = rng.standard_normal((n, S)).astype(np.float32)
    else:
        x = (rng.uniform(-1, 1, size=(n, S)) ** 5).astype(np.float32)
    st = {}
    got = pq.train(x, S, trial, pq_m=1, max_iters=25, tol=0.0, ctx=ctx, stats=st)
    want = orc.pq_train(x, S, trial, 1, n_threads=THREADS, max_iters=25, tol=0.0)
    assert st["reseeds"] >= 1
    assert got.codebooks.tobytes() == want.tobytes()


def test_bound_pruning_matches_exhaustive(ctx, orc):
    """Lloyd iterations that skip rows by their distance bounds give the same
    bytes as computing every distance, and as the oracle (fixed iterations,
    tolerance mode and a reseeding case)."""
    x = _rows(40_000, 32, 21)
    for iters, tol in ((20, -math.inf), (25, 1e-4)):
        st_p, st_e = {}, {}
        pruned = pq.train(x, 32, 5, pq_m=8, max_iters=iters, tol=tol, ctx=ctx, stats=st_p)
        ctx.check(ctx.lib.mvr_ctx_set_exhaustive_assign(ctx.handle, 1))
        try:
            full = pq.train(x, 32, 5, pq_m=8, max_iters=iters, tol=tol, ctx=ctx, stats=st_e)
        finally:
            ctx.check(ctx.lib.mvr_ctx_set_exhaustive_assign(ctx.handle, 0))
        assert pruned.codebooks.tobytes() == full.codebooks.tobytes()
        assert st_p["iters_max"] == st_e["iters_max"]
        want = orc.pq_train(x, 32, 5, 8, n_threads=THREADS, max_iters=iters, tol=tol)
        assert pruned.codebooks.tobytes() == want.tobytes()


def test_candidate_scan_matches_full_scans(ctx, orc):
    """Pruned Lloyd passes that scan only the centroids near a row's current
    one give the same bytes as full scans of the failing rows and as the
    oracle, on adversarial sets (exact duplicates, quantised grids with many
    equal distances, magnitudes over many binades, non-finite-free but huge
    rows) and with fewer centroids than the neighbour table (kmeans.fit)."""
    for name, x, dim, m in _filter_datasets():
        for iters, tol in ((12, -math.inf), (25, 1e-4)):
            st_c, st_f = {}, {}
            got = pq.train(x, dim, 9, pq_m=m, max_iters=iters, tol=tol, ctx=ctx, stats=st_c)
            ctx.check(ctx.lib.mvr_ctx_set_candidate_scan(ctx.handle, 0))
            try:
                full = pq.train(x, dim, 9, pq_m=m, max_iters=iters, tol=tol, ctx=ctx, stats=st_f)
            finally:
                ctx.check(ctx.lib.mvr_ctx_set_candidate_scan(ctx.handle, 1))
            assert got.codebooks.tobytes() == full.codebooks.tobytes(), name
            assert st_c["iters_max"] == st_f["iters_max"], name
            want = orc.pq_train(x, dim, 9, m, n_threads=THREADS, max_iters=iters, tol=tol)
            assert got.codebooks.tobytes() == want.tobytes(), name
    for dim, k in ((4, 9), (2, 31), (4, 33), (1, 256)):
        xs = synth.unit_rows(7_000, dim, seed=k) if dim > 1 else \
            np.random.default_rng(k).standard_normal(7_000).astype(np.float32)
        g = kmeans.fit(xs, dim, kmeans.KMeansParams(k=k, seed=k, max_iters=15, tol=-math.inf), ctx=ctx)
        w = orc.kmeans_fit(xs, dim, k, k, max_iters=15, tol=-math.inf)
        assert np.array_equal(g.assignments, w.assignments)
        assert g.centroids.tobytes() == np.ascontiguousarray(w.centroids, dtype=np.float32).tobytes()
        assert np.float32(g.wcss).tobytes() == np.float32(w.wcss).tobytes()


def _filter_report(ctx):
    import ctypes as C

    v, r = C.c_uint64(0), C.c_uint64(0)
    ctx.check(ctx.lib.mvr_ctx_filter_report(ctx.handle, C.byref(v), C.byref(r)))
    return v.value, r.value


def _filter_datasets():
    rng = np.random.default_rng(21)
    base = synth.unit_rows(300, 32, seed=4)
    yield "unit64", _rows(30_011, 64, seed=31), 64, 16
    yield "unit32_s2", _rows(20_000, 32, seed=32), 32, 16
    yield "unit8_s1", _rows(9_000, 8, seed=33), 8, 8
    yield "dup", base[rng.integers(0, 300, size=12_000)], 32, 16  # exact ties, zero distances
    yield "scaled_up", (_rows(8_000, 16, seed=34) * 1e3).astype(np.float32), 16, 4
    yield "scaled_down", (_rows(8_000, 16, seed=35) * 1e-3).astype(np.float32), 16, 4
    mixed = _rows(8_000, 16, seed=36)
    mixed[::7] *= 1e4
    mixed[3::11] *= 1e-5
    yield "mixed", mixed.astype(np.float32), 16, 4
    big = _rows(5_000, 16, seed=37)
    big[::13] *= 1e15  # |x|^2 above 2^60: the exact scan takes these rows
    yield "huge", big.astype(np.float32), 16, 4
    q = (np.round(_rows(6_000, 16, seed=38) * 8) / 8).astype(np.float32)  # a coarse grid: many equal distances
    yield "grid", q, 16, 4


@pytest.mark.parametrize("name,x,dim,m", list(_filter_datasets()), ids=lambda v: v if isinstance(v, str) else "")
def test_tensor_filter_matches_exact_scans(ctx, orc, name, x, dim, m):
    """The tensor-core filtered assignment (switched on for PQ) and the exact
    scans (the PQ default) give the same codebooks and codes, equal to the
    oracle; no winner falls outside the filter's error bound."""
    st_f, st_e = {}, {}
    ctx.check(ctx.lib.mvr_ctx_set_pq_tensor_filter(ctx.handle, 1))
    try:
        f = pq.train(x, dim, 5, pq_m=m, max_iters=8, tol=1e-4, ctx=ctx, stats=st_f)
        codes_f = f.encode_batch(x)
    finally:
        ctx.check(ctx.lib.mvr_ctx_set_pq_tensor_filter(ctx.handle, 0))
    ctx.check(ctx.lib.mvr_ctx_set_tensor_filter(ctx.handle, 0))
    try:
        e = pq.train(x, dim, 5, pq_m=m, max_iters=8, tol=1e-4, ctx=ctx, stats=st_e)
        codes_e = e.encode_batch(x)
    finally:
        ctx.check(ctx.lib.mvr_ctx_set_tensor_filter(ctx.handle, 1))
    want = orc.pq_train(x, dim, 5, m, n_threads=THREADS, max_iters=8, tol=1e-4)
    assert f.codebooks.tobytes() == want.tobytes()
    assert e.codebooks.tobytes() == want.tobytes()
    assert np.array_equal(codes_f, codes_e)
    assert np.array_equal(codes_f, orc.pq_encode(want, dim, m, x, n_threads=THREADS))
    assert st_f["filter_violations"] == 0 and st_e["filter_rows_rechecked"] == 0
    viol, _ = _filter_report(ctx)
    assert viol == 0



def test_host_encode_chunked_matches_device(ctx):
    """mvr_pq_encode with page-locked rows (copied and encoded in chunks that
    overlap) and with pageable rows returns the device entry point's codes."""
    import ctypes as C

    import torch

    n, dim, m = 600_000, 64, 16
    x = synth.unit_rows(n, dim, seed=77).reshape(-1)
    cb = (np.random.default_rng(5).standard_normal(m * 256 * 4) * 0.3).astype(np.float32)
    x_pin = torch.from_numpy(x).pin_memory()
    out_pin = torch.empty(n * m, dtype=torch.uint8).pin_memory()
    ctx.check(ctx.lib.mvr_pq_encode(ctx.handle, C.c_void_p(cb.ctypes.data), dim, m, C.c_void_p(x_pin.data_ptr()),
                                    n, C.c_void_p(out_pin.data_ptr())))
    dx, dcb = x_pin.cuda(), torch.from_numpy(cb).cuda()
    dcodes = torch.empty(n * m, dtype=torch.uint8, device="cuda")
    ctx.check(ctx.lib.mvr_pq_encode_device(ctx.handle, C.c_void_p(dcb.data_ptr()), dim, m, C.c_void_p(dx.data_ptr()),
                                           n, C.c_void_p(dcodes.data_ptr())))
    ctx.sync()
    want = dcodes.cpu().numpy()
    assert np.array_equal(out_pin.numpy(), want)
    p = pq.PQ(dim=dim, sub_dim=4, codebooks=cb, pq_m=m)
    assert np.array_equal(p.encode_batch(x.reshape(n, dim)).reshape(-1), want)


def test_subspace_groups_match_one_group(ctx, orc):
    """pq.train with its subspaces in two groups on two streams (the default)
    gives the bytes of one group and of the oracle, assignments included."""
    import ctypes as C

    from ir_multivector_retrieval_b200._lib import PqTrainStats

    torch = pytest.importorskip("torch")
    x = synth.unit_rows(50_000, 64, seed=31)
    want = orc.pq_train(x, 64, 13, 16, n_threads=8, max_iters=6, tol=-math.inf)
    dx = torch.from_numpy(x).cuda()
    out = {}
    for groups in (1, 2):
        ctx.check(ctx.lib.mvr_ctx_set_pq_groups(ctx.handle, groups))
        cb = torch.empty(16 * 256 * 4, dtype=torch.float32, device="cuda")
        asg = torch.empty(16 * 50_000, dtype=torch.int32, device="cuda")
        st = PqTrainStats()
        torch.cuda.synchronize()
        ctx.check(ctx.lib.mvr_pq_train_sharded_device(ctx.handle, C.c_void_p(dx.data_ptr()), 50_000, 0, 50_000, 64,
                                                      13, 1, 16, 6, C.c_float(-math.inf), C.c_void_p(cb.data_ptr()),
                                                      C.c_void_p(asg.data_ptr()), C.byref(st)))
        assert st.groups == groups
        out[groups] = (cb.cpu().numpy().tobytes(), asg.cpu().numpy().tobytes())
    ctx.check(ctx.lib.mvr_ctx_set_pq_groups(ctx.handle, 2))
    assert out[1] == out[2]
    assert out[2][0] == want.tobytes()
    with pytest.raises(MvrError):
        ctx.check(ctx.lib.mvr_ctx_set_pq_groups(ctx.handle, 3))
