"""GPU parity of tac.clusterFlat and general-dimension kmeans.fit against the
CPU oracle.

Bar: bit-exact. Assignments and kappa_per_token are integers (exact
equality); centroids and WCSS are compared byte for byte.
"""
import numpy as np
import pytest

from ir_multivector_retrieval_b200 import kmeans, synth, tac
from ir_multivector_retrieval_b200._lib import MvrError

pytestmark = pytest.mark.gpu


def _same_bytes(a, b):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return a.shape == b.shape and a.tobytes() == b.tobytes()


def _check_kmeans(ctx, orc, x, dim, k, seed, max_iters, tol):
    got = kmeans.fit(x, dim, kmeans.KMeansParams(k=k, seed=seed, max_iters=max_iters, tol=tol), ctx=ctx)
    want = orc.kmeans_fit(x, dim, k, seed, max_iters=max_iters, tol=tol)
    assert got.iters_run == want.iters_run
    assert np.array_equal(got.assignments, want.assignments)
    assert _same_bytes(got.centroids, want.centroids)
    assert np.float32(got.wcss).tobytes() == np.float32(want.wcss).tobytes()
    return got


# --------------------------------------------------------------- kmeans.fit
@pytest.mark.parametrize("dim", [3, 8, 17, 64, 96, 128, 256])
@pytest.mark.parametrize("k", [1, 2, 9, 64])
def test_kmeans_general_dims(ctx, orc, dim, k):
    x = synth.unit_rows(2_011, dim, seed=dim * 7 + k)
    _check_kmeans(ctx, orc, x, dim, k, seed=k + dim, max_iters=25, tol=1e-4)


@pytest.mark.parametrize("dim,k,tol,iters", [(3, 40, float("-inf"), 7), (64, 33, 0.0, 12), (128, 5, 1e-2, 25)])
def test_kmeans_general_modes(ctx, orc, dim, k, tol, iters):
    x = synth.unit_rows(3_001, dim, seed=5)
    _check_kmeans(ctx, orc, x, dim, k, seed=11, max_iters=iters, tol=tol)


@pytest.mark.parametrize("dim,k", [(2, 257), (4, 300), (1, 600), (64, 700)])
def test_kmeans_more_than_256_centroids(ctx, orc, dim, k):
    if dim == 1:  # unit rows of dim 1 are +-1 only
        x = np.random.default_rng(k).standard_normal(5_000).astype(np.float32)
    else:
        x = synth.unit_rows(5_000, dim, seed=k)
    _check_kmeans(ctx, orc, x, dim, k, seed=3, max_iters=6, tol=1e-4)


def test_kmeans_clustered_with_empty_clusters(ctx, orc):
    # few distinct points, many centroids: duplicates make zero weights and
    # Lloyd steps that empty clusters and reseed them
    rng = np.random.default_rng(0)
    pts = rng.standard_normal((12, 6)).astype(np.float32)
    x = pts[rng.integers(0, 12, size=900)]
    x[::7] += np.float32(1e-3) * rng.standard_normal((x[::7].shape[0], 6)).astype(np.float32)
    _check_kmeans(ctx, orc, x.reshape(-1), 6, 20, seed=8, max_iters=25, tol=1e-4)


def test_kmeans_general_degenerate(ctx, orc):
    x = synth.unit_rows(5, 3, seed=1)
    got = _check_kmeans(ctx, orc, x, 3, 8, seed=0, max_iters=25, tol=1e-4)
    assert list(got.assignments) == [0, 1, 2, 3, 4]
    assert got.wcss == 0.0 and got.iters_run == 0


def test_kmeans_general_errors(ctx, orc):
    x = synth.unit_rows(300, 5, seed=2)
    x[17, 2] = np.inf
    with pytest.raises(MvrError) as e:
        kmeans.fit(x, 5, kmeans.KMeansParams(k=4, seed=1), ctx=ctx)
    assert e.value.name == "NonFinite"
    same = np.tile(np.float32([0.5, -1, 2, 0, 3]), 200)
    with pytest.raises(MvrError) as e:
        kmeans.fit(same, 5, kmeans.KMeansParams(k=3, seed=1), ctx=ctx)
    assert e.value.name == "AllZero"
    with pytest.raises(Exception):
        orc.kmeans_fit(same, 5, 3, 1)
    # the context stays usable after a failing problem
    _check_kmeans(ctx, orc, synth.unit_rows(300, 5, seed=3), 5, 4, seed=1, max_iters=25, tol=1e-4)


# ------------------------------------------------------------ clusterFlat
def _check_cluster(ctx, orc, ids, vec, dim, kappa, seed, **kw):
    p = tac.ClusteringParams(kappa_total=kappa, seed=seed, **kw)
    got = tac.cluster_flat(ids, vec, dim, p, ctx=ctx)
    want = orc.tac_cluster_flat(ids, vec, dim, kappa, seed, mu=p.mu, tau=p.tau, eps=p.epsilon, theta=p.theta,
                                max_iters=p.max_iters, tol=p.tol, n_threads=p.n_threads)
    assert np.array_equal(got.kappa_per_token, want.kappa_per_token)
    assert np.array_equal(got.assignments, want.assignments)
    assert _same_bytes(got.centroids, want.centroids)
    assert np.float32(got.wcss_total).tobytes() == np.float32(want.wcss_total).tobytes()
    return got


def test_cluster_flat_tiny_themes(ctx, orc):
    # the reference's tiny-corpus invariants case (src/tac/tac.zig:1131-1182)
    rng = np.random.default_rng(7)
    counts = [10, 10, 6, 4]
    themes = [(1, 0), (0, 1), (-1, 0), (0, -1)]
    ids, vec = [], []
    for tid, c in enumerate(counts):
        for _ in range(c):
            ids.append(tid)
            vec.append([themes[tid][0] + rng.standard_normal() * 0.05, themes[tid][1] + rng.standard_normal() * 0.05])
    vec = np.array(vec, np.float32)
    got = _check_cluster(ctx, orc, ids, vec, 2, 14, 42, mu=3, tau=5, epsilon=1, theta=1)
    assert got.kappa_per_token.sum() == 14 and got.kappa_per_token[3] == 2
    assert (got.assignments < 14).all()


def test_cluster_flat_absent_token_and_theme_centroids(ctx, orc):
    # src/tac/tac.zig:1218-1306
    ids = [1, 1, 1, 1, 2, 2, 2, 2, 3, 3, 3, 3]
    v = np.float32([0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8, 0.9, 1.0, 1.1, 1.2])
    got = _check_cluster(ctx, orc, ids, v, 1, 6, 0, mu=3, tau=5, epsilon=1, theta=1)
    assert list(got.kappa_per_token) == [0, 2, 2, 2]
    themes = [(10, 0), (0, 10), (-10, 0)]
    rng = np.random.default_rng(99)
    ids, vec = [], []
    for tid, t in enumerate(themes):
        for _ in range(6):
            ids.append(tid)
            vec.append([t[0] + rng.standard_normal() * 0.05, t[1] + rng.standard_normal() * 0.05])
    got = _check_cluster(ctx, orc, ids, np.array(vec, np.float32), 2, 3, 0, mu=2, tau=5, epsilon=1, theta=1)
    assert list(got.assignments) == ids


def test_cluster_flat_deterministic(ctx, orc):
    # src/tac/tac.zig:1184-1216: same inputs, identical output
    c = synth.make_corpus(6_000, 16, n_anchors=300, seed=5)
    a = _check_cluster(ctx, orc, c.token_ids, c.vectors, 16, 900, 7, mu=8, tau=16, epsilon=2, theta=4)
    b = tac.cluster_flat(c.token_ids, c.vectors, 16, tac.ClusteringParams(900, 7, 8, 16, 2, 4), ctx=ctx)
    assert np.array_equal(a.assignments, b.assignments) and _same_bytes(a.centroids, b.centroids)


@pytest.mark.parametrize("n,dim,kappa,theta,threads", [(20_000, 64, 4096, 10, 1), (20_000, 64, 4096, 10, 8),
                                                       (30_000, 128, 6000, 10, 1), (25_000, 24, 5000, 10, 3)])
def test_cluster_flat_synthetic(ctx, orc, n, dim, kappa, theta, threads):
    c = synth.make_corpus(n, dim, seed=n + dim)
    got = _check_cluster(ctx, orc, c.token_ids, c.vectors, dim, kappa, 42, theta=theta, n_threads=threads)
    assert got.kappa_per_token.sum() == kappa


def test_cluster_flat_config0_shape(ctx, orc):
    # 117,645 x 64 synthetic corpus; kappa 12,288 (10,240 leaves this
    # generator's 11,050 tail centroids no room: BudgetTooSmall, as in the
    # reference), theta 10
    c = synth.make_corpus(117_645, 64, seed=42)
    got = _check_cluster(ctx, orc, c.token_ids, c.vectors, 64, 12_288, 42, theta=10)
    assert got.kappa_per_token.sum() == 12_288
    with pytest.raises(MvrError) as e:
        tac.cluster_flat(c.token_ids, c.vectors, 64, tac.ClusteringParams(10_240, 42, theta=10), ctx=ctx)
    assert e.value.name == "BudgetTooSmall"


def test_cluster_flat_fixed_iterations(ctx, orc):
    c = synth.make_corpus(15_000, 32, n_anchors=800, seed=3)
    _check_cluster(ctx, orc, c.token_ids, c.vectors, 32, 2500, 1, mu=16, tau=32, epsilon=2, theta=4,
                   max_iters=5, tol=float("-inf"))


def test_cluster_flat_errors(ctx, orc):
    ids = np.array([0, 1, 1, 2], np.uint32)
    v = synth.unit_rows(4, 4, seed=0)
    cases = [
        (np.array([], np.uint32), np.array([], np.float32), 4, 4, "EmptyTokenDump"),
        (ids, v, 0, 4, "InvalidThresholds"),
        (ids, v[:3], 4, 4, "InvalidThresholds"),
        (ids, v, 4, 0, "BudgetTooSmall"),
        (ids, v, 4, 2, "BudgetTooSmall"),
    ]
    for i, x, dim, kappa, name in cases:
        with pytest.raises(MvrError) as e:
            tac.cluster_flat(i, x, dim, tac.ClusteringParams(kappa, 0, mu=3, tau=5, epsilon=1, theta=1), ctx=ctx)
        assert e.value.name == name
        with pytest.raises(Exception):
            orc.tac_cluster_flat(i, x, dim, kappa, 0, mu=3, tau=5, eps=1, theta=1)
    # a NaN coordinate makes its token's spread NaN: the budget phases and
    # the k-means reject it with the same status as the oracle
    bad = synth.make_corpus(3_000, 8, n_anchors=50, seed=1)
    for tok, row in [(0, 3), (7, 0)]:
        vec = bad.vectors.copy()
        vec[np.flatnonzero(bad.token_ids == tok)[row], 1] = np.nan
        with pytest.raises(Exception) as w:
            orc.tac_cluster_flat(bad.token_ids, vec, 8, 600, 0, mu=8, tau=16, eps=2, theta=2)
        with pytest.raises(MvrError) as e:
            tac.cluster_flat(bad.token_ids, vec, 8, tac.ClusteringParams(600, 0, mu=8, tau=16, epsilon=2, theta=2),
                             ctx=ctx)
        assert e.value.code == w.value.code
    # the context stays usable
    _check_cluster(ctx, orc, bad.token_ids, bad.vectors, 8, 600, 0, mu=8, tau=16, epsilon=2, theta=2)


# ----------------------------------------------- tensor-core filtered Lloyd
def _km_filter_datasets():
    rng = np.random.default_rng(8)
    yield "unit", synth.unit_rows(9_000, 64, seed=41), 300
    c = synth.make_corpus(30_000, 64, n_anchors=40, seed=3)
    yield "anchors", c.vectors, 700
    base = synth.unit_rows(150, 64, seed=42)
    yield "dup", base[rng.integers(0, 150, size=6_000)], 100  # zero distances, equal centroids
    yield "scaled_up", (synth.unit_rows(5_000, 64, seed=43) * 1e3).astype(np.float32), 128
    yield "scaled_down", (synth.unit_rows(5_000, 64, seed=44) * 1e-3).astype(np.float32), 128
    mixed = synth.unit_rows(6_000, 64, seed=45)
    mixed[::5] *= 1e4
    mixed[2::7] *= 1e-4
    yield "mixed", mixed.astype(np.float32), 200
    big = synth.unit_rows(4_000, 64, seed=46)
    big[::9] *= 1e15  # |x|^2 above 2^60: these rows take the full scan
    yield "huge", big.astype(np.float32), 64
    grid = (np.round(synth.unit_rows(5_000, 64, seed=47) * 4) / 4).astype(np.float32)  # many equal distances
    yield "grid", grid, 96


@pytest.mark.parametrize("name,x,k", list(_km_filter_datasets()), ids=lambda v: v if isinstance(v, str) else "")
def test_km_tensor_filter_matches_exact(ctx, orc, name, x, k):
    """64-dim k-means with k >= 64 runs its Lloyd assignment through the
    tensor-core filter; the exact scans and the oracle give the same bytes."""
    got = _check_kmeans(ctx, orc, x, 64, k, seed=5, max_iters=8, tol=1e-4)
    ctx.check(ctx.lib.mvr_ctx_set_tensor_filter(ctx.handle, 0))
    try:
        ex = kmeans.fit(x, 64, kmeans.KMeansParams(k=k, seed=5, max_iters=8, tol=1e-4), ctx=ctx)
    finally:
        ctx.check(ctx.lib.mvr_ctx_set_tensor_filter(ctx.handle, 1))
    assert np.array_equal(got.assignments, ex.assignments)
    assert _same_bytes(got.centroids, ex.centroids)


def test_cluster_flat_tensor_filter_matches_exact(ctx, orc):
    c = synth.make_corpus(117_645, 64, seed=42)
    p = tac.ClusteringParams(12_288, 42, theta=10)
    a = tac.cluster_flat(c.token_ids, c.vectors, 64, p, ctx=ctx)
    ctx.check(ctx.lib.mvr_ctx_set_tensor_filter(ctx.handle, 0))
    try:
        b = tac.cluster_flat(c.token_ids, c.vectors, 64, p, ctx=ctx)
    finally:
        ctx.check(ctx.lib.mvr_ctx_set_tensor_filter(ctx.handle, 1))
    assert np.array_equal(a.assignments, b.assignments) and _same_bytes(a.centroids, b.centroids)
    assert np.float32(a.wcss_total).tobytes() == np.float32(b.wcss_total).tobytes()


@pytest.mark.parametrize("kind", ["unit", "dup", "grid", "wide"])
def test_kmeans_long_problem_wcss(ctx, orc, kind):
    """Problems of 32,768 rows and more take the segmented exact WCSS sum;
    the reported WCSS and the convergence decisions match the reference's
    serial f32 sum."""
    rng = np.random.default_rng(len(kind))
    n, dim = 40_000, 8
    if kind == "unit":
        x = synth.unit_rows(n, dim, seed=2)
    elif kind == "dup":  # zero distances: the sum stays 0 for a while
        x = synth.unit_rows(60, dim, seed=3)[rng.integers(0, 60, size=n)]
    elif kind == "grid":  # coarse values: many exact ties in the sum's rounding
        x = (np.round(synth.unit_rows(n, dim, seed=4) * 4) / 4).astype(np.float32)
    else:  # magnitudes over many binades
        x = (synth.unit_rows(n, dim, seed=5) * 10.0 ** rng.integers(-6, 6, size=(n, 1))).astype(np.float32)
    for k, tol, iters in ((12, 1e-4, 25), (40, 0.0, 6)):
        _check_kmeans(ctx, orc, x, dim, k, seed=k, max_iters=iters, tol=tol)
    _check_kmeans(ctx, orc, synth.unit_rows(36_000, 64, seed=6), 64, 80, seed=1, max_iters=10, tol=1e-4)


def test_spread_wait_expiry_reports_timeout(ctx, orc):
    """The bounded mbarrier wait of the spread kernel's bulk-copy ring, made
    to run out (the test-only limit of 0 polls): the call fails with
    MVR_E_TIMEOUT after the kernel has waited for its copies still in
    flight, and the context stays usable: the next call is bit-exact."""
    from ir_multivector_retrieval_b200 import _lib

    c = synth.make_corpus(20_000, 64, seed=20_064)
    p = tac.ClusteringParams(4096, 42, theta=10)
    ctx.check(ctx.lib.mvr_ctx_set_wait_limit(ctx.handle, 0))
    try:
        with pytest.raises(MvrError) as e:
            tac.cluster_flat(c.token_ids, c.vectors, 64, p, ctx=ctx)
        assert e.value.code == 102  # MVR_E_TIMEOUT
    finally:
        ctx.check(ctx.lib.mvr_ctx_set_wait_limit(ctx.handle, _lib.WAIT_LIMIT_DEFAULT))
    _check_cluster(ctx, orc, c.token_ids, c.vectors, 64, 4096, 42, theta=10)
