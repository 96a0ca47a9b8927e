"""The HNSW oracle (hnsw_oracle.c) against the reference's own HNSW tests
(src/index/hnsw.zig:1240-1515): recall@10 >= 0.9 on 1024 random unit
vectors for the serial and the parallel path, the same graph for the same
seed, the same graph for every thread count >= 2, and the small-graph smoke
and search checks. No GPU."""
import numpy as np

from tests.hnsw_fixtures import brute_top, clustered, rng_rows


def _same(a, b):
    assert a.entry_point == b.entry_point and a.max_level == b.max_level
    assert np.array_equal(a.node_levels, b.node_levels)
    for L in range(a.max_level + 1):
        assert np.array_equal(a.layer_offsets[L], b.layer_offsets[L])
        assert np.array_equal(a.layer_neighbours[L], b.layer_neighbours[L])


def _recall(orc, g, base, q, dim, n_q=16, k=10, ef=60):
    tot = 0
    for i in range(n_q):
        qq = q[i * dim:(i + 1) * dim]
        tot += len(set(brute_top(orc, base, qq, dim, k).tolist()) & set(orc.hnsw_search(g, base, qq, k, ef).tolist()))
    return tot / (n_q * k)


def test_recall_serial_1024x64(orc):  # hnsw.zig:1283 (defaults: n_threads 1)
    base, q = rng_rows(orc, 20260501, 1024, 64, 16)
    g = orc.hnsw_build(base, 64, 42, n_threads=1)
    assert _recall(orc, g, base, q, 64) >= 0.9


def test_recall_parallel_1024x64(orc):  # hnsw.zig:1438 (n_threads 10)
    base, q = rng_rows(orc, 20260502, 1024, 64, 16)
    g = orc.hnsw_build(base, 64, 42, n_threads=10)
    assert _recall(orc, g, base, q, 64) >= 0.9


def test_same_seed_same_graph(orc):  # hnsw.zig:1364
    base, _ = rng_rows(orc, 2026, 128, 16)
    a = orc.hnsw_build(base, 16, 999, ef_construction=64, m=8, n_threads=1)
    b = orc.hnsw_build(base, 16, 999, ef_construction=64, m=8, n_threads=1)
    _same(a, b)


def test_parallel_deterministic_across_thread_counts(orc):  # hnsw.zig:1401
    base, _ = rng_rows(orc, 20260501, 600, 16)
    a = orc.hnsw_build(base, 16, 17, ef_construction=64, m=8, n_threads=2, workers=1)
    b = orc.hnsw_build(base, 16, 17, ef_construction=64, m=8, n_threads=10, workers=7)
    _same(a, b)
    s = orc.hnsw_build(base, 16, 17, ef_construction=64, m=8, n_threads=1)
    assert any(not np.array_equal(x, y) for x, y in zip(s.layer_neighbours, a.layer_neighbours))


def test_smoke_four_unit_vectors(orc):  # hnsw.zig:1245
    c = np.array([1, 0, 0, 1, -1, 0, 0, -1], dtype=np.float32)
    g = orc.hnsw_build(c, 2, 7, ef_construction=16, m=4, n_threads=1)
    assert g.n == 4 and g.entry_point < 4


def test_search_small_graph(orc):  # hnsw.zig:1256
    c = np.array([1.0, 0.0, 0.9, 0.4359, 0.0, 1.0, -1.0, 0.0, 0.0, -1.0], dtype=np.float32)
    g = orc.hnsw_build(c, 2, 1, ef_construction=32, m=4, n_threads=1)
    q = np.array([1.0, 0.0], dtype=np.float32)
    out = orc.hnsw_search(g, c, q, 3, 16)
    assert out.size == 3 and out[0] == 0
    sims = [orc.dot(q, c[i * 2:i * 2 + 2]) for i in out]
    assert all(sims[i + 1] <= sims[i] + 1e-6 for i in range(2))


def test_graph_invariants_clustered(orc):
    """Caps (2M on layer 0, M above), no self loops or repeated neighbours,
    every listed neighbour present on the layer, levels within 31."""
    x = clustered(3000, 64, 3, orc=orc)
    g = orc.hnsw_build(x, 64, 5, ef_construction=200, m=16, n_threads=2)
    assert g.node_levels.max() == g.max_level <= 31
    assert g.node_levels[g.entry_point] == g.max_level
    for L in range(g.max_level + 1):
        cap = 32 if L == 0 else 16
        o, nb = g.layer_offsets[L], g.layer_neighbours[L]
        assert o[0] == 0 and o[-1] == nb.size
        deg = np.diff(o.astype(np.int64))
        assert deg.max() <= cap
        assert np.all(deg[g.node_levels < L] == 0)
        assert np.all(g.node_levels[nb] >= L)
        for i in np.nonzero(deg)[0][:500]:
            lst = nb[o[i]:o[i + 1]]
            assert i not in lst and np.unique(lst).size == lst.size


def test_levels_follow_pick_level(orc):
    """levels[i] = floor(-ln(1 - nextFloat) / ln M), levels[0] drawn first
    (hnsw.zig:343, :949-956)."""
    import math
    x = clustered(500, 8, 1, orc=orc)
    g = orc.hnsw_build(x, 8, 123, ef_construction=16, m=4, n_threads=2)
    r = orc.Rng(123)
    ml = np.float32(1.0) / np.float32(math.log(np.float32(4)))
    want = []
    for _ in range(500):
        u = np.float32(1.0) - np.float32(r.f32())
        want.append(min(31, int(np.floor(np.float32(-np.log(u)) * ml))))
    assert g.node_levels.tolist() == want
