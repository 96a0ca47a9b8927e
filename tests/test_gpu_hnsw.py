"""GPU parity of hnsw.build (src/index/hnsw.zig:314-946): the CUDA build's
graph (levels, entry point, top level, every layer's CSR offsets and
neighbour lists) is byte-identical to the oracle's on the reference's test
inputs and on clustered centroid sets, for the serial and the parallel
path; plus vec.normalizeRowsInPlace and the error statuses.

Bar: bit-exact (integer graph)."""
import numpy as np
import pytest

from ir_multivector_retrieval_b200 import hnsw
from ir_multivector_retrieval_b200._lib import MvrError
from tests.hnsw_fixtures import brute_top, clustered, rng_rows

pytestmark = pytest.mark.gpu


def _same(g, o):
    assert (g.n, g.entry_point, g.max_level) == (o.n, o.entry_point, o.max_level)
    assert np.array_equal(g.node_levels, o.node_levels)
    for L in range(o.max_level + 1):
        assert np.array_equal(g.layer_offsets[L], o.layer_offsets[L]), f"layer {L} offsets"
        assert np.array_equal(g.layer_neighbours[L], o.layer_neighbours[L]), f"layer {L} neighbours"


CASES = [
    # name, data, dim, seed, ef, m, n_threads
    ("smoke4", lambda orc: np.array([1, 0, 0, 1, -1, 0, 0, -1], np.float32), 2, 7, 16, 4, 1),
    ("search5", lambda orc: np.array([1.0, 0.0, 0.9, 0.4359, 0.0, 1.0, -1.0, 0.0, 0.0, -1.0], np.float32), 2, 1,
     32, 4, 1),
    ("seed128x16", lambda orc: rng_rows(orc, 2026, 128, 16)[0], 16, 999, 64, 8, 1),
    ("par600x16", lambda orc: rng_rows(orc, 20260501, 600, 16)[0], 16, 17, 64, 8, 2),
    ("recall1024_serial", lambda orc: rng_rows(orc, 20260501, 1024, 64)[0], 64, 42, 1500, 32, 1),
    ("recall1024_par", lambda orc: rng_rows(orc, 20260502, 1024, 64)[0], 64, 42, 1500, 32, 10),
    ("clustered4096", lambda orc: clustered(4096, 64, 11, orc=orc), 64, 0xDEADBEEF + 5, 1500, 32, 2),
    ("dups2000", lambda orc: clustered(2000, 64, 12, dup=4, orc=orc), 64, 3, 300, 16, 2),
    ("tight3000", lambda orc: clustered(3000, 64, 13, spread=0.02, orc=orc), 64, 4, 400, 32, 2),
    ("dim128_1500", lambda orc: clustered(1500, 128, 14, orc=orc), 128, 5, 500, 24, 2),
    ("odd_dim_700x12", lambda orc: clustered(700, 12, 15, orc=orc), 12, 6, 100, 8, 2),
    ("odd_dim_300x7", lambda orc: clustered(300, 7, 16, orc=orc), 7, 7, 50, 5, 1),
]


@pytest.mark.parametrize("name,make,dim,seed,ef,m,nt", CASES, ids=[c[0] for c in CASES])
def test_build_matches_oracle(ctx, orc, name, make, dim, seed, ef, m, nt):
    x = make(orc)
    o = orc.hnsw_build(x, dim, seed, ef_construction=ef, m=m, n_threads=nt)
    g = hnsw.build(x, dim, seed, ef_construction=ef, m=m, n_threads=nt, ctx=ctx)
    _same(g, o)
    assert g.kernel_launches > 0


def test_build_with_zero_rows_and_single_node(ctx, orc):
    x = clustered(400, 16, 17, orc=orc).reshape(400, 16)
    x[::7] = 0.0  # zero rows stay zero after normalisation: similarity 0 to everything
    x = x.reshape(-1)
    _same(hnsw.build(x, 16, 8, ef_construction=40, m=6, ctx=ctx),
          orc.hnsw_build(x, 16, 8, ef_construction=40, m=6, n_threads=2))
    one = np.ones(16, np.float32) / 4
    g = hnsw.build(one, 16, 1, ctx=ctx)
    assert g.n == 1 and g.entry_point == 0 and all(b.size == 0 for b in g.layer_neighbours)


def test_build_from_device_tensor(ctx, orc):
    import torch
    x = clustered(1000, 64, 18, orc=orc)
    g = hnsw.build(torch.from_numpy(x).cuda(), 64, 9, ef_construction=200, m=16, ctx=ctx)
    _same(g, orc.hnsw_build(x, 64, 9, ef_construction=200, m=16, n_threads=2))


def test_gpu_graph_recall(ctx, orc):
    """The reference's recall test (hnsw.zig:1283) on the GPU-built graph."""
    base, q = rng_rows(orc, 20260502, 1024, 64, 16)
    g = hnsw.build(base, 64, 42, n_threads=10, ctx=ctx)
    tot = 0
    for i in range(16):
        qq = q[i * 64:(i + 1) * 64]
        tot += len(set(brute_top(orc, base, qq, 64, 10).tolist()) & set(orc.hnsw_search(g, base, qq, 10, 60).tolist()))
    assert tot / 160 >= 0.9


@pytest.mark.parametrize("dim", [2, 7, 16, 64, 128])
def test_normalize_rows_matches_oracle(ctx, orc, dim):
    rng = np.random.default_rng(dim)
    x = (rng.standard_normal((333, dim)) * rng.uniform(0.01, 100, (333, 1))).astype(np.float32)
    x[5] = 0.0
    got = hnsw.normalize_rows(x, dim, ctx=ctx)
    assert got.tobytes() == orc.normalize_rows(x, dim).tobytes()


def test_errors(ctx):
    with pytest.raises(MvrError) as e:
        hnsw.build(np.zeros(10, np.float32), 3, 1, ctx=ctx)
    assert e.value.name == "DimMismatch"
    with pytest.raises(MvrError) as e:
        hnsw.build(np.zeros(0, np.float32), 4, 1, ctx=ctx)
    assert e.value.name == "EmptyCorpus"
    with pytest.raises(MvrError) as e:
        hnsw.build(np.ones(64, np.float32), 4, 1, m=33, ctx=ctx)
    assert e.value.name == "InvalidArgument"
    with pytest.raises(MvrError) as e:  # the beam lives in one CTA's shared memory
        hnsw.build(np.ones(64, np.float32), 4, 1, ef_construction=2049, ctx=ctx)
    assert e.value.name == "InvalidArgument"
    with pytest.raises(MvrError) as e:
        hnsw.normalize_rows(np.ones(10, np.float32), 3, ctx=ctx)
    assert e.value.name == "LengthMismatch"


def test_thread_count_contract(ctx, orc):
    """build_determinism_test.zig / hnsw.zig:1401: the graph is the same for
    every n_threads >= 2 and differs on the serial path (n_threads 1)."""
    base, _ = rng_rows(orc, 20260501, 600, 16)
    g2 = hnsw.build(base, 16, 17, ef_construction=64, m=8, n_threads=2, ctx=ctx)
    g10 = hnsw.build(base, 16, 17, ef_construction=64, m=8, n_threads=10, ctx=ctx)
    g1 = hnsw.build(base, 16, 17, ef_construction=64, m=8, n_threads=1, ctx=ctx)
    _same(g2, g10)
    assert any(not np.array_equal(a, b) for a, b in zip(g1.layer_neighbours, g2.layer_neighbours))
