"""GPU parity of the query side: PQ.buildDistanceTable and refine.refine
(MaxSim from centroids, PQ codes and residual norms) against the oracle on
an index built by the GPU build chain; top-10 documents must be identical.

Bar: bit-exact scores."""
import numpy as np
import pytest

from ir_multivector_retrieval_b200 import refine, storage, synth, tac
from ir_multivector_retrieval_b200._lib import MvrError

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dim,pq_m", [(64, 16), (64, 32), (64, 64), (128, 32), (12, 3)])
def test_distance_table_matches_oracle(ctx, orc, dim, pq_m):
    rng = np.random.default_rng(dim + pq_m)
    cb = rng.standard_normal(pq_m * 256 * (dim // pq_m)).astype(np.float32)
    q = synth.unit_rows(32, dim, seed=pq_m)
    got = refine.distance_table(cb, dim, pq_m, q, ctx=ctx)
    assert got.tobytes() == orc.pq_distance_table(cb, dim, pq_m, q, 32).tobytes()


@pytest.fixture(scope="module")
def small_index(ctx):
    c = synth.make_corpus(20_000, 64, seed=9)
    build = storage.build_codes(c.token_ids, c.vectors, 64, tac.ClusteringParams(kappa_total=4096, seed=3, theta=10),
                                pq_m=16, ctx=ctx)
    return c, refine.index_view(build, c.doc_offsets, 64, ctx=ctx)


@pytest.mark.parametrize("n_q", [32, 7, 70])
def test_refine_scores_and_top10_match_oracle(ctx, orc, small_index, n_q):
    c, ix = small_index
    rng = np.random.default_rng(n_q)
    # seeded synthetic queries: corpus tokens with fresh noise, normalised
    pick = rng.integers(0, c.n, size=n_q)
    q = c.vectors[pick] + np.float32(0.2) * rng.standard_normal((n_q, 64)).astype(np.float32)
    q = (q / np.linalg.norm(q, axis=1, keepdims=True)).astype(np.float32)
    table = refine.distance_table(ix.codebooks, 64, 16, q, ctx=ctx)
    assert table.tobytes() == orc.pq_distance_table(ix.codebooks, 64, 16, q, n_q).tobytes()
    docs = np.arange(ix.n_docs, dtype=np.uint32)
    got = refine.refine_batch(ix, table, q, docs, ctx=ctx)
    want = np.array([orc.refine(ix.centroids, 64, 16, ix.doc_section, ix.n_docs, ix.doc_token_offsets,
                                ix.residual_norms, table, q, n_q, int(d)) for d in docs], dtype=np.float32)
    assert got.tobytes() == want.tobytes()
    g10, _ = refine.top_k(got, docs)
    w10, _ = refine.top_k(want, docs)
    assert np.array_equal(g10, w10)


def test_refine_errors(ctx, orc, small_index):
    _, ix = small_index
    q = synth.unit_rows(4, 64, seed=1)
    table = refine.distance_table(ix.codebooks, 64, 16, q, ctx=ctx)
    with pytest.raises(MvrError) as e:
        refine.refine_batch(ix, table, q, [0, ix.n_docs], ctx=ctx)
    assert e.value.name == "DocOutOfRange"
    with pytest.raises(MvrError) as e:
        refine.refine_batch(ix, table[:-1], q, [0], ctx=ctx)
    assert e.value.name == "TableSizeMismatch"
    with pytest.raises(MvrError) as e:
        refine.distance_table(ix.codebooks, 64, 16, q[:, :63], ctx=ctx)
    assert e.value.name == "NQMismatch"
    # a doc whose token range disagrees with its stored count is corrupt
    bad = refine.IndexView(**{**ix.__dict__, "doc_token_offsets": ix.doc_token_offsets.copy()})
    bad.doc_token_offsets[1] += 1
    with pytest.raises(MvrError) as e:
        refine.refine_batch(bad, table, q, [0], ctx=ctx)
    assert e.value.name == "DocLayoutCorrupt"
    with pytest.raises(Exception):
        orc.refine(bad.centroids, 64, 16, bad.doc_section, bad.n_docs, bad.doc_token_offsets, bad.residual_norms,
                   table, q, 4, 0)
