"""GPU parity of the index builder's last two stages against the oracle:
inverted_list.build (src/index/inverted_list.zig:64-150) and
storage.serialise (src/index/storage.zig:560-665), then the image read back
by the oracle's restatement of storage.parse (:765-860) and searched by
refine on seeded queries.

Bar: bit-exact (integer lists, byte-identical images, identical scores and
top-10)."""
import zlib

import numpy as np
import pytest

from ir_multivector_retrieval_b200 import refine, storage, synth, tac
from ir_multivector_retrieval_b200._lib import MvrError

pytestmark = pytest.mark.gpu


def _ilists_equal(ctx, orc, a, off, kappa):
    got = storage.inverted_lists_build(a, off, kappa, ctx=ctx)
    want = orc.inverted_lists_build(a, off, kappa)
    assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1])
    return got


def test_inverted_lists_reference_cases(ctx, orc):
    # inverted_list.zig:162-245
    o, p = _ilists_equal(ctx, orc, np.array([1, 3, 1, 1, 0, 3], np.uint32), np.array([0, 2, 4, 6], np.uint64), 4)
    assert list(p[o[1]:o[2]]) == [0, 1] and list(p[o[3]:o[4]]) == [0, 2]
    _ilists_equal(ctx, orc, np.zeros(5, np.uint32), np.arange(6, dtype=np.uint64), 1)
    _ilists_equal(ctx, orc, np.full(4, 2, np.uint32), np.array([0, 4], np.uint64), 5)
    _ilists_equal(ctx, orc, np.array([0, 1], np.uint32), np.array([0, 1, 1, 2], np.uint64), 3)
    _ilists_equal(ctx, orc, np.zeros(0, np.uint32), np.array([0, 0, 0], np.uint64), 7)  # no tokens at all
    for a, off, k, name in (([0, 5], [0, 2], 3, "AssignmentOutOfRange"), ([0, 0, 0], [0, 2, 1, 3], 1, "DocOffsetsBad"),
                            ([0], [0, 1], 0, "KappaZero"), ([0, 0], [0, 1], 1, "DocOffsetsBad"),
                            ([0], [1, 1], 1, "DocOffsetsBad")):
        with pytest.raises(MvrError) as e:
            storage.inverted_lists_build(np.array(a, np.uint32), np.array(off, np.uint64), k, ctx=ctx)
        assert e.value.name == name


@pytest.mark.parametrize("n,kappa,docs", [(100_000, 4096, 1500), (300_001, 70_000, 9000), (5000, 300_000, 100)])
def test_inverted_lists_random(ctx, orc, n, kappa, docs):
    rng = np.random.default_rng(n)
    a = rng.integers(0, kappa, size=n).astype(np.uint32)
    a[::3] = a[0]  # a hot centroid, many duplicates inside docs
    cuts = np.sort(rng.integers(0, n + 1, size=docs - 1))  # includes empty docs
    off = np.concatenate([[0], cuts, [n]]).astype(np.uint64)
    _ilists_equal(ctx, orc, a, off, kappa)


@pytest.fixture(scope="module")
def built(ctx):
    c = synth.make_corpus(20_000, 64, seed=9)
    p = tac.ClusteringParams(kappa_total=4096, seed=3, theta=10)
    b = storage.build_index(c.token_ids, c.vectors, c.doc_offsets, 64, p, pq_m=16, hnsw_ef_construction=64,
                            hnsw_m=8, ctx=ctx)
    return c, b


def test_serialised_image_matches_oracle(ctx, orc, built):
    c, b = built
    g = b.hnsw
    bc = b.codes
    parts = orc.tac_parts(dim=64, kappa=4096, sub_dim=4, pq_m=16, centroids=b.centroids_normalised,
                          assignments=bc.clustering.assignments, pq_codes=bc.codes, doc_offsets=c.doc_offsets,
                          codebooks=bc.pq.codebooks, hnsw_entry_point=g.entry_point, hnsw_node_levels=g.node_levels,
                          hnsw_layer_offsets=g.layer_offsets, hnsw_layer_neighbours=g.layer_neighbours,
                          ilist_offsets=b.ilist_offsets, ilist_payload=b.ilist_payload, residual_norms=bc.norms)
    want = orc.tac_serialise(parts)
    assert b.image == want
    # the footer is the CRC-32 of everything before it (std.hash.Crc32)
    footer = int.from_bytes(b.image[104:112], "little")
    assert int.from_bytes(b.image[footer:footer + 4], "little") == zlib.crc32(b.image[:footer])
    # the inverted lists in the image are the oracle's from the same assignments
    ilo, ilp = orc.inverted_lists_build(bc.clustering.assignments, c.doc_offsets, 4096)
    assert np.array_equal(ilo, b.ilist_offsets) and np.array_equal(ilp, b.ilist_payload)


def test_parse_then_refine_top10(ctx, orc, built):
    """serialise -> parse (oracle) -> refine on seeded queries: the same
    scores and top-10 as refine on the in-memory parts, on the GPU and in the
    oracle."""
    c, b = built
    v = orc.tac_parse(b.image, 16)
    assert v["header"]["n_tokens"] == c.n and v["header"]["kappa"] == 4096
    assert v["centroids"].tobytes() == b.centroids_normalised.tobytes()
    assert v["codebooks"].tobytes() == b.codes.pq.codebooks.tobytes()
    assert np.array_equal(v["doc_token_offsets"], c.doc_offsets)
    parsed = refine.IndexView(v["centroids"], 64, 16, v["codebooks"], v["doc_section"], int(v["header"]["n_docs"]),
                              v["doc_token_offsets"], v["residual_norms"])
    mem = refine.IndexView(b.centroids_normalised, 64, 16, np.ascontiguousarray(b.codes.pq.codebooks),
                           storage.write_doc_layouts(c.doc_offsets, b.codes.clustering.assignments, b.codes.codes, 16,
                                                     ctx=ctx),
                           c.doc_offsets.size - 1, np.ascontiguousarray(c.doc_offsets, np.uint64), b.codes.norms)
    rng = np.random.default_rng(5)
    pick = rng.integers(0, c.n, size=32)
    q = c.vectors[pick] + np.float32(0.2) * rng.standard_normal((32, 64)).astype(np.float32)
    q = (q / np.linalg.norm(q, axis=1, keepdims=True)).astype(np.float32)
    table = refine.distance_table(parsed.codebooks, 64, 16, q, ctx=ctx)
    docs = np.arange(parsed.n_docs, dtype=np.uint32)
    from_file = refine.refine_batch(parsed, table, q, docs, ctx=ctx)
    in_memory = refine.refine_batch(mem, table, q, docs, ctx=ctx)
    want = np.array([orc.refine(parsed.centroids, 64, 16, parsed.doc_section, parsed.n_docs, parsed.doc_token_offsets,
                                parsed.residual_norms, table, q, 32, int(d)) for d in docs], dtype=np.float32)
    assert from_file.tobytes() == in_memory.tobytes() == want.tobytes()
    t_file, _ = refine.top_k(from_file, docs)
    t_orc, _ = refine.top_k(want, docs)
    assert np.array_equal(t_file, t_orc)


def test_serialise_errors(ctx, built):
    c, b = built
    with pytest.raises(MvrError) as e:
        storage.serialise(dim=64, kappa=4096, sub_dim=4, pq_m=16, centroids=b.centroids_normalised,
                          assignments=b.codes.clustering.assignments[:-1], pq_codes=b.codes.codes,
                          doc_offsets=c.doc_offsets, codebooks=b.codes.pq.codebooks, hnsw=b.hnsw,
                          ilist_offsets=b.ilist_offsets, ilist_payload=b.ilist_payload,
                          residual_norms=b.codes.norms, ctx=ctx)
    assert e.value.name == "InvalidArgument"
