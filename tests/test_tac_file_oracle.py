"""The CPU restatement of inverted_list.build and the .tac image
(oracle/tac_file_oracle.c) against the reference's own tests of those
functions (src/index/inverted_list.zig:162-245, src/index/storage.zig:
988-1231), read as text and replayed here; plus the CRC-32 against zlib's
(the same IEEE polynomial as Zig's std.hash.Crc32)."""
import zlib

import numpy as np
import pytest

from ir_multivector_retrieval_b200 import synth


def _ilists(orc, a, off, kappa):
    return orc.inverted_lists_build(np.array(a, np.uint32), np.array(off, np.uint64), kappa)


def _list(offsets, payload, j):
    return list(payload[int(offsets[j]):int(offsets[j + 1])])


def test_ilists_hand_checked_tiny_case(orc):
    # inverted_list.zig:162-178
    o, p = _ilists(orc, [1, 3, 1, 1, 0, 3], [0, 2, 4, 6], 4)
    assert _list(o, p, 0) == [2] and _list(o, p, 1) == [0, 1]
    assert _list(o, p, 2) == [] and _list(o, p, 3) == [0, 2]


def test_ilists_ascending_dedup_and_empty_doc(orc):
    # inverted_list.zig:180-209
    o, p = _ilists(orc, [0, 0, 0, 0, 0], [0, 1, 2, 3, 4, 5], 1)
    assert _list(o, p, 0) == [0, 1, 2, 3, 4]
    o, p = _ilists(orc, [2, 2, 2, 2], [0, 4], 5)
    assert _list(o, p, 2) == [0] and int(o[5]) == 1
    o, p = _ilists(orc, [0, 1], [0, 1, 1, 2], 3)
    assert _list(o, p, 0) == [0] and _list(o, p, 1) == [2] and _list(o, p, 2) == []


def test_ilists_errors_and_invariants(orc):
    # inverted_list.zig:211-245
    with pytest.raises(orc.OracleError) as e:
        _ilists(orc, [0, 5], [0, 2], 3)
    assert e.value.code == 26  # AssignmentOutOfRange
    with pytest.raises(orc.OracleError) as e:
        _ilists(orc, [0, 0, 0], [0, 2, 1, 3], 1)
    assert e.value.code == 27  # DocOffsetsBad
    with pytest.raises(orc.OracleError) as e:
        _ilists(orc, [0], [0, 1], 0)
    assert e.value.code == 28  # KappaZero
    o, p = _ilists(orc, [0, 1, 2, 0, 1, 2, 0, 1, 2], [0, 3, 6, 9], 3)
    assert np.all(np.diff(o.astype(np.int64)) >= 0) and int(o[3]) == p.size


def test_crc32_is_zlib(orc):
    rng = np.random.default_rng(1)
    for n in (0, 1, 7, 8, 9, 1000, 65537):
        b = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        assert orc.crc32(b) == zlib.crc32(b)


def _fixture(orc):
    """The reference's storage.zig:1000-1114 fixture shape: dim 32, M=32
    (sub_dim 1), kappa 8, 4 docs of 3 tokens, round-robin assignments, PQ
    trained on normalised residuals, norms 1 + 0.1 i, HNSW (m 4, efc 32),
    inverted lists. Values come from this repository's seeded generators
    (the reference's use its own RNG)."""
    dim, kappa, pq_m = 32, 8, 32
    cents = synth.unit_rows(kappa, dim, seed=2026)
    asg = np.arange(12, dtype=np.uint32) % kappa
    doc_off = np.arange(0, 13, 3, dtype=np.uint64)
    res = synth.unit_rows(300, dim, seed=7)  # enough rows for 256 centroids per subspace
    cb = orc.pq_train(res, dim, 7, pq_m, max_iters=5)
    codes = orc.pq_encode(cb, dim, pq_m, res[:12])
    norms = (1.0 + 0.1 * np.arange(12)).astype(np.float32)
    g = orc.hnsw_build(cents, dim, 11, ef_construction=32, m=4, n_threads=1)
    ilo, ilp = orc.inverted_lists_build(asg, doc_off, kappa)
    parts = orc.tac_parts(dim=dim, kappa=kappa, sub_dim=1, pq_m=pq_m, centroids=cents, assignments=asg,
                          pq_codes=codes, doc_offsets=doc_off, codebooks=cb, hnsw_entry_point=g.entry_point,
                          hnsw_node_levels=g.node_levels, hnsw_layer_offsets=g.layer_offsets,
                          hnsw_layer_neighbours=g.layer_neighbours, ilist_offsets=ilo, ilist_payload=ilp,
                          residual_norms=norms)
    return parts, dict(cents=cents, asg=asg, doc_off=doc_off, cb=cb, codes=codes, norms=norms, g=g, ilo=ilo,
                       ilp=ilp)


def test_serialise_parse_round_trip(orc):
    # storage.zig:988-997 (header 112 bytes in a 128-byte region, magic,
    # version 2) and :1116-1194 (every section recovered)
    parts, f = _fixture(orc)
    img = orc.tac_serialise(parts)
    assert img[:8] == b"TAC_IDX1" and int.from_bytes(img[8:12], "little") == 2
    assert img[112:128] == bytes(16)
    assert int.from_bytes(img[48:56], "little") == 128
    assert len(img) % 8 == 0
    v = orc.tac_parse(img, 32)
    h = v["header"]
    assert (h["dim"], h["kappa"], h["n_docs"], h["n_tokens"], h["pq_m"], h["sub_dim"]) == (32, 8, 4, 12, 32, 1)
    assert v["centroids"].tobytes() == f["cents"].tobytes()
    assert v["codebooks"].tobytes() == np.ascontiguousarray(f["cb"], np.float32).tobytes()
    g = f["g"]
    assert v["hnsw"]["entry_point"] == g.entry_point and v["hnsw"]["max_level"] == g.max_level
    assert np.array_equal(v["hnsw"]["node_levels"], g.node_levels)
    for a, b in zip(v["hnsw"]["layer_offsets"] + v["hnsw"]["layer_neighbours"], g.layer_offsets + g.layer_neighbours):
        assert np.array_equal(a, b)
    assert np.array_equal(v["ilist_offsets"], f["ilo"]) and np.array_equal(v["ilist_payload"], f["ilp"])
    assert v["residual_norms"].tobytes() == f["norms"].tobytes()
    assert np.array_equal(v["doc_token_offsets"], f["doc_off"])
    assert v["doc_section"] == orc.write_doc_layouts(f["doc_off"], f["asg"], f["codes"], 32)
    # a reader built with another PQ_M refuses the image (storage.zig:776)
    with pytest.raises(orc.OracleError) as e:
        orc.tac_parse(img, 16)
    assert e.value.code == 23


def test_parse_rejects_tampering(orc):
    # storage.zig:1196-1231
    parts, _ = _fixture(orc)
    img = bytearray(orc.tac_serialise(parts))
    bad = bytearray(img)
    bad[0] = ord("X")
    with pytest.raises(orc.OracleError) as e:
        orc.tac_parse(bytes(bad), 32)
    assert e.value.code == 23  # InvalidIndex
    bad = bytearray(img)
    bad[128] ^= 0x80
    with pytest.raises(orc.OracleError) as e:
        orc.tac_parse(bytes(bad), 32)
    assert e.value.code == 25  # IndexCorrupt
    with pytest.raises(orc.OracleError) as e:
        orc.tac_parse(bytes(16), 32)
    assert e.value.code == 23
    bad = bytearray(img)
    bad[8] = 3  # version
    with pytest.raises(orc.OracleError) as e:
        orc.tac_parse(bytes(bad), 32)
    assert e.value.code == 24  # UnsupportedVersion
