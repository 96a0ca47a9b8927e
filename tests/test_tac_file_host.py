"""Host-only parts of the .tac writer (no GPU): the image size
(storage.computeSize, src/index/storage.zig:490-551) against the oracle's
restatement, and the CRC-32 combination used to checksum the image on
several host threads against zlib."""
import ctypes as C
import zlib

import numpy as np

from ir_multivector_retrieval_b200 import _lib
from ir_multivector_retrieval_b200 import storage


def test_crc32_combine_matches_zlib():
    lib = _lib.load()
    rng = np.random.default_rng(3)
    for la, lb in ((0, 5), (1, 1), (13, 1000), (4096, 8191), (100_000, 1), (7, 0)):
        a = rng.integers(0, 256, la, dtype=np.uint8).tobytes()
        b = rng.integers(0, 256, lb, dtype=np.uint8).tobytes()
        got = lib.mvr_crc32_combine(zlib.crc32(a), zlib.crc32(b), lb)
        assert got == zlib.crc32(a + b)


def test_file_size_matches_oracle(orc):
    rng = np.random.default_rng(4)
    kappa, dim, pq_m, n_docs = 50, 16, 4, 9
    lens = rng.integers(0, 7, n_docs)
    off = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint64)
    n = int(off[-1])
    asg = rng.integers(0, kappa, n).astype(np.uint32)
    ilo, ilp = orc.inverted_lists_build(asg, off, kappa)

    class G:  # a two-layer graph of 50 nodes
        entry_point = 3
        node_levels = np.zeros(kappa, np.uint8)
        layer_offsets = [np.arange(kappa + 1, dtype=np.uint32) * 2, np.zeros(kappa + 1, np.uint32)]
        layer_neighbours = [rng.integers(0, kappa, 2 * kappa).astype(np.uint32), np.zeros(0, np.uint32)]

    kw = dict(dim=dim, kappa=kappa, sub_dim=dim // pq_m, pq_m=pq_m,
              centroids=rng.standard_normal(kappa * dim).astype(np.float32), assignments=asg,
              pq_codes=rng.integers(0, 256, n * pq_m).astype(np.uint8), doc_offsets=off,
              codebooks=rng.standard_normal(pq_m * 256 * (dim // pq_m)).astype(np.float32),
              ilist_offsets=ilo, ilist_payload=ilp, residual_norms=rng.random(n).astype(np.float32))
    p, _keep = storage._parts(hnsw=G, **kw)
    got = C.c_uint64(0)
    assert _lib.load().mvr_tac_file_size(C.byref(p), C.byref(got)) == 0
    op, _okeep = orc.tac_parts(hnsw_entry_point=G.entry_point, hnsw_node_levels=G.node_levels,
                               hnsw_layer_offsets=G.layer_offsets, hnsw_layer_neighbours=G.layer_neighbours, **kw)
    want = orc.load().orc_tac_file_size(C.byref(op))
    assert got.value == want == len(orc.tac_serialise((op, _okeep)))
