"""Query side of the index: the reference's ``PQ.buildDistanceTable``
(src/index/pq.zig:92-123) and ``refine.refine`` (src/retrieval/refine.zig:
83-155) on the GPU, for a batch of candidate documents per query.

``IndexView`` holds the sections a refine reads (TAC centroids, the per-doc
section of ``storage.write_doc_layouts``, doc token offsets, residual
norms); ``index_view`` assembles one from ``storage.build_codes``.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib, storage
from ._lib import ptr


@dataclass
class IndexView:
    centroids: np.ndarray  # kappa x dim f32
    dim: int
    pq_m: int
    codebooks: np.ndarray  # pq_m * 256 * (dim / pq_m) f32
    doc_section: bytes  # storage.write_doc_layouts
    n_docs: int
    doc_token_offsets: np.ndarray  # n_docs + 1 u64
    residual_norms: np.ndarray  # n_tokens f32

    @property
    def kappa(self) -> int:
        return self.centroids.size // self.dim


def index_view(build: storage.BuildCodes, doc_offsets, dim: int, ctx=None) -> IndexView:
    off = np.ascontiguousarray(doc_offsets, dtype=np.uint64)
    m = build.pq.pq_m
    sec = storage.write_doc_layouts(off, build.clustering.assignments, build.codes, m, ctx=ctx)
    return IndexView(np.ascontiguousarray(build.clustering.centroids, dtype=np.float32).reshape(-1), dim, m,
                     np.ascontiguousarray(build.pq.codebooks, dtype=np.float32), sec, off.size - 1, off,
                     np.ascontiguousarray(build.norms, dtype=np.float32))


def distance_table(codebooks, dim: int, pq_m: int, query, ctx=None) -> np.ndarray:
    """[pq_m][256][n_q] dot products of the query's sub-vectors with every
    codeword (pq.zig:92-123)."""
    q = np.ascontiguousarray(query, dtype=np.float32).reshape(-1)
    cb = np.ascontiguousarray(codebooks, dtype=np.float32).reshape(-1)
    n_q = q.size // dim if dim else 0
    ctx = ctx or _lib.default_context()
    out = np.empty(pq_m * 256 * max(n_q, 1), dtype=np.float32)
    ctx.check(ctx.lib.mvr_pq_distance_table(ctx.handle, ptr(cb), dim, pq_m, ptr(q), q.size, n_q, ptr(out),
                                            pq_m * 256 * n_q))
    return out


def refine_batch(index: IndexView, table, query, doc_ids, ctx=None) -> np.ndarray:
    """MaxSim scores S(q, d) of the candidate docs (refine.zig:83-155)."""
    q = np.ascontiguousarray(query, dtype=np.float32).reshape(-1)
    t = np.ascontiguousarray(table, dtype=np.float32).reshape(-1)
    ids = np.ascontiguousarray(doc_ids, dtype=np.uint32).reshape(-1)
    sec = np.frombuffer(index.doc_section, dtype=np.uint8)
    n_q = q.size // index.dim
    ctx = ctx or _lib.default_context()
    scores = np.empty(max(ids.size, 1), dtype=np.float32)
    ctx.check(ctx.lib.mvr_refine_batch(ctx.handle, ptr(index.centroids), index.kappa, index.dim, index.pq_m,
                                       ptr(np.ascontiguousarray(sec)), sec.size, index.n_docs,
                                       ptr(index.doc_token_offsets), ptr(index.residual_norms),
                                       index.residual_norms.size, ptr(t), t.size, ptr(q), q.size, n_q, ptr(ids),
                                       ids.size, ptr(scores)))
    return scores[: ids.size]


def top_k(scores, doc_ids, k: int = 10):
    """Highest scores first, ties to the smaller doc id."""
    s = np.asarray(scores)
    d = np.asarray(doc_ids)
    order = np.lexsort((d, -s))
    return d[order[:k]], s[order[:k]]


__all__ = ["IndexView", "index_view", "distance_table", "refine_batch", "top_k"]
_ = C
