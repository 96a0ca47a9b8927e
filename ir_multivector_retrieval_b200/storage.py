"""Build-stage glue of the reference's ``storage.build`` around the hot path.

``residuals_and_norms`` replaces ``storage.residualsAndNormsChunk``
(src/index/storage.zig:255-278): per row, ``r = v - c[a]`` against the
un-normalised TAC centroid, ``norm = sqrt(sum fl(r_d^2))`` in coordinate
order, and ``r * fl(1/norm)`` when ``norm > 0``.

``build_codes`` runs build steps 1, 3 and 4 (storage.zig:341, :380,
:389-400): ``tac.clusterFlat`` -> residuals -> ``pq.train`` (seed
``params.seed +% 0xa1b2c3d4``) -> ``PQ.encode`` of every row.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib, pq, tac
from ._lib import ptr

PQ_SEED_OFFSET = 0xA1B2C3D4  # storage.zig:380


def residuals_and_norms(vectors, centroids, assignments, dim: int, ctx=None):
    """(residuals n x dim f32, norms n f32) computed on the GPU."""
    v = np.ascontiguousarray(vectors, dtype=np.float32).reshape(-1)
    c = np.ascontiguousarray(centroids, dtype=np.float32).reshape(-1)
    a = np.ascontiguousarray(assignments, dtype=np.uint32).reshape(-1)
    n = v.size // dim
    kappa = c.size // dim
    ctx = ctx or _lib.default_context()
    res = np.empty(n * dim, dtype=np.float32)
    norms = np.empty(n, dtype=np.float32)
    ctx.check(ctx.lib.mvr_residuals_norms(ctx.handle, ptr(v), ptr(c), kappa, ptr(a), n, dim, ptr(res),
                                          ptr(norms)))
    return res.reshape(n, dim), norms


@dataclass
class BuildCodes:
    clustering: tac.ClusteringResult
    residuals: np.ndarray  # n x dim, unit (or zero) rows
    norms: np.ndarray  # n
    pq: pq.PQ
    codes: np.ndarray  # n x pq_m u8


def build_codes(token_ids, vectors, dim: int, params: tac.ClusteringParams, *, pq_m: int = pq.PQ_M_REFERENCE,
                pq_iters: int = 25, pq_tol: float = 1e-4, ctx=None) -> BuildCodes:
    """storage.build steps 1/3/4 on the GPU; every stage is bit-exact with
    the reference's arithmetic."""
    ctx = ctx or _lib.default_context()
    cl = tac.cluster_flat(token_ids, vectors, dim, params, ctx=ctx)
    res, norms = residuals_and_norms(vectors, cl.centroids, cl.assignments, dim, ctx=ctx)
    book = pq.train(res, dim, (params.seed + PQ_SEED_OFFSET) & (2**64 - 1), pq_m=pq_m, max_iters=pq_iters,
                    tol=pq_tol, ctx=ctx)
    codes = book.encode_batch(res)
    return BuildCodes(cl, res, norms, book, codes)


def doc_layouts_bytes(doc_offsets, pq_m: int) -> int:
    """Size of the .tac per-doc section (storage.zig:506-508)."""
    off = np.ascontiguousarray(doc_offsets, dtype=np.uint64)
    n = C.c_uint64(0)
    st = _lib.load().mvr_doc_layouts_bytes(ptr(off), off.size - 1, pq_m, C.byref(n))
    if st:
        raise _lib.MvrError(st, "doc_layouts_bytes")
    return int(n.value)


def write_doc_layouts(doc_offsets, assignments, codes, pq_m: int, ctx=None) -> bytes:
    """storage.writeDocLayouts (storage.zig:705-749) on the GPU: the doc
    index plus one [n_d | assignments | codes | pad] block per doc."""
    off = np.ascontiguousarray(doc_offsets, dtype=np.uint64)
    a = np.ascontiguousarray(assignments, dtype=np.uint32).reshape(-1)
    c = np.ascontiguousarray(codes, dtype=np.uint8).reshape(-1)
    ctx = ctx or _lib.default_context()
    n = doc_layouts_bytes(off, pq_m)
    out = np.empty(n, dtype=np.uint8)
    ctx.check(ctx.lib.mvr_write_doc_layouts(ctx.handle, ptr(off), off.size - 1, ptr(a), ptr(c), a.size, pq_m,
                                            ptr(out), n))
    return out.tobytes()


def crc32(data: bytes, crc: int = 0) -> int:
    """The .tac footer checksum (std.hash.Crc32, storage.zig:655-660)."""
    buf = np.frombuffer(data, dtype=np.uint8)
    return int(_lib.load().mvr_crc32(crc, ptr(buf) if buf.size else None, buf.size))


__all__ = ["residuals_and_norms", "build_codes", "BuildCodes", "PQ_SEED_OFFSET", "doc_layouts_bytes",
           "write_doc_layouts", "crc32"]
_ = C  # ctypes kept for symmetry with the other modules
