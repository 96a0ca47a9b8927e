"""Build-stage glue of the reference's ``storage.build`` around the hot path.

``residuals_and_norms`` replaces ``storage.residualsAndNormsChunk``
(src/index/storage.zig:255-278): per row, ``r = v - c[a]`` against the
un-normalised TAC centroid, ``norm = sqrt(sum fl(r_d^2))`` in coordinate
order, and ``r * fl(1/norm)`` when ``norm > 0``.

``build_codes`` runs build steps 1, 3 and 4 (storage.zig:341, :380,
:389-400): ``tac.clusterFlat`` -> residuals -> ``pq.train`` (seed
``params.seed +% 0xa1b2c3d4``) -> ``PQ.encode`` of every row.

``inverted_lists_build`` replaces ``inverted_list.build``; ``serialise``
replaces ``storage.serialise`` (the .tac image: header, centroids, HNSW, PQ
codebooks, inverted lists, per-doc layouts, doc token offsets, residual
norms, footer CRC-32); ``build_index`` is ``storage.build`` end to end.
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


def inverted_lists_build(assignments, doc_offsets, kappa: int, ctx=None):
    """inverted_list.build (src/index/inverted_list.zig:64-150) on the GPU:
    (offsets u64[kappa + 1], payload u32[offsets[kappa]]) in the reference's
    CSR layout (per centroid the ascending ids of the docs that have a token
    in it, once each)."""
    a = np.ascontiguousarray(assignments, dtype=np.uint32).reshape(-1)
    off = np.ascontiguousarray(doc_offsets, dtype=np.uint64)
    ctx = ctx or _lib.default_context()
    offsets = np.zeros(int(kappa) + 1, dtype=np.uint64)
    payload = np.zeros(max(1, a.size), dtype=np.uint32)
    total = C.c_uint64(0)
    ctx.check(ctx.lib.mvr_inverted_lists_build(ctx.handle, ptr(a) if a.size else None, a.size,
                                               ptr(off) if off.size else None, off.size, int(kappa), ptr(offsets),
                                               ptr(payload), payload.size, C.byref(total)), "inverted_lists_build")
    return offsets, payload[: total.value].copy()


def _parts(*, dim, kappa, sub_dim, pq_m, centroids, assignments, pq_codes, doc_offsets, codebooks, hnsw,
           ilist_offsets, ilist_payload, residual_norms):
    keep = {
        "centroids": np.ascontiguousarray(centroids, dtype=np.float32).reshape(-1),
        "assignments": np.ascontiguousarray(assignments, dtype=np.uint32).reshape(-1),
        "pq_codes": np.ascontiguousarray(pq_codes, dtype=np.uint8).reshape(-1),
        "doc_offsets": np.ascontiguousarray(doc_offsets, dtype=np.uint64),
        "codebooks": np.ascontiguousarray(codebooks, dtype=np.float32).reshape(-1),
        "levels": np.ascontiguousarray(hnsw.node_levels, dtype=np.uint8),
        "offs": [np.ascontiguousarray(o, dtype=np.uint32) for o in hnsw.layer_offsets],
        "nbrs": [np.ascontiguousarray(o, dtype=np.uint32) for o in hnsw.layer_neighbours],
        "ilo": np.ascontiguousarray(ilist_offsets, dtype=np.uint64),
        "ilp": np.ascontiguousarray(ilist_payload, dtype=np.uint32),
        "norms": np.ascontiguousarray(residual_norms, dtype=np.float32).reshape(-1),
    }
    nl = len(keep["offs"])
    keep["offp"] = (C.c_void_p * nl)(*[o.ctypes.data for o in keep["offs"]])
    keep["nbrp"] = (C.c_void_p * nl)(*[(o.ctypes.data if o.size else keep["offs"][0].ctypes.data)
                                       for o in keep["nbrs"]])
    p = _lib.TacParts()
    p.dim, p.kappa, p.sub_dim, p.pq_m = int(dim), int(kappa), int(sub_dim), int(pq_m)
    p.n_docs = keep["doc_offsets"].size - 1
    p.n_tokens = keep["assignments"].size
    p.centroids = keep["centroids"].ctypes.data
    p.assignments = keep["assignments"].ctypes.data
    p.pq_codes = keep["pq_codes"].ctypes.data
    p.doc_offsets = keep["doc_offsets"].ctypes.data
    p.codebooks = keep["codebooks"].ctypes.data
    p.hnsw_n = keep["levels"].size
    p.hnsw_entry_point = int(hnsw.entry_point)
    p.hnsw_max_level = nl - 1
    p.hnsw_node_levels = keep["levels"].ctypes.data
    p.hnsw_layer_offsets = C.cast(keep["offp"], C.c_void_p)
    p.hnsw_layer_neighbours = C.cast(keep["nbrp"], C.c_void_p)
    p.ilist_offsets = keep["ilo"].ctypes.data
    p.ilist_payload = keep["ilp"].ctypes.data if keep["ilp"].size else keep["ilo"].ctypes.data
    p.residual_norms = keep["norms"].ctypes.data
    return p, keep


def serialise(*, dim: int, kappa: int, sub_dim: int, pq_m: int, centroids, assignments, pq_codes, doc_offsets,
              codebooks, hnsw, ilist_offsets, ilist_payload, residual_norms, ctx=None) -> bytes:
    """storage.serialise (src/index/storage.zig:560-665): the whole .tac
    image of a built index (the reference's BuildOutput fields; ``hnsw`` any
    object with node_levels / entry_point / layer_offsets /
    layer_neighbours, e.g. hnsw.Hnsw)."""
    ctx = ctx or _lib.default_context()
    p, _keep = _parts(dim=dim, kappa=kappa, sub_dim=sub_dim, pq_m=pq_m, centroids=centroids,
                      assignments=assignments, pq_codes=pq_codes, doc_offsets=doc_offsets, codebooks=codebooks,
                      hnsw=hnsw, ilist_offsets=ilist_offsets, ilist_payload=ilist_payload,
                      residual_norms=residual_norms)
    n = C.c_uint64(0)
    ctx.check(ctx.lib.mvr_tac_file_size(C.byref(p), C.byref(n)), "tac_file_size")
    buf = np.empty(n.value, dtype=np.uint8)
    w = C.c_uint64(0)
    ctx.check(ctx.lib.mvr_tac_serialise(ctx.handle, C.byref(p), ptr(buf), buf.size, C.byref(w)), "tac_serialise")
    return buf[: w.value].tobytes()


@dataclass
class BuiltIndex:
    """What build_index produces: the image and the parts it was made of."""

    image: bytes
    codes: BuildCodes
    centroids_normalised: np.ndarray
    hnsw: object
    ilist_offsets: np.ndarray
    ilist_payload: np.ndarray


def build_index(token_ids, vectors, doc_offsets, dim: int, params: tac.ClusteringParams, *,
                pq_m: int = pq.PQ_M_REFERENCE, pq_iters: int = 25, pq_tol: float = 1e-4,
                hnsw_ef_construction: int = 1500, hnsw_m: int = 32, hnsw_threads: int = 2,
                ctx=None) -> BuiltIndex:
    """storage.build (src/index/storage.zig:324-470) end to end on the GPU:
    clusterFlat -> residuals + norms -> pq.train (seed +% 0xa1b2c3d4) ->
    PQ.encode -> normalised centroids -> hnsw.build (seed +% 0xdeadbeef) ->
    inverted lists -> serialise."""
    from . import hnsw as hnsw_mod

    if dim == 0 or dim % pq_m:
        raise _lib.MvrError(_lib.CODES["InvalidIndex"], "dim must be a positive multiple of pq_m")
    ctx = ctx or _lib.default_context()
    bc = build_codes(token_ids, vectors, dim, params, pq_m=pq_m, pq_iters=pq_iters, pq_tol=pq_tol, ctx=ctx)
    cent = hnsw_mod.normalize_rows(bc.clustering.centroids, dim, ctx=ctx)
    g = hnsw_mod.build(cent, dim, (params.seed + hnsw_mod.STORAGE_SEED_OFFSET) & (2**64 - 1),
                       ef_construction=hnsw_ef_construction, m=hnsw_m, n_threads=hnsw_threads, ctx=ctx)
    ilo, ilp = inverted_lists_build(bc.clustering.assignments, doc_offsets, params.kappa_total, ctx=ctx)
    img = serialise(dim=dim, kappa=params.kappa_total, sub_dim=dim // pq_m, pq_m=pq_m, centroids=cent,
                    assignments=bc.clustering.assignments, pq_codes=bc.codes, doc_offsets=doc_offsets,
                    codebooks=bc.pq.codebooks, hnsw=g, ilist_offsets=ilo, ilist_payload=ilp,
                    residual_norms=bc.norms, ctx=ctx)
    return BuiltIndex(img, bc, cent, g, ilo, ilp)


__all__ = ["residuals_and_norms", "build_codes", "BuildCodes", "PQ_SEED_OFFSET", "doc_layouts_bytes",
           "write_doc_layouts", "crc32", "inverted_lists_build", "serialise", "build_index", "BuiltIndex"]
_ = C  # ctypes kept for symmetry with the other modules
