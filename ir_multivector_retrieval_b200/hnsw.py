"""HNSW over the TAC centroids on the GPU: the reference's ``hnsw.build``
(src/index/hnsw.zig:314-946) and the centroid normalisation the storage
layer runs before it (``vec.normalizeRowsInPlace``, storage.zig:408-411).

``build`` returns an ``Hnsw`` holding the reference's frozen graph: node
levels, the entry point, the top level and, per layer, CSR offsets (n + 1
entries from 0) and neighbour ids. ``n_threads <= 1`` builds the reference's
serial path, ``n_threads >= 2`` its chunked deferred-commit path (the same
graph for every count >= 2).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _lib
from ._lib import ptr

HNSW_M = 32  # constants.HNSW_M
HNSW_EFC = 1500  # constants.HNSW_EFC
STORAGE_SEED_OFFSET = 0xDEADBEEF  # storage.zig:421: hnsw seed = build seed +% 0xdeadbeef


@dataclass
class Hnsw:
    dim: int
    n: int
    entry_point: int
    max_level: int
    node_levels: np.ndarray  # u8[n]
    layer_offsets: list = field(default_factory=list)  # per layer u32[n + 1]
    layer_neighbours: list = field(default_factory=list)  # per layer u32[offsets[-1]]
    device_ms: float = 0.0
    kernel_launches: int = 0

    def neighbours(self, node: int, layer: int) -> np.ndarray:
        o = self.layer_offsets[layer]
        return self.layer_neighbours[layer][int(o[node]): int(o[node + 1])]


def _take(lib, h) -> Hnsw:
    n, ep, ml = C.c_uint32(), C.c_uint32(), C.c_uint32()
    ms, launches = C.c_float(), C.c_uint64()
    lib.mvr_hnsw_info(h, C.byref(n), C.byref(ep), C.byref(ml), C.byref(ms), C.byref(launches))
    nn = n.value
    levels = np.ctypeslib.as_array(lib.mvr_hnsw_node_levels(h), shape=(nn,)).copy()
    offs, nbrs = [], []
    for L in range(ml.value + 1):
        offs.append(np.ctypeslib.as_array(lib.mvr_hnsw_layer_offsets(h, L), shape=(nn + 1,)).copy())
        cnt = C.c_uint64()
        p = lib.mvr_hnsw_layer_neighbours(h, L, C.byref(cnt))
        nbrs.append(np.ctypeslib.as_array(p, shape=(cnt.value,)).copy() if cnt.value else
                    np.zeros(0, dtype=np.uint32))
    return Hnsw(0, nn, ep.value, ml.value, levels, offs, nbrs, float(ms.value), int(launches.value))


def build(centroids, dim: int, seed: int, ef_construction: int = HNSW_EFC, m: int = HNSW_M, n_threads: int = 2,
          ctx=None) -> Hnsw:
    """hnsw.build on L2-normalised centroids (a host array or a device
    tensor)."""
    ctx = ctx or _lib.default_context()
    lib = ctx.lib
    h = C.c_void_p()
    seed = int(seed) & (2**64 - 1)
    if hasattr(centroids, "is_cuda") and centroids.is_cuda:
        x = centroids.contiguous().view(-1)
        assert str(x.dtype) == "torch.float32"
        ctx.check(lib.mvr_hnsw_build_device(ctx.handle, ptr(x), x.numel(), dim, seed, ef_construction, m,
                                            n_threads, C.byref(h)), "hnsw.build")
    else:
        x = np.ascontiguousarray(centroids, dtype=np.float32).reshape(-1)
        ctx.check(lib.mvr_hnsw_build(ctx.handle, ptr(x), x.size, dim, seed, ef_construction, m, n_threads,
                                     C.byref(h)), "hnsw.build")
    try:
        g = _take(lib, h)
    finally:
        lib.mvr_hnsw_free(h)
    g.dim = dim
    return g


def normalize_rows(rows, dim: int, ctx=None):
    """vec.normalizeRowsInPlace on the GPU: returns a normalised copy of a
    host array, or normalises a device tensor in place."""
    ctx = ctx or _lib.default_context()
    if hasattr(rows, "is_cuda") and rows.is_cuda:
        ctx.check(ctx.lib.mvr_normalize_rows_device(ctx.handle, ptr(rows), rows.numel(), dim), "normalize_rows")
        return rows
    x = np.ascontiguousarray(rows, dtype=np.float32).reshape(-1).copy()
    ctx.check(ctx.lib.mvr_normalize_rows(ctx.handle, ptr(x), x.size, dim), "normalize_rows")
    return x


__all__ = ["Hnsw", "build", "normalize_rows", "HNSW_M", "HNSW_EFC", "STORAGE_SEED_OFFSET"]
