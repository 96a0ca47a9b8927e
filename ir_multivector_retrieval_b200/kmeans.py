"""``kmeans.fit`` (src/tac/kmeans.zig:67-232) over the B200 library.

k-means++ seeding, Lloyd iterations with the reference's in-order centroid
sums, empty-cluster reseeding and relative-WCSS stopping; results are
bit-identical with the reference arithmetic.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import CODES, MvrError, ptr


@dataclass
class KMeansParams:
    """Reference ``KMeansParams`` (kmeans.zig:28-41)."""

    k: int
    seed: int
    max_iters: int = 25
    tol: float = 1e-4
    n_threads: int = 1


@dataclass
class KMeansResult:
    """Reference ``KMeansResult`` (kmeans.zig:43-54)."""

    centroids: np.ndarray  # k * dim float32
    assignments: np.ndarray  # n uint32
    wcss: float
    iters_run: int


def validate(vectors_len: int, dim: int, k: int) -> None:
    """kmeans.fit's validation order (kmeans.zig:73-76)."""
    if k == 0:
        raise MvrError(CODES["KmeansBudgetTooSmall"], "k == 0")
    if dim == 0:
        raise MvrError(CODES["DimMismatch"], "dim == 0")
    if vectors_len == 0:
        raise MvrError(CODES["EmptyVectorSet"], "no vectors")
    if vectors_len % dim != 0:
        raise MvrError(CODES["DimMismatch"], "len % dim != 0")


def fit(vectors, dim: int, p: KMeansParams, ctx=None) -> KMeansResult:
    v = np.ascontiguousarray(vectors, dtype=np.float32).reshape(-1)
    validate(v.size, dim, p.k)
    ctx = ctx or _lib.default_context()
    n = v.size // dim
    cent = np.empty(p.k * dim, dtype=np.float32)
    asg = np.empty(n, dtype=np.uint32)
    w = C.c_float(0)
    it = C.c_uint32(0)
    ctx.check(ctx.lib.mvr_kmeans_fit(ctx.handle, ptr(v), v.size, dim, p.k, p.max_iters,
                                     C.c_float(p.tol), p.seed & (2**64 - 1), p.n_threads,
                                     ptr(cent), ptr(asg), C.byref(w), C.byref(it)))
    return KMeansResult(centroids=cent, assignments=asg, wcss=float(w.value), iters_run=int(it.value))
