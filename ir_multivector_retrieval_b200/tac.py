"""TAC clustering: the reference's ``tac.zig`` interface over the B200
library.

``cluster_flat`` replaces ``tac.clusterFlat`` (src/tac/tac.zig:563-838);
``allocate_budgets`` the budget phases 1-4 (tac.zig:390-402).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import ClusteringParams as _CParams
from ._lib import MvrError, ptr

TAC_MU, TAC_TAU, TAC_EPSILON, TAC_THETA = 128, 256, 4, 39  # src/constants.zig:10-13


@dataclass
class ClusteringParams:
    """Reference ``ClusteringParams`` (tac.zig:35-57)."""

    kappa_total: int
    seed: int
    mu: int = TAC_MU
    tau: int = TAC_TAU
    epsilon: int = TAC_EPSILON
    theta: int = TAC_THETA
    max_iters: int = 25
    tol: float = 1e-4
    n_threads: int = 1

    def to_c(self) -> _CParams:
        return _CParams(self.kappa_total, self.mu, self.tau, self.epsilon, self.theta, self.max_iters,
                        self.tol, self.seed & (2**64 - 1), self.n_threads)


@dataclass
class ClusteringResult:
    """Reference ``ClusteringResult`` (tac.zig:410-426)."""

    centroids: np.ndarray  # kappa_total * dim float32, token-id order
    assignments: np.ndarray  # n uint32 global centroid ids
    kappa_per_token: np.ndarray  # n_distinct uint32
    wcss_total: float


def allocate_budgets(freqs, spreads, kappa_total: int, p: ClusteringParams) -> np.ndarray:
    f = np.ascontiguousarray(freqs, dtype=np.uint32)
    s = np.ascontiguousarray(spreads, dtype=np.float32)
    k = np.zeros(f.size, dtype=np.uint32)
    frac = np.zeros(f.size, dtype=np.float32)
    cp = p.to_c()
    st = _lib.load().mvr_tac_allocate_budgets(ptr(f), ptr(s), ptr(k), ptr(frac), f.size, kappa_total,
                                              C.byref(cp))
    if st:
        raise MvrError(st, "allocate_budgets")
    return k


def last_stats(ctx=None) -> dict:
    """Timing report of the context's most recent ``cluster_flat`` call."""
    ctx = ctx or _lib.default_context()
    st = _lib.TacStats()
    ctx.check(ctx.lib.mvr_tac_last_stats(ctx.handle, C.byref(st)))
    return st.as_dict()


def partition_tokens(freqs, kappa, n_ranks: int) -> np.ndarray:
    """Owner rank of every token's k-means in the sharded clusterFlat
    (longest-processing-time split of the work n_j * (k_j + 1))."""
    f = np.ascontiguousarray(freqs, dtype=np.uint32)
    k = np.ascontiguousarray(kappa, dtype=np.uint32)
    if f.size != k.size:
        raise ValueError("freqs and kappa differ in length")
    out = np.zeros(max(f.size, 1), dtype=np.uint32)
    st = _lib.load().mvr_tac_partition_tokens(ptr(f), ptr(k), f.size, n_ranks, ptr(out))
    if st:
        raise _lib.MvrError(st, "partition_tokens")
    return out[: f.size]


def cluster_flat(token_ids, vectors, dim: int, p: ClusteringParams, ctx=None, *,
                 sharded: bool = False) -> ClusteringResult:
    """tac.clusterFlat (src/tac/tac.zig:563-838) on the GPU. With
    ``sharded=True`` the call is collective over the context's communicator
    (every rank passes the same inputs and gets the same full result)."""
    ids = np.ascontiguousarray(token_ids, dtype=np.uint32).reshape(-1)
    v = np.ascontiguousarray(vectors, dtype=np.float32).reshape(-1)
    ctx = ctx or _lib.default_context()
    nd = int(ids.max()) + 1 if ids.size else 1
    cent = np.zeros(max(p.kappa_total, 1) * max(dim, 1), dtype=np.float32)
    asg = np.zeros(max(ids.size, 1), dtype=np.uint32)
    kap = np.zeros(nd, dtype=np.uint32)
    ndo = C.c_uint64(0)
    w = C.c_float(0)
    cp = p.to_c()
    fn = ctx.lib.mvr_tac_cluster_flat_sharded if sharded else ctx.lib.mvr_tac_cluster_flat
    ctx.check(fn(ctx.handle, ptr(ids), ids.size, ptr(v), v.size, dim, C.byref(cp), ptr(cent), ptr(asg), ptr(kap), nd,
                 C.byref(ndo), C.byref(w)))
    return ClusteringResult(cent[: p.kappa_total * dim], asg[: ids.size], kap[: ndo.value], float(w.value))
