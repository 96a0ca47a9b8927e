"""Product quantisation: the reference's ``pq.zig`` interface over the B200
library.

``train`` replaces ``pq.train`` (src/index/pq.zig:158-164), ``PQ.encode``
replaces ``PQ.encode`` (pq.zig:59-76) and ``PQ.encode_batch`` the encode
stage of the build (src/index/storage.zig:287-295, :389-400). Codebook
layout is the reference's ``codebook[m][c][k] = codebooks[((m*256)+c)*sub_dim+k]``
(pq.zig:14-15). The subspace count ``pq_m`` is a run-time argument here; the
reference fixes it at compile time (``constants.PQ_M = 32``).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _lib
from ._lib import CODES, MvrError, PqTrainStats, ptr

PQ_CENTROIDS = 256
PQ_M_REFERENCE = 32  # src/constants.zig:16


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).reshape(-1)


def validate_train(residuals_len: int, dim: int, pq_m: int) -> None:
    """pq.train's validation order (src/index/pq.zig:165-168)."""
    if dim == 0:
        raise MvrError(CODES["DimMismatch"], "dim == 0")
    if pq_m == 0 or dim % pq_m != 0:
        raise MvrError(CODES["DimNotDivisibleByM"], f"dim {dim} % pq_m {pq_m} != 0")
    if residuals_len == 0:
        raise MvrError(CODES["EmptyCorpus"], "empty residual set")
    if residuals_len % dim != 0:
        raise MvrError(CODES["DimMismatch"], "len % dim != 0")


@dataclass
class PQ:
    """Trained codebooks (reference ``pq.PQ``, src/index/pq.zig:41-56)."""

    dim: int
    sub_dim: int
    codebooks: np.ndarray  # float32, pq_m * 256 * sub_dim
    pq_m: int = PQ_M_REFERENCE
    ctx: object = field(default=None, repr=False, compare=False)

    def codebook_entry(self, m: int, c: int) -> np.ndarray:
        base = (m * PQ_CENTROIDS + c) * self.sub_dim
        return self.codebooks[base : base + self.sub_dim]

    def encode(self, residual) -> np.ndarray:
        """Codes of one residual (``PQ.encode``). DimMismatch if the length
        is not ``dim``."""
        r = _f32(residual)
        if r.size != self.dim:
            raise MvrError(CODES["DimMismatch"], f"residual has {r.size} floats, dim {self.dim}")
        return self.encode_batch(r)[0]

    def encode_batch(self, residuals) -> np.ndarray:
        """Codes of n row-major residuals, shape (n, pq_m), uint8."""
        r = _f32(residuals)
        if r.size % self.dim != 0:
            raise MvrError(CODES["DimMismatch"], "len % dim != 0")
        n = r.size // self.dim
        out = np.empty((n, self.pq_m), dtype=np.uint8)
        if n == 0:
            return out
        ctx = self.ctx or _lib.default_context()
        cb = _f32(self.codebooks)
        ctx.check(ctx.lib.mvr_pq_encode(ctx.handle, ptr(cb), self.dim, self.pq_m, ptr(r), n, ptr(out)))
        return out

    def decode(self, codes) -> np.ndarray:
        """Concatenated codewords (``PQ.decode``, pq.zig:79-88)."""
        c = np.ascontiguousarray(codes, dtype=np.uint8).reshape(-1, self.pq_m)
        out = np.empty((c.shape[0], self.dim), dtype=np.float32)
        st = _lib.load().mvr_pq_decode(ptr(_f32(self.codebooks)), self.dim, self.pq_m, ptr(c),
                                       c.shape[0], ptr(out))
        if st:
            raise MvrError(st, "decode")
        return out[0] if np.ndim(codes) == 1 else out


def train(residuals, dim: int, seed: int, n_threads: int = 1, *, pq_m: int = PQ_M_REFERENCE,
          max_iters: int = 25, tol: float = 1e-4, ctx=None, stats: dict | None = None) -> PQ:
    """``pq.train(residuals, dim, seed, n_threads, gpa)`` on the GPU.

    Each subspace m runs ``kmeans.fit(k=256, max_iters, tol, seed +% m)``;
    the reference hard-codes ``max_iters=25, tol=1e-4``. ``tol=-inf`` runs
    exactly ``max_iters`` Lloyd iterations. ``stats`` (a dict) receives the
    device timings.
    """
    r = _f32(residuals)
    validate_train(r.size, dim, pq_m)
    ctx = ctx or _lib.default_context()
    sub = dim // pq_m
    cb = np.empty(pq_m * PQ_CENTROIDS * sub, dtype=np.float32)
    st = PqTrainStats()
    ctx.check(ctx.lib.mvr_pq_train(ctx.handle, ptr(r), r.size, dim, seed & (2**64 - 1), n_threads,
                                   pq_m, max_iters, C.c_float(tol), ptr(cb), C.byref(st)))
    if stats is not None:
        stats.update({k: getattr(st, k) for k, _ in PqTrainStats._fields_})
    return PQ(dim=dim, sub_dim=sub, codebooks=cb, pq_m=pq_m, ctx=ctx)
