"""Inputs of the reference's HNSW tests (src/index/hnsw.zig:1240-1515),
regenerated with the restated RNG: x = nextFloat() * 2 - 1 per coordinate,
then vec.normalizeInPlace per row."""
import numpy as np


def rng_rows(orc, seed: int, n: int, dim: int, n_queries: int = 0, per_row: bool = True):
    """``per_row`` normalises each row as it is drawn (the recall tests);
    otherwise the whole buffer is drawn first (the determinism tests) — the
    draws are the same either way, only the order of normalisation differs,
    which does not change any value."""
    r = orc.Rng(seed)
    raw = np.array([r.f32() for _ in range((n + n_queries) * dim)], dtype=np.float32)
    x = raw * np.float32(2.0) - np.float32(1.0)
    base = orc.normalize_rows(x[: n * dim], dim)
    q = orc.normalize_rows(x[n * dim:], dim) if n_queries else None
    return base, q


def clustered(n: int, dim: int, seed: int, spread: float = 0.35, dup: int = 1, orc=None):
    """Centroid-like points: n/2 directions, each point one of them plus
    noise, normalised; `dup` > 1 repeats every row (exact similarity ties)."""
    rng = np.random.default_rng(seed)
    base_n = max(1, n // dup)
    anchors = rng.standard_normal((max(1, base_n // 2), dim)).astype(np.float32)
    x = anchors[rng.integers(0, anchors.shape[0], base_n)] + np.float32(spread) * rng.standard_normal(
        (base_n, dim)).astype(np.float32)
    x = np.repeat(x, dup, axis=0)[:n]
    if x.shape[0] < n:
        x = np.concatenate([x, x[: n - x.shape[0]]])
    return orc.normalize_rows(x.reshape(-1), dim)


def brute_top(orc, base, q, dim: int, k: int):
    X = base.reshape(-1, dim)
    d = np.array([orc.dot(q, X[j]) for j in range(X.shape[0])], dtype=np.float32)
    return np.argsort(-d, kind="stable")[:k]
