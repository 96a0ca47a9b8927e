"""ctypes binding of the CPU parity oracle (``oracle/libmvr_oracle.so``).

TEST INFRASTRUCTURE ONLY. Imported by tests/, ``__graft_entry__.smoke()``
and the CPU-baseline leg of ``bench.py`` — never by the product package.
The oracle restates the reference's algorithm in plain C (see the header of
``mvr_oracle.c`` for what is pinned and what is not).
"""
from __future__ import annotations

import ctypes as C
import subprocess
import threading
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "libmvr_oracle.so"
_lock = threading.Lock()
_lib = None

_P = C.c_void_p


class OracleError(Exception):
    def __init__(self, code: int, what: str = ""):
        self.code = code
        super().__init__(f"oracle status {code} {what}")


def build(force: bool = False) -> Path:
    srcs = [HERE / "mvr_oracle.c", HERE / "hnsw_oracle.c", HERE / "mvr_oracle.h", HERE.parent / "include" / "mvr.h"]
    if force or not LIB.exists() or any(s.stat().st_mtime > LIB.stat().st_mtime for s in srcs):
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def load() -> C.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            if not LIB.exists():
                build()
            lib = C.CDLL(str(LIB))
            sig = {
                "orc_set_reduce_tree": (None, [C.c_int]),
                "orc_set_lane_count": (None, [C.c_int]),
                "orc_set_workers": (None, [C.c_int]),
                "orc_l2sq": (C.c_float, [_P, _P, C.c_uint32]),
                "orc_argmin": (C.c_int64, [_P, C.c_uint64]),
                "orc_argmax": (C.c_int64, [_P, C.c_uint64]),
                "orc_rng_init": (None, [_P, C.c_uint64]),
                "orc_rng_next": (C.c_uint64, [_P]),
                "orc_rng_index": (C.c_uint64, [_P, C.c_uint64]),
                "orc_rng_f64": (C.c_double, [_P]),
                "orc_rng_f32": (C.c_float, [_P]),
                "orc_weighted_sample": (C.c_int, [_P, _P, C.c_uint64, C.POINTER(C.c_uint64)]),
                "orc_kmeans_fit": (C.c_int, [_P, C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32,
                                             C.c_float, C.c_uint64, C.c_uint32, _P, _P, _P, _P, _P]),
                "orc_pq_train": (C.c_int, [_P, C.c_uint64, C.c_uint32, C.c_uint64, C.c_uint32,
                                           C.c_uint32, C.c_uint32, C.c_float, _P]),
                "orc_pq_encode": (C.c_int, [_P, C.c_uint32, C.c_uint32, _P, C.c_uint64, _P, C.c_uint32]),
                "orc_pq_lloyd_iters": (C.c_int, [_P, C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32,
                                                 C.c_uint32, _P]),
                "orc_residuals_norms": (C.c_int, [_P, _P, _P, C.c_uint64, C.c_uint32, _P, _P]),
                "orc_tac_allocate_tail": (C.c_int, [_P, _P, C.c_uint64, C.c_uint32, C.c_uint32,
                                                    C.c_uint32, C.POINTER(C.c_uint32)]),
                "orc_tac_damped_phase2": (C.c_int, [_P, _P, _P, _P, C.c_uint64, C.c_uint32,
                                                    C.c_uint32, C.c_uint32]),
                "orc_tac_bound_phase3": (C.c_int, [_P, _P, C.c_uint64, C.c_uint32, C.c_uint32,
                                                   C.c_uint32, C.c_uint32]),
                "orc_tac_reconcile_phase4": (C.c_int, [_P, _P, _P, C.c_uint64, C.c_uint32, C.c_uint32,
                                                       C.c_uint32, C.c_uint32, C.c_uint32]),
                "orc_tac_allocate_budgets": (C.c_int, [_P, _P, _P, _P, C.c_uint64, C.c_uint32,
                                                       C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]),
                "orc_tac_spreads": (C.c_int, [_P, C.c_uint64, _P, C.c_uint32, C.c_uint64, _P, _P]),
                "orc_tac_cluster_flat": (C.c_int, [_P, C.c_uint64, _P, C.c_uint64, C.c_uint32,
                                                   C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                                   C.c_uint32, C.c_uint32, C.c_float, C.c_uint64,
                                                   C.c_uint32, _P, _P, _P, C.c_uint64,
                                                   C.POINTER(C.c_uint64), C.POINTER(C.c_float)]),
                "orc_crc32": (C.c_uint32, [_P, C.c_uint64]),
                "orc_inverted_lists_build": (C.c_int, [_P, C.c_uint64, _P, C.c_uint64, C.c_uint32, _P, _P,
                                                       C.c_uint64, C.POINTER(C.c_uint64)]),
                "orc_tac_file_size": (C.c_uint64, [_P]),
                "orc_tac_serialise": (C.c_int, [_P, _P, C.c_uint64, C.POINTER(C.c_uint64)]),
                "orc_tac_parse": (C.c_int, [_P, C.c_uint64, C.c_uint32, _P]),
            }
            for name, (res, args) in sig.items():
                f = getattr(lib, name)
                f.restype = res
                f.argtypes = args
            _lib = lib
        return _lib


def _p(a: np.ndarray) -> C.c_void_p:
    return C.c_void_p(a.ctypes.data)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).reshape(-1)


def _u32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint32).reshape(-1)


def set_reduce_tree(tree: bool) -> None:
    load().orc_set_reduce_tree(1 if tree else 0)


def set_lane_count(n: int) -> None:
    load().orc_set_lane_count(int(n))


def l2sq(a, b) -> float:
    a, b = _f32(a), _f32(b)
    assert a.size == b.size
    return float(np.float32(load().orc_l2sq(_p(a), _p(b), a.size)))


def argmin(v) -> int:
    v = _f32(v)
    return int(load().orc_argmin(_p(v), v.size))


def argmax(v) -> int:
    v = _f32(v)
    return int(load().orc_argmax(_p(v), v.size))


class Rng:
    """Restated Zig ``std.Random.DefaultPrng`` (Xoshiro256++)."""

    def __init__(self, seed: int):
        self.state = (C.c_uint64 * 4)()
        load().orc_rng_init(self.state, seed & (2**64 - 1))

    def next(self) -> int:
        return int(load().orc_rng_next(self.state))

    def index(self, n: int) -> int:
        return int(load().orc_rng_index(self.state, n))

    def f64(self) -> float:
        return float(load().orc_rng_f64(self.state))

    def f32(self) -> float:
        return float(load().orc_rng_f32(self.state))

    def weighted_sample(self, w) -> int:
        w = _f32(w)
        out = C.c_uint64(0)
        st = load().orc_weighted_sample(self.state, _p(w), w.size, C.byref(out))
        if st:
            raise OracleError(st, "weighted_sample")
        return int(out.value)


@dataclass
class KMeansResult:
    centroids: np.ndarray
    assignments: np.ndarray
    wcss: float
    iters_run: int
    trace: np.ndarray | None = None


def kmeans_fit(vectors, dim: int, k: int, seed: int, max_iters: int = 25, tol: float = 1e-4,
               n_threads: int = 1, trace: bool = False) -> KMeansResult:
    v = _f32(vectors)
    n = v.size // dim if dim else 0
    cent = np.zeros(max(k, 1) * max(dim, 1), dtype=np.float32)
    asg = np.zeros(max(n, 1), dtype=np.uint32)
    tr = np.zeros(max(max_iters, 1) * max(n, 1), dtype=np.uint32) if trace else None
    w = C.c_float(0)
    it = C.c_uint32(0)
    st = load().orc_kmeans_fit(_p(v), v.size, dim, k, max_iters, C.c_float(tol), seed & (2**64 - 1),
                               n_threads, _p(cent), _p(asg), C.byref(w), C.byref(it),
                               _p(tr) if tr is not None else None)
    if st:
        raise OracleError(st, "kmeans_fit")
    return KMeansResult(cent[: k * dim], asg[:n], float(w.value), int(it.value),
                        tr.reshape(max_iters, n)[: it.value] if tr is not None else None)


def pq_train(residuals, dim: int, seed: int, pq_m: int, n_threads: int = 1, max_iters: int = 25,
             tol: float = 1e-4) -> np.ndarray:
    r = _f32(residuals)
    s = dim // pq_m if pq_m and dim % pq_m == 0 else 1
    cb = np.zeros(max(pq_m, 1) * 256 * s, dtype=np.float32)
    st = load().orc_pq_train(_p(r), r.size, dim, seed & (2**64 - 1), n_threads, pq_m, max_iters,
                             C.c_float(tol), _p(cb))
    if st:
        raise OracleError(st, "pq_train")
    return cb


def pq_encode(codebooks, dim: int, pq_m: int, residuals, n_threads: int = 1) -> np.ndarray:
    r = _f32(residuals)
    n = r.size // dim
    out = np.zeros((n, pq_m), dtype=np.uint8)
    st = load().orc_pq_encode(_p(_f32(codebooks)), dim, pq_m, _p(r), n, _p(out), n_threads)
    if st:
        raise OracleError(st, "pq_encode")
    return out


def pq_lloyd_iters(residuals, dim: int, pq_m: int, iters: int, n_threads: int, codebooks) -> np.ndarray:
    r = _f32(residuals)
    cb = _f32(codebooks).copy()
    st = load().orc_pq_lloyd_iters(_p(r), r.size // dim, dim, pq_m, iters, n_threads, _p(cb))
    if st:
        raise OracleError(st, "pq_lloyd_iters")
    return cb


def residuals_norms(vectors, centroids, assignments, dim: int):
    v = _f32(vectors)
    n = v.size // dim
    res = np.zeros(n * dim, dtype=np.float32)
    norms = np.zeros(n, dtype=np.float32)
    load().orc_residuals_norms(_p(v), _p(_f32(centroids)), _p(_u32(assignments)), n, dim, _p(res), _p(norms))
    return res, norms


def _check(st, what):
    if st:
        raise OracleError(st, what)


def tac_allocate_tail(freqs, kappa_total, mu, tau):
    f = _u32(freqs)
    k = np.zeros(f.size, dtype=np.uint32)
    b = C.c_uint32(0)
    _check(load().orc_tac_allocate_tail(_p(f), _p(k), f.size, mu, tau, kappa_total, C.byref(b)), "tail")
    return k, int(b.value)


def tac_damped_phase2(freqs, spreads, kappa, budget, mu, tau):
    f, s, k = _u32(freqs), _f32(spreads), _u32(kappa).copy()
    frac = np.zeros(f.size, dtype=np.float32)
    _check(load().orc_tac_damped_phase2(_p(f), _p(s), _p(k), _p(frac), f.size, budget, mu, tau), "phase2")
    return k, frac


def tac_bound_phase3(freqs, kappa, mu, tau, eps, theta):
    f, k = _u32(freqs), _u32(kappa).copy()
    _check(load().orc_tac_bound_phase3(_p(f), _p(k), f.size, mu, tau, eps, theta), "phase3")
    return k


def tac_reconcile_phase4(freqs, kappa, frac, kappa_total, mu, tau, eps, theta):
    f, k, fr = _u32(freqs), _u32(kappa).copy(), _f32(frac)
    _check(load().orc_tac_reconcile_phase4(_p(f), _p(k), _p(fr), f.size, kappa_total, mu, tau, eps, theta),
           "phase4")
    return k


def tac_allocate_budgets(freqs, spreads, kappa_total, mu=128, tau=256, eps=4, theta=39):
    f, s = _u32(freqs), _f32(spreads)
    k = np.zeros(f.size, dtype=np.uint32)
    frac = np.zeros(f.size, dtype=np.float32)
    _check(load().orc_tac_allocate_budgets(_p(f), _p(s), _p(k), _p(frac), f.size, kappa_total, mu, tau,
                                           eps, theta), "allocate_budgets")
    return k


def tac_spreads(token_ids, vectors, dim: int):
    ids = _u32(token_ids)
    v = _f32(vectors)
    nd = int(ids.max()) + 1
    freqs = np.zeros(nd, dtype=np.uint32)
    spreads = np.zeros(nd, dtype=np.float32)
    load().orc_tac_spreads(_p(ids), ids.size, _p(v), dim, nd, _p(freqs), _p(spreads))
    return freqs, spreads


@dataclass
class ClusterResult:
    centroids: np.ndarray
    assignments: np.ndarray
    kappa_per_token: np.ndarray
    wcss_total: float


def tac_cluster_flat(token_ids, vectors, dim: int, kappa_total: int, seed: int, mu=128, tau=256,
                     eps=4, theta=39, max_iters=25, tol=1e-4, n_threads=1, workers: int = 1) -> ClusterResult:
    """clusterFlat restated. `n_threads` is the reference's thread count (it
    only changes how wcss_total is chunked, tac.zig:712-825); `workers` runs
    the per-token k-means on that many host threads (same bytes)."""
    load().orc_set_workers(int(workers))
    ids = _u32(token_ids)
    v = _f32(vectors)
    nd = int(ids.max()) + 1 if ids.size else 1
    cent = np.zeros(max(kappa_total, 1) * max(dim, 1), dtype=np.float32)
    asg = np.zeros(max(ids.size, 1), dtype=np.uint32)
    kap = np.zeros(nd, dtype=np.uint32)
    ndo = C.c_uint64(0)
    w = C.c_float(0)
    _check(load().orc_tac_cluster_flat(_p(ids), ids.size, _p(v), v.size, dim, kappa_total, mu, tau, eps,
                                       theta, max_iters, C.c_float(tol), seed & (2**64 - 1), n_threads,
                                       _p(cent), _p(asg), _p(kap), nd, C.byref(ndo), C.byref(w)),
           "cluster_flat")
    return ClusterResult(cent[: kappa_total * dim], asg[: ids.size], kap, float(w.value))


def write_doc_layouts(doc_offsets, assignments, codes, pq_m: int) -> bytes:
    """storage.writeDocLayouts restated (oracle/mvr_oracle.c)."""
    off = np.ascontiguousarray(doc_offsets, dtype=np.uint64)
    a = _u32(assignments)
    c = np.ascontiguousarray(codes, dtype=np.uint8).reshape(-1)
    n_docs = off.size - 1
    cap = (n_docs + 1) * 8 + int(sum(((4 + int(off[d + 1] - off[d]) * (4 + pq_m)) + 7) // 8 * 8
                                    for d in range(n_docs))) + 8
    out = np.zeros(cap, dtype=np.uint8)
    lib = load()
    lib.orc_write_doc_layouts.restype = C.c_uint64
    n = lib.orc_write_doc_layouts(_p(off), C.c_uint64(n_docs), _p(a), _p(c), C.c_uint32(pq_m), _p(out),
                                  C.c_uint64(cap))
    if n == 0:
        raise OracleError(18, "write_doc_layouts")
    return out[:n].tobytes()


def dot(a, b) -> float:
    a, b = _f32(a), _f32(b)
    lib = load()
    lib.orc_dot.restype = C.c_float
    return float(lib.orc_dot(_p(a), _p(b), C.c_uint32(a.size)))


def pq_distance_table(codebooks, dim: int, pq_m: int, query, n_q: int) -> np.ndarray:
    q = _f32(query)
    out = np.zeros(pq_m * 256 * n_q, dtype=np.float32)
    _check(load().orc_pq_distance_table(_p(_f32(codebooks)), dim, pq_m, _p(q), C.c_uint64(q.size), n_q, _p(out),
                                        C.c_uint64(out.size)), "pq_distance_table")
    return out


def refine(centroids, dim: int, pq_m: int, doc_section: bytes, n_docs: int, doc_token_offsets, norms, table,
           query, n_q: int, doc_id: int) -> float:
    sec = np.frombuffer(doc_section, dtype=np.uint8)
    off = np.ascontiguousarray(doc_token_offsets, dtype=np.uint64)
    t, q = _f32(table), _f32(query)
    out = C.c_float(0)
    _check(load().orc_refine(_p(_f32(centroids)), dim, pq_m, _p(np.ascontiguousarray(sec)), C.c_uint64(n_docs),
                             _p(off), _p(_f32(norms)), _p(t), C.c_uint64(t.size), _p(q), C.c_uint64(q.size), n_q,
                             doc_id, C.byref(out)), "refine")
    return float(out.value)


# ---- HNSW over the centroids (hnsw_oracle.c, src/index/hnsw.zig) ----

@dataclass
class HnswGraph:
    """Frozen per-layer CSR graph, the reference's ``Hnsw`` (hnsw.zig:136-170)."""
    n: int
    dim: int
    entry_point: int
    max_level: int
    node_levels: np.ndarray  # u8[n]
    layer_offsets: list  # per layer u32[n + 1]
    layer_neighbours: list  # per layer u32[offsets[-1]]


class _HnswStats(C.Structure):
    _fields_ = [(f, C.c_uint64) for f in ("searches", "expansions", "sims", "accepted", "heur_examined",
                                            "heur_dots")]


def hnsw_build(centroids, dim: int, seed: int, ef_construction: int = 1500, m: int = 32, n_threads: int = 2,
               workers: int = 0) -> HnswGraph:
    """hnsw.build (hnsw.zig:314-475) on already normalised centroids."""
    import os
    x = _f32(centroids)
    lib = load()
    lib.orc_hnsw_build.restype = C.c_int
    lib.orc_hnsw_build.argtypes = [_P, C.c_uint64, C.c_uint32, C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32,
                                   C.c_uint32, C.POINTER(C.c_void_p)]
    h = C.c_void_p()
    w = workers or (os.cpu_count() or 1)
    _check(lib.orc_hnsw_build(_p(x), C.c_uint64(x.size), dim, C.c_uint64(seed & (2**64 - 1)), ef_construction, m,
                              n_threads, w, C.byref(h)), "hnsw_build")
    try:
        n, ep, ml = C.c_uint32(), C.c_uint32(), C.c_uint32()
        lib.orc_hnsw_info.argtypes = [C.c_void_p, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                                      C.POINTER(C.c_uint32)]
        lib.orc_hnsw_info(h, C.byref(n), C.byref(ep), C.byref(ml))
        levels = np.zeros(n.value, dtype=np.uint8)
        lib.orc_hnsw_levels.argtypes = [C.c_void_p, _P]
        lib.orc_hnsw_levels(h, _p(levels))
        lib.orc_hnsw_layer_size.restype = C.c_uint64
        lib.orc_hnsw_layer_size.argtypes = [C.c_void_p, C.c_uint32]
        lib.orc_hnsw_layer.argtypes = [C.c_void_p, C.c_uint32, _P, _P]
        offs, nbrs = [], []
        for L in range(ml.value + 1):
            o = np.zeros(n.value + 1, dtype=np.uint32)
            b = np.zeros(max(1, lib.orc_hnsw_layer_size(h, L)), dtype=np.uint32)
            lib.orc_hnsw_layer(h, L, _p(o), _p(b))
            offs.append(o)
            nbrs.append(b[: int(o[-1])])
        return HnswGraph(n.value, dim, ep.value, ml.value, levels, offs, nbrs)
    finally:
        lib.orc_hnsw_free.argtypes = [C.c_void_p]
        lib.orc_hnsw_free(h)


def hnsw_last_stats() -> dict:
    st = _HnswStats()
    lib = load()
    lib.orc_hnsw_last_stats.argtypes = [C.c_void_p]
    lib.orc_hnsw_last_stats(C.byref(st))
    return {f: int(getattr(st, f)) for f, _ in _HnswStats._fields_}


def hnsw_search(g: HnswGraph, centroids, query, k: int, ef: int) -> np.ndarray:
    """hnsw.search (hnsw.zig:1117-1150): top-k node ids, most similar first."""
    x, q = _f32(centroids), _f32(query)
    lib = load()
    offs = [np.ascontiguousarray(o, dtype=np.uint32) for o in g.layer_offsets]
    nbrs = [np.ascontiguousarray(b if b.size else np.zeros(1, np.uint32), dtype=np.uint32)
            for b in g.layer_neighbours]
    po = (C.c_void_p * len(offs))(*[o.ctypes.data for o in offs])
    pn = (C.c_void_p * len(nbrs))(*[b.ctypes.data for b in nbrs])
    out = np.zeros(max(k, 1), dtype=np.uint32)
    wr = C.c_uint32()
    lib.orc_hnsw_search_csr.argtypes = [_P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p,
                                        C.c_void_p, _P, C.c_uint32, C.c_uint32, _P, C.POINTER(C.c_uint32)]
    _check(lib.orc_hnsw_search_csr(_p(x), g.n, g.dim, g.entry_point, g.max_level, po, pn, _p(q), k, ef, _p(out),
                                   C.byref(wr)), "hnsw_search")
    return out[: wr.value].copy()


def normalize_rows(v, dim: int) -> np.ndarray:
    """vec.normalizeRowsInPlace (vec.zig:185-253) on a copy."""
    x = _f32(v).copy()
    lib = load()
    lib.orc_normalize_rows.argtypes = [_P, C.c_uint64, C.c_uint32]
    lib.orc_normalize_rows(_p(x), C.c_uint64(x.size // dim), dim)
    return x


# ---------------------------------------------------------------- .tac image

class TacParts(C.Structure):
    """Mirror of mvr_tac_parts (include/mvr.h): the reference's BuildOutput."""

    _fields_ = [("dim", C.c_uint32), ("kappa", C.c_uint32), ("sub_dim", C.c_uint32), ("pq_m", C.c_uint32),
                ("n_docs", C.c_uint64), ("n_tokens", C.c_uint64),
                ("centroids", C.c_void_p), ("assignments", C.c_void_p), ("pq_codes", C.c_void_p),
                ("doc_offsets", C.c_void_p), ("codebooks", C.c_void_p),
                ("hnsw_n", C.c_uint32), ("hnsw_entry_point", C.c_uint32), ("hnsw_max_level", C.c_uint32),
                ("hnsw_node_levels", C.c_void_p), ("hnsw_layer_offsets", C.c_void_p),
                ("hnsw_layer_neighbours", C.c_void_p), ("ilist_offsets", C.c_void_p),
                ("ilist_payload", C.c_void_p), ("residual_norms", C.c_void_p)]


class TacView(C.Structure):
    _fields_ = [("version", C.c_uint32), ("dim", C.c_uint32), ("kappa", C.c_uint32), ("pq_m", C.c_uint32),
                ("pq_bits", C.c_uint32), ("sub_dim", C.c_uint32), ("n_docs", C.c_uint64),
                ("n_tokens", C.c_uint64), ("centroids_off", C.c_uint64), ("hnsw_n", C.c_uint32),
                ("hnsw_entry_point", C.c_uint32), ("hnsw_max_level", C.c_uint32), ("hnsw_levels_off", C.c_uint64),
                ("hnsw_layer_offsets_off", C.c_uint64 * 256), ("hnsw_layer_neighbours_off", C.c_uint64 * 256),
                ("hnsw_layer_edges", C.c_uint64 * 256), ("pq_off", C.c_uint64), ("ilist_offsets_off", C.c_uint64),
                ("ilist_payload_off", C.c_uint64), ("ilist_total", C.c_uint64), ("doc_index_off", C.c_uint64),
                ("doc_payload_off", C.c_uint64), ("doc_payload_len", C.c_uint64), ("doc_tok_off", C.c_uint64),
                ("norms_off", C.c_uint64), ("footer_off", C.c_uint64)]


def crc32(data: bytes) -> int:
    b = np.frombuffer(data, dtype=np.uint8)
    return int(load().orc_crc32(_p(b) if b.size else None, b.size))


def inverted_lists_build(assignments, doc_offsets, kappa: int):
    """inverted_list.build restated: (offsets kappa+1 u64, payload u32)."""
    a = _u32(assignments)
    off = np.ascontiguousarray(doc_offsets, dtype=np.uint64)
    offsets = np.zeros(int(kappa) + 1, dtype=np.uint64)
    payload = np.zeros(max(1, a.size), dtype=np.uint32)
    total = C.c_uint64(0)
    _check(load().orc_inverted_lists_build(_p(a) if a.size else None, a.size, _p(off) if off.size else None,
                                           off.size, int(kappa), _p(offsets), _p(payload), payload.size,
                                           C.byref(total)), "inverted_lists_build")
    return offsets, payload[: total.value].copy()


def tac_parts(*, dim, kappa, sub_dim, pq_m, centroids, assignments, pq_codes, doc_offsets, codebooks,
              hnsw_entry_point, hnsw_node_levels, hnsw_layer_offsets, hnsw_layer_neighbours, ilist_offsets,
              ilist_payload, residual_norms):
    """A TacParts plus the arrays it points into (keep both alive)."""
    keep = {
        "centroids": np.ascontiguousarray(centroids, dtype=np.float32).reshape(-1),
        "assignments": np.ascontiguousarray(assignments, dtype=np.uint32).reshape(-1),
        "pq_codes": np.ascontiguousarray(pq_codes, dtype=np.uint8).reshape(-1),
        "doc_offsets": np.ascontiguousarray(doc_offsets, dtype=np.uint64),
        "codebooks": np.ascontiguousarray(codebooks, dtype=np.float32).reshape(-1),
        "levels": np.ascontiguousarray(hnsw_node_levels, dtype=np.uint8),
        "offs": [np.ascontiguousarray(o, dtype=np.uint32) for o in hnsw_layer_offsets],
        "nbrs": [np.ascontiguousarray(o, dtype=np.uint32) for o in hnsw_layer_neighbours],
        "ilo": np.ascontiguousarray(ilist_offsets, dtype=np.uint64),
        "ilp": np.ascontiguousarray(ilist_payload, dtype=np.uint32),
        "norms": np.ascontiguousarray(residual_norms, dtype=np.float32).reshape(-1),
    }
    L = len(keep["offs"])
    keep["offp"] = (C.c_void_p * L)(*[o.ctypes.data for o in keep["offs"]])
    keep["nbrp"] = (C.c_void_p * L)(*[(o.ctypes.data if o.size else keep["offs"][0].ctypes.data)
                                      for o in keep["nbrs"]])
    p = TacParts()
    p.dim, p.kappa, p.sub_dim, p.pq_m = dim, kappa, sub_dim, pq_m
    p.n_docs = keep["doc_offsets"].size - 1
    p.n_tokens = keep["assignments"].size
    p.centroids = keep["centroids"].ctypes.data
    p.assignments = keep["assignments"].ctypes.data
    p.pq_codes = keep["pq_codes"].ctypes.data
    p.doc_offsets = keep["doc_offsets"].ctypes.data
    p.codebooks = keep["codebooks"].ctypes.data
    p.hnsw_n = keep["levels"].size
    p.hnsw_entry_point = hnsw_entry_point
    p.hnsw_max_level = L - 1
    p.hnsw_node_levels = keep["levels"].ctypes.data
    p.hnsw_layer_offsets = C.cast(keep["offp"], C.c_void_p)
    p.hnsw_layer_neighbours = C.cast(keep["nbrp"], C.c_void_p)
    p.ilist_offsets = keep["ilo"].ctypes.data
    p.ilist_payload = keep["ilp"].ctypes.data if keep["ilp"].size else keep["ilo"].ctypes.data
    p.residual_norms = keep["norms"].ctypes.data
    return p, keep


def tac_serialise(parts_and_keep) -> bytes:
    """storage.serialise restated: the whole image (computeSize bytes)."""
    p, _keep = parts_and_keep
    lib = load()
    n = int(lib.orc_tac_file_size(C.byref(p)))
    buf = np.zeros(n, dtype=np.uint8)
    w = C.c_uint64(0)
    _check(lib.orc_tac_serialise(C.byref(p), _p(buf), n, C.byref(w)), "tac_serialise")
    return buf[: w.value].tobytes()


def tac_parse(image: bytes, reader_pq_m: int) -> dict:
    """storage.parse restated: every section as numpy arrays (copies).
    Raises OracleError with the reference's StorageError code."""
    b = np.frombuffer(image, dtype=np.uint8)
    v = TacView()
    _check(load().orc_tac_parse(_p(b) if b.size else None, b.size, int(reader_pq_m), C.byref(v)), "tac_parse")

    def arr(off, dtype, count):
        return np.frombuffer(image, dtype=dtype, count=int(count), offset=int(off)).copy()

    n = v.hnsw_n
    layers_off = [arr(v.hnsw_layer_offsets_off[L], np.uint32, n + 1) for L in range(v.hnsw_max_level + 1)]
    layers_nbr = [arr(v.hnsw_layer_neighbours_off[L], np.uint32, v.hnsw_layer_edges[L])
                  for L in range(v.hnsw_max_level + 1)]
    return {
        "header": {k: getattr(v, k) for k in ("version", "dim", "kappa", "pq_m", "pq_bits", "sub_dim", "n_docs",
                                             "n_tokens")},
        "centroids": arr(v.centroids_off, np.float32, v.kappa * v.dim),
        "hnsw": {"n": n, "entry_point": v.hnsw_entry_point, "max_level": v.hnsw_max_level,
                 "node_levels": arr(v.hnsw_levels_off, np.uint8, n), "layer_offsets": layers_off,
                 "layer_neighbours": layers_nbr},
        "codebooks": arr(v.pq_off, np.float32, v.pq_m * 256 * v.sub_dim),
        "ilist_offsets": arr(v.ilist_offsets_off, np.uint64, v.kappa + 1),
        "ilist_payload": arr(v.ilist_payload_off, np.uint32, v.ilist_total),
        "doc_index": arr(v.doc_index_off, np.uint64, v.n_docs + 1),
        "doc_section": bytes(image[v.doc_index_off: v.doc_payload_off + v.doc_payload_len]),
        "doc_token_offsets": arr(v.doc_tok_off, np.uint64, v.n_docs + 1),
        "residual_norms": arr(v.norms_off, np.float32, v.n_tokens),
    }
