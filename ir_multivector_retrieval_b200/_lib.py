"""ctypes binding of ``libmvr_b200.so`` (the C ABI in ``include/mvr.h``).

The shared library is the product; this module only declares its
signatures. It fails loudly when the library is missing: there is no CPU
fallback anywhere in the package.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "libmvr_b200.so"

# Status codes of include/mvr.h, named after the reference's Zig errors.
WAIT_LIMIT_DEFAULT = 4194304  # MVR_WAIT_LIMIT_DEFAULT in include/mvr.h

STATUS_NAMES = {
    0: "Ok",
    1: "KmeansBudgetTooSmall",
    2: "EmptyVectorSet",
    3: "DimMismatch",
    4: "DimNotDivisibleByM",
    5: "EmptyCorpus",
    6: "OutBufferWrongSize",
    7: "NQMismatch",
    8: "EmptyDistribution",
    9: "NonFinite",
    10: "AllZero",
    11: "BudgetTooSmall",
    12: "BudgetTooLarge",
    13: "InvalidThresholds",
    14: "EmptyTokenDump",
    15: "LengthMismatch",
    16: "EmptyInput",
    17: "OutOfMemory",
    18: "BufferTooSmall",
    19: "QueryShapeMismatch",
    20: "TableSizeMismatch",
    21: "DocOutOfRange",
    22: "DocLayoutCorrupt",
    23: "InvalidIndex",
    24: "UnsupportedVersion",
    25: "IndexCorrupt",
    26: "AssignmentOutOfRange",
    27: "DocOffsetsBad",
    28: "KappaZero",
    100: "CudaError",
    101: "NcclError",
    102: "Timeout",
    103: "InvalidArgument",
    104: "NoDevice",
    105: "DeviceLimit",
}
CODES = {v: k for k, v in STATUS_NAMES.items()}


class MvrError(Exception):
    """A failing status from the library. ``name`` is the reference's Zig
    error name (e.g. ``"DimNotDivisibleByM"``)."""

    def __init__(self, code: int, message: str = ""):
        self.code = int(code)
        self.name = STATUS_NAMES.get(self.code, f"Status{code}")
        super().__init__(f"{self.name}: {message}" if message else self.name)


class PqTrainStats(C.Structure):
    _fields_ = [
        ("seed_ms", C.c_double),
        ("lloyd_ms", C.c_double),
        ("total_ms", C.c_double),
        ("iters_max", C.c_uint32),
        ("iters_min", C.c_uint32),
        ("seed_fallbacks", C.c_uint32),
        ("reseeds", C.c_uint32),
        ("assign_ms", C.c_double),
        ("assign_launches", C.c_uint32),
        ("launches", C.c_uint32),
        ("assign_first_ms", C.c_double),
        ("lloyd_rows_total", C.c_uint64),
        ("lloyd_rows_exact", C.c_uint64),
        ("filter_rows_rechecked", C.c_uint64),
        ("filter_violations", C.c_uint32),
        ("seed_update_ms_sampled", C.c_double),
        ("seed_update_samples", C.c_uint32),
        ("list_ms", C.c_double),
        ("list_launches", C.c_uint32),
        ("list_distances", C.c_uint64),
        ("groups", C.c_uint32),
        ("host_enqueue_ms", C.c_double),
    ]


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


class TacStats(C.Structure):
    _fields_ = [
        ("total_ms", C.c_double),
        ("host_ms", C.c_double),
        ("h2d_ms", C.c_double),
        ("spread_ms", C.c_double),
        ("seed_ms", C.c_double),
        ("lloyd_ms", C.c_double),
        ("d2h_ms", C.c_double),
        ("problems", C.c_uint32),
        ("iters_max", C.c_uint32),
        ("seed_fallbacks", C.c_uint32),
        ("launches", C.c_uint32),
        ("filter_rows_rechecked", C.c_uint64),
        ("filter_violations", C.c_uint32),
        ("filter_rows_full_scan", C.c_uint64),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


class ClusteringParams(C.Structure):
    _fields_ = [
        ("kappa_total", C.c_uint32),
        ("mu", C.c_uint32),
        ("tau", C.c_uint32),
        ("epsilon", C.c_uint32),
        ("theta", C.c_uint32),
        ("max_iters", C.c_uint32),
        ("tol", C.c_float),
        ("seed", C.c_uint64),
        ("n_threads", C.c_uint32),
    ]


_P = C.c_void_p
_F = C.POINTER(C.c_float)
_U8 = C.POINTER(C.c_uint8)
_U32 = C.POINTER(C.c_uint32)
_U64 = C.POINTER(C.c_uint64)

# name -> (restype, argtypes)
SIGNATURES = {
    "mvr_ctx_create": (C.c_int, [C.c_int, C.POINTER(_P)]),
    "mvr_ctx_destroy": (C.c_int, [_P]),
    "mvr_last_error": (C.c_char_p, [_P]),
    "mvr_status_name": (C.c_char_p, [C.c_int]),
    "mvr_ctx_set_stream": (C.c_int, [_P, _P]),
    "mvr_ctx_trim": (C.c_int, [_P]),
    "mvr_ctx_sync": (C.c_int, [_P]),
    "mvr_tac_last_stats": (C.c_int, [_P, C.POINTER(TacStats)]),
    "mvr_ctx_set_serial_draws": (C.c_int, [_P, C.c_int]),
    "mvr_doc_layouts_bytes": (C.c_int, [_P, C.c_uint64, C.c_uint32, C.POINTER(C.c_uint64)]),
    "mvr_write_doc_layouts": (C.c_int, [_P, _P, C.c_uint64, _P, _P, C.c_uint64, C.c_uint32, _P, C.c_uint64]),
    "mvr_write_doc_layouts_device": (C.c_int, [_P, _P, C.c_uint64, _P, _P, C.c_uint64, C.c_uint32, _P, C.c_uint64]),
    "mvr_crc32": (C.c_uint32, [C.c_uint32, _P, C.c_uint64]),
    "mvr_crc32_combine": (C.c_uint32, [C.c_uint32, C.c_uint32, C.c_uint64]),
    "mvr_inverted_lists_build": (C.c_int, [_P, _P, C.c_uint64, _P, C.c_uint64, C.c_uint32, _P, _P, C.c_uint64,
                                           C.POINTER(C.c_uint64)]),
    "mvr_tac_file_size": (C.c_int, [_P, C.POINTER(C.c_uint64)]),
    "mvr_tac_serialise": (C.c_int, [_P, _P, _P, C.c_uint64, C.POINTER(C.c_uint64)]),
    "mvr_pq_distance_table": (C.c_int, [_P, _P, C.c_uint32, C.c_uint32, _P, C.c_uint64, C.c_uint32, _P, C.c_uint64]),
    "mvr_pq_distance_table_device": (
        C.c_int, [_P, _P, C.c_uint32, C.c_uint32, _P, C.c_uint64, C.c_uint32, _P, C.c_uint64]),
    "mvr_refine_batch": (
        C.c_int,
        [_P, _P, C.c_uint32, C.c_uint32, C.c_uint32, _P, C.c_uint64, C.c_uint64, _P, _P, C.c_uint64, _P, C.c_uint64,
         _P, C.c_uint64, C.c_uint32, _P, C.c_uint64, _P],
    ),
    "mvr_refine_batch_device": (
        C.c_int,
        [_P, _P, C.c_uint32, C.c_uint32, C.c_uint32, _P, C.c_uint64, C.c_uint64, _P, _P, C.c_uint64, _P, C.c_uint64,
         _P, C.c_uint64, C.c_uint32, _P, C.c_uint64, _P, _P],
    ),
    "mvr_ctx_set_exhaustive_assign": (C.c_int, [_P, C.c_int]),
    "mvr_ctx_set_tensor_filter": (C.c_int, [_P, C.c_int]),
    "mvr_ctx_set_pq_tensor_filter": (C.c_int, [_P, C.c_int]),
    "mvr_ctx_set_wait_limit": (C.c_int, [_P, C.c_uint32]),
    "mvr_ctx_set_candidate_scan": (C.c_int, [_P, C.c_int]),
    "mvr_ctx_set_pq_groups": (C.c_int, [_P, C.c_int]),
    "mvr_measure_f32x2_rate": (C.c_int, [_P, C.POINTER(C.c_double)]),
    "mvr_ctx_filter_report": (C.c_int, [_P, _U64, _U64]),
    "mvr_comm_unique_id_bytes": (C.c_size_t, []),
    "mvr_comm_unique_id": (C.c_int, [_P, C.c_size_t]),
    "mvr_ctx_init_comm": (C.c_int, [_P, C.c_int, C.c_int, _P, C.c_size_t]),
    "mvr_ctx_comm_size": (C.c_int, [_P]),
    "mvr_ctx_comm_rank": (C.c_int, [_P]),
    "mvr_pq_train_sharded_device": (
        C.c_int,
        [_P, _P, C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint32, C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32,
         C.c_float, _P, _P, C.POINTER(PqTrainStats)],
    ),
    "mvr_kmeans_fit": (
        C.c_int,
        [_P, _P, C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_float, C.c_uint64,
         C.c_uint32, _P, _P, _P, _P],
    ),
    "mvr_kmeans_fit_noalloc": (
        C.c_int,
        [_P, C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_float, C.c_uint64, _P, _P, _P, _P, _P],
    ),
    "mvr_pq_train": (
        C.c_int,
        [_P, _P, C.c_uint64, C.c_uint32, C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32,
         C.c_float, _P, C.POINTER(PqTrainStats)],
    ),
    "mvr_pq_train_device": (
        C.c_int,
        [_P, _P, C.c_uint64, C.c_uint32, C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32,
         C.c_float, _P, C.POINTER(PqTrainStats)],
    ),
    "mvr_pq_encode": (C.c_int, [_P, _P, C.c_uint32, C.c_uint32, _P, C.c_uint64, _P]),
    "mvr_pq_encode_device": (C.c_int, [_P, _P, C.c_uint32, C.c_uint32, _P, C.c_uint64, _P]),
    "mvr_pq_decode": (C.c_int, [_P, C.c_uint32, C.c_uint32, _P, C.c_uint64, _P]),
    "mvr_residuals_norms": (
        C.c_int, [_P, _P, _P, C.c_uint32, _P, C.c_uint64, C.c_uint32, _P, _P]),
    "mvr_residuals_norms_device": (
        C.c_int, [_P, _P, _P, C.c_uint32, _P, C.c_uint64, C.c_uint32, _P, _P]),
    "mvr_clustering_params_default": (None, [C.POINTER(ClusteringParams), C.c_uint32, C.c_uint64]),
    "mvr_tac_cluster_flat": (
        C.c_int,
        [_P, _P, C.c_uint64, _P, C.c_uint64, C.c_uint32, C.POINTER(ClusteringParams), _P, _P,
         _P, C.c_uint64, _U64, _F],
    ),
    "mvr_tac_cluster_flat_sharded": (
        C.c_int,
        [_P, _P, C.c_uint64, _P, C.c_uint64, C.c_uint32, C.POINTER(ClusteringParams), _P, _P,
         _P, C.c_uint64, _U64, _F],
    ),
    "mvr_tac_partition_tokens": (C.c_int, [_P, _P, C.c_uint64, C.c_uint32, _P]),
    "mvr_hnsw_build": (C.c_int, [_P, _P, C.c_uint64, C.c_uint32, C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32,
                                 C.POINTER(C.c_void_p)]),
    "mvr_hnsw_build_device": (C.c_int, [_P, _P, C.c_uint64, C.c_uint32, C.c_uint64, C.c_uint32, C.c_uint32,
                                        C.c_uint32, C.POINTER(C.c_void_p)]),
    "mvr_hnsw_info": (None, [_P, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                             C.POINTER(C.c_float), C.POINTER(C.c_uint64)]),
    "mvr_hnsw_node_levels": (C.POINTER(C.c_uint8), [_P]),
    "mvr_hnsw_layer_offsets": (C.POINTER(C.c_uint32), [_P, C.c_uint32]),
    "mvr_hnsw_layer_neighbours": (C.POINTER(C.c_uint32), [_P, C.c_uint32, C.POINTER(C.c_uint64)]),
    "mvr_hnsw_free": (None, [_P]),
    "mvr_normalize_rows": (C.c_int, [_P, _P, C.c_uint64, C.c_uint32]),
    "mvr_normalize_rows_device": (C.c_int, [_P, _P, C.c_uint64, C.c_uint32]),
    "mvr_tac_allocate_budgets": (
        C.c_int, [_P, _P, _P, _P, C.c_uint64, C.c_uint32, C.POINTER(ClusteringParams)]),
}

_lib = None
_lock = threading.Lock()


def load() -> C.CDLL:
    """Load the shared library (once). Raises if it has not been built."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with "
                    "`python -m ir_multivector_retrieval_b200.build` (there is no CPU fallback)"
                )
            lib = C.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
        return _lib


def ptr(a) -> C.c_void_p:
    """Raw address of a numpy array or a torch tensor (device or host)."""
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        return C.c_void_p(a.ctypes.data)
    if hasattr(a, "data_ptr"):
        return C.c_void_p(a.data_ptr())
    raise TypeError(f"cannot take the address of {type(a)!r}")


class Context:
    """A CUDA device context of the library (``mvr_ctx``)."""

    def __init__(self, device: int = 0):
        self.lib = load()
        h = C.c_void_p()
        st = self.lib.mvr_ctx_create(int(device), C.byref(h))
        if st != 0:
            raise MvrError(st, f"mvr_ctx_create(device={device})")
        self.handle = h
        self.device = device

    def check(self, status: int, what: str = "") -> None:
        if status != 0:
            msg = self.lib.mvr_last_error(self.handle)
            raise MvrError(status, (msg.decode() if msg else "") or what)

    def set_stream(self, stream_handle: int | None) -> None:
        self.check(self.lib.mvr_ctx_set_stream(self.handle, C.c_void_p(stream_handle or 0)))

    def sync(self) -> None:
        self.check(self.lib.mvr_ctx_sync(self.handle))

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.mvr_ctx_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_default: dict[int, Context] = {}


def default_context(device: int | None = None) -> Context:
    """Per-device shared context used by the reference-style functions."""
    dev = int(os.environ.get("MVR_DEVICE", "0")) if device is None else int(device)
    with _lock:
        ctx = _default.get(dev)
    if ctx is None:
        ctx = Context(dev)
        with _lock:
            _default[dev] = ctx
    return ctx
