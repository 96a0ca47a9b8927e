"""Several GPUs, one process per GPU: row-sharded ``pq.train``.

The reference trains on one host; here rank g of a ``torch.distributed``
group holds the contiguous rows ``shard_rows(n_total, world, g)`` on its GPU.
``init_comm`` joins each rank's library context to an NCCL communicator (the
unique id travels over the torch group, gloo or nccl); ``train_sharded`` then
returns on every rank the codebooks the one-GPU ``pq.train`` computes on the
whole matrix — byte for byte, for any number of ranks. The exchange steps
(all in the library, on the context stream): per k-means++ draw an
all-gather of per-chunk weight bounds plus the owner's row; per Lloyd
iteration an all-reduce of cluster counts and the in-order centroid sums
continued rank after rank (``relay_order`` models that step).
"""
from __future__ import annotations

import ctypes as C
import hashlib

import numpy as np

from . import _lib
from ._lib import PqTrainStats

PQ_CENTROIDS = 256


def shard_rows(n_total: int, world: int, rank: int) -> tuple[int, int]:
    """(row0, n_local) of rank's contiguous shard; sizes differ by at most 1."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world")
    lo = n_total * rank // world
    hi = n_total * (rank + 1) // world
    return lo, hi - lo


def exchange_unique_id(make_id, group=None) -> bytes:
    """Rank 0 makes the id (``make_id()``), every rank of the torch group
    receives it."""
    import torch.distributed as dist

    obj = [make_id() if dist.get_rank(group) == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]


def init_comm(ctx, group=None) -> None:
    """Join ``ctx`` to an NCCL communicator spanning the torch group."""
    import torch.distributed as dist

    lib = ctx.lib
    n = lib.mvr_comm_unique_id_bytes()

    def make():
        buf = (C.c_ubyte * n)()
        ctx.check(lib.mvr_comm_unique_id(buf, n))
        return bytes(buf)

    uid = exchange_unique_id(make, group)
    buf = (C.c_ubyte * n).from_buffer_copy(uid)
    ctx.check(lib.mvr_ctx_init_comm(ctx.handle, dist.get_world_size(group), dist.get_rank(group), buf, n))


def train_sharded(ctx, d_rows_ptr: int, n_local: int, row0: int, n_total: int, dim: int, seed: int, *,
                  pq_m: int, max_iters: int = 25, tol: float = 1e-4, d_codebooks_ptr: int,
                  d_assign_ptr: int | None = None) -> dict:
    """Row-sharded pq.train on device pointers (collective over the
    communicator); returns the timing report."""
    st = PqTrainStats()
    ctx.check(ctx.lib.mvr_pq_train_sharded_device(
        ctx.handle, C.c_void_p(d_rows_ptr), n_local, row0, n_total, dim, seed & (2**64 - 1), 1, pq_m, max_iters,
        C.c_float(tol), C.c_void_p(d_codebooks_ptr), C.c_void_p(d_assign_ptr) if d_assign_ptr else None,
        C.byref(st)))
    return {k: getattr(st, k) for k, _ in PqTrainStats._fields_}


def relay_order(shards, start=None):
    """Model of the Lloyd exchange step: f32 running sums carried through the
    shards in rank order, each rank adding its rows in row order. Equals the
    reference's single serial loop over the concatenated rows."""
    acc = np.float32(0) if start is None else np.float32(start)
    for rows in shards:
        for v in np.asarray(rows, dtype=np.float32):
            acc = np.float32(acc + v)
    return acc


def codebook_digest(codebooks) -> str:
    """sha256 of the codebook bytes (equal across GPU counts)."""
    return hashlib.sha256(np.ascontiguousarray(codebooks, dtype=np.float32).tobytes()).hexdigest()


__all__ = ["shard_rows", "exchange_unique_id", "init_comm", "train_sharded", "relay_order", "codebook_digest",
           "PQ_CENTROIDS"]
_ = _lib
