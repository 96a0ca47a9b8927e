"""B200-native PQ / k-means build path of the TAC multivector index.

Drop-in for the reference's ``pq.train``, ``PQ.encode``, ``kmeans.fit`` and
``tac.clusterFlat`` (BleedingDev/ir-multivector-retrieval). The compute runs
in ``libmvr_b200.so`` (hand-written sm_100a CUDA behind the C ABI of
``include/mvr.h``); these modules mirror the reference's interfaces.
"""
from ._lib import Context, MvrError, default_context, load  # noqa: F401

__all__ = ["Context", "MvrError", "default_context", "load", "pq", "kmeans", "synth"]
