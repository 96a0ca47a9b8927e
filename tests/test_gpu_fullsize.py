"""Parity at the size the bench measures: the whole
1,521,797 x 64 corpus, against the CPU oracle on all host threads.

* pq.train, M = 16 x 4, 256 centroids, k-means++ and the full 20 Lloyd
  iterations (tol = -inf) with the build's seed (storage.zig:380: params.seed
  +% 0xa1b2c3d4): codebooks byte for byte (pq.zig:301-336,
  kmeans.zig:177-221), then PQ.encode of every row (pq.zig:59-76).
* tac.clusterFlat with kappa 32,768 and the paper-strict thresholds (mu 128,
  tau 256, eps 4, theta 39; tac.zig:458-514, :563-838): assignments,
  kappa_per_token, centroids and wcss_total byte for byte.

Bar: bit-exact. The oracle takes about a minute in total on 16 host cores.
"""
import math
import os

import numpy as np
import pytest

from ir_multivector_retrieval_b200 import pq, synth, tac

pytestmark = pytest.mark.gpu
THREADS = max(1, os.cpu_count() or 1)
N = 1_521_797
SEED = 42 + 0xA1B2C3D4


@pytest.fixture(scope="module")
def corpus():
    return synth.make_corpus(N, 64, seed=42)


def test_pq_train_20_iterations_and_encode_full_size(ctx, orc, corpus):
    x = synth.anchor_residuals(corpus)
    stats = {}
    got = pq.train(x, 64, SEED, pq_m=16, max_iters=20, tol=-math.inf, ctx=ctx, stats=stats)
    assert stats["iters_min"] == 20 and stats["iters_max"] == 20
    want = orc.pq_train(x, 64, SEED, 16, n_threads=THREADS, max_iters=20, tol=-math.inf)
    assert got.codebooks.tobytes() == want.tobytes()
    codes = got.encode_batch(x)
    assert np.array_equal(codes, orc.pq_encode(want, 64, 16, x, n_threads=THREADS))


def test_cluster_flat_full_size(ctx, orc, corpus):
    p = tac.ClusteringParams(kappa_total=32_768, seed=42)
    got = tac.cluster_flat(corpus.token_ids, corpus.vectors, 64, p, ctx=ctx)
    want = orc.tac_cluster_flat(corpus.token_ids, corpus.vectors, 64, 32_768, 42, max_iters=p.max_iters,
                                tol=p.tol, n_threads=p.n_threads, workers=THREADS)
    assert np.array_equal(got.kappa_per_token, want.kappa_per_token)
    assert np.array_equal(got.assignments, want.assignments)
    assert got.centroids.tobytes() == np.ascontiguousarray(want.centroids, dtype=np.float32).tobytes()
    assert np.float32(got.wcss_total).tobytes() == np.float32(want.wcss_total).tobytes()


def test_configs4_shape_on_a_row_sample(ctx, orc):
    """BASELINE configs[4]'s PQ shape (dim 128, M = 32 x 4, 256 centroids,
    25 Lloyd iterations) on a seeded 150,000-row block of its 50M-row corpus
    (made on the GPU): codebooks byte for byte, then the codes of the block."""
    import torch

    from ir_multivector_retrieval_b200 import synth

    xd, _ = synth.device_residuals(50_000_000, 128, seed=42, device="cuda", row0=12_000_000, n_rows=150_000)
    x = xd.cpu().numpy()
    got = pq.train(x, 128, SEED, pq_m=32, max_iters=25, tol=-math.inf, ctx=ctx)
    want = orc.pq_train(x, 128, SEED, 32, n_threads=THREADS, max_iters=25, tol=-math.inf)
    assert got.codebooks.tobytes() == want.tobytes()
    assert np.array_equal(got.encode_batch(x), orc.pq_encode(want, 128, 32, x, n_threads=THREADS))
    del xd
    torch.cuda.empty_cache()
