"""GPU parity of the build chain around the hot path: residuals + norms
(storage.residualsAndNormsChunk) and storage.build steps 1/3/4
(clusterFlat -> residuals -> pq.train -> encode) against the oracle chain.

Bar: bit-exact at every stage.
"""
import numpy as np
import pytest

from ir_multivector_retrieval_b200 import storage, synth, tac

pytestmark = pytest.mark.gpu
THREADS = 8


def _same(a, b):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return a.size == b.size and a.tobytes() == b.tobytes()


@pytest.mark.parametrize("n,dim,kappa", [(5_000, 64, 700), (3_001, 128, 300), (2_000, 17, 150), (700, 3, 40)])
def test_residuals_norms(ctx, orc, n, dim, kappa):
    rng = np.random.default_rng(n + dim)
    v = rng.standard_normal((n, dim)).astype(np.float32)
    c = rng.standard_normal((kappa, dim)).astype(np.float32)
    a = rng.integers(0, kappa, size=n).astype(np.uint32)
    v[7] = c[a[7]]  # a zero residual: norm 0, row left as is
    v[9, 0] = np.float32(1e-30) + c[a[9], 0]
    got_r, got_n = storage.residuals_and_norms(v, c, a, dim, ctx=ctx)
    want_r, want_n = orc.residuals_norms(v, c, a, dim)
    assert _same(got_r, want_r) and _same(got_n, want_n)
    assert got_n[7] == 0.0 and not np.any(got_r[7])


@pytest.mark.parametrize("n,dim,kappa,pq_m", [(20_000, 64, 4096, 16), (12_000, 64, 3000, 32), (9_000, 128, 2350, 32)])
def test_build_chain_matches_oracle(ctx, orc, n, dim, kappa, pq_m):
    c = synth.make_corpus(n, dim, seed=n)
    p = tac.ClusteringParams(kappa_total=kappa, seed=7, theta=10)
    got = storage.build_codes(c.token_ids, c.vectors, dim, p, pq_m=pq_m, ctx=ctx)
    cl = orc.tac_cluster_flat(c.token_ids, c.vectors, dim, kappa, 7, theta=10)
    assert np.array_equal(got.clustering.assignments, cl.assignments)
    assert _same(got.clustering.centroids, cl.centroids)
    res, norms = orc.residuals_norms(c.vectors, cl.centroids, cl.assignments, dim)
    assert _same(got.residuals, res) and _same(got.norms, norms)
    cb = orc.pq_train(res, dim, (7 + storage.PQ_SEED_OFFSET) & (2**64 - 1), pq_m, n_threads=THREADS)
    assert _same(got.pq.codebooks, cb)
    codes = orc.pq_encode(cb, dim, pq_m, res, n_threads=THREADS)
    assert np.array_equal(got.codes, codes)


@pytest.mark.parametrize("m", [16, 32, 3])
def test_doc_layouts_match_oracle(ctx, orc, m):
    rng = np.random.default_rng(m)
    n_d = rng.integers(0, 120, size=3_000)
    n_d[::17] = 0  # empty docs
    off = np.concatenate([[0], np.cumsum(n_d)]).astype(np.uint64)
    n = int(off[-1])
    asg = rng.integers(0, 2**32 - 1, size=n, dtype=np.uint64).astype(np.uint32)
    codes = rng.integers(0, 256, size=(n, m), dtype=np.uint8)
    got = storage.write_doc_layouts(off, asg, codes, m, ctx=ctx)
    want = orc.write_doc_layouts(off, asg, codes, m)
    assert got == want


def test_doc_layouts_device_entry_and_short_buffer(ctx, orc):
    torch = pytest.importorskip("torch")
    import ctypes as C

    from ir_multivector_retrieval_b200._lib import MvrError, ptr

    rng = np.random.default_rng(2)
    n_d = rng.integers(1, 60, size=500)
    off = np.concatenate([[0], np.cumsum(n_d)]).astype(np.uint64)
    n = int(off[-1])
    asg = rng.integers(0, 30_000, size=n).astype(np.uint32)
    codes = rng.integers(0, 256, size=(n, 16), dtype=np.uint8)
    size = storage.doc_layouts_bytes(off, 16)
    d_asg = torch.from_numpy(asg.view(np.int32)).cuda()
    d_codes = torch.from_numpy(codes).cuda()
    d_out = torch.empty(size, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    ctx.check(ctx.lib.mvr_write_doc_layouts_device(ctx.handle, ptr(off), off.size - 1, ptr(d_asg), ptr(d_codes), n,
                                                   16, ptr(d_out), size))
    ctx.sync()
    assert d_out.cpu().numpy().tobytes() == orc.write_doc_layouts(off, asg, codes, 16)
    with pytest.raises(MvrError) as e:
        ctx.check(ctx.lib.mvr_write_doc_layouts_device(ctx.handle, ptr(off), off.size - 1, ptr(d_asg),
                                                       ptr(d_codes), n, 16, ptr(d_out), size - 1))
    assert e.value.name == "BufferTooSmall"
    _ = C
