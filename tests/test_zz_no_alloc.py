"""``mvr_kmeans_fit_noalloc``: k-means for callers that cannot allocate GPU memory.

Hosts whose own allocator owns the device (or whose memory budget is fixed up front)
cannot let a library call cudaMalloc/cudaFree. This entry point takes device inputs and
outputs plus a stream and uses only a fixed scratch array compiled into the library. The
test calls it through the C ABI twice in a row, with different shapes, and checks each
result bit for bit against the ordinary entry point ``mvr_kmeans_fit`` and against the CPU
restatement of ``kmeans.fit``; further cases cover k >= n, no assignment output and the
largest accepted size. It lives in its own file, collected last, so a failure here does not
hide the other tests.
"""
import ctypes as C
import math

import numpy as np
import pytest

from ir_multivector_retrieval_b200 import _lib, kmeans

pytestmark = pytest.mark.gpu


def _call_noalloc(lib, dx, n, dim, k, iters, tol, seed, dcent, dasg, stream):
    w = C.c_float(0.0)
    it = C.c_uint32(0)
    st = lib.mvr_kmeans_fit_noalloc(
        C.c_void_p(dx.data_ptr()), n * dim, dim, k, iters, C.c_float(tol), seed,
        C.c_void_p(dcent.data_ptr()), C.c_void_p(dasg.data_ptr()) if dasg is not None else None,
        C.byref(w), C.byref(it), C.c_void_p(stream.cuda_stream))
    return st, w.value, it.value


def _run_case(torch, lib, stream, ctx, orc, n, dim, k, iters, tol, seed, with_assign=True):
    x = np.random.default_rng(seed).standard_normal(n * dim).astype(np.float32)
    want = kmeans.fit(x, dim, kmeans.KMeansParams(k=k, seed=seed, max_iters=iters, tol=tol), ctx=ctx)
    with torch.cuda.stream(stream):
        dx = torch.from_numpy(x).cuda()
        dcent = torch.full((k * dim,), float("nan"), dtype=torch.float32, device="cuda")
        dasg = torch.full((n,), -1, dtype=torch.int32, device="cuda") if with_assign else None
    st, wcss, iters_run = _call_noalloc(lib, dx, n, dim, k, iters, tol, seed, dcent, dasg, stream)
    assert st == 0, lib.mvr_status_name(st).decode()
    stream.synchronize()
    got_cent = dcent.cpu().numpy()
    # against the ordinary entry point (same library, allocating path) ...
    assert got_cent.tobytes() == want.centroids.tobytes()
    assert np.float32(wcss).tobytes() == np.float32(want.wcss).tobytes()
    assert iters_run == want.iters_run
    # ... and against the CPU restatement of kmeans.fit itself
    ref = orc.kmeans_fit(x, dim, k, seed, max_iters=iters, tol=tol)
    assert got_cent.tobytes() == np.ascontiguousarray(ref.centroids, dtype=np.float32).tobytes()
    assert np.float32(wcss).tobytes() == np.float32(ref.wcss).tobytes()
    assert iters_run == ref.iters_run
    if with_assign:
        got_asg = dasg.cpu().numpy().view(np.uint32)
        assert np.array_equal(got_asg, want.assignments)
        assert np.array_equal(got_asg, ref.assignments)


def test_noalloc_matches_kmeans_fit_on_two_calls(ctx, orc):
    torch = pytest.importorskip("torch")
    lib = _lib.load()
    stream = torch.cuda.Stream()
    # two calls in a row with different shapes: the second must not see the
    # first one's leftovers in the shared array
    _run_case(torch, lib, stream, ctx, orc, 5000, 4, 64, 25, 1e-4, 11)       # reference stopping rule
    _run_case(torch, lib, stream, ctx, orc, 3000, 2, 17, 12, -math.inf, 5)   # fixed iteration count, odd k


def test_noalloc_edge_shapes(ctx, orc):
    torch = pytest.importorskip("torch")
    lib = _lib.load()
    stream = torch.cuda.Stream()
    _run_case(torch, lib, stream, ctx, orc, 40, 4, 64, 25, 1e-4, 3)              # k >= n: degenerate path
    _run_case(torch, lib, stream, ctx, orc, 2000, 1, 9, 7, -math.inf, 8, with_assign=False)  # no assignments out
    _run_case(torch, lib, stream, ctx, orc, 65536, 4, 256, 6, -math.inf, 21)     # the largest accepted size


def test_noalloc_rejects_sizes_beyond_its_scratch(ctx):
    torch = pytest.importorskip("torch")
    lib = _lib.load()
    stream = torch.cuda.Stream()
    n = 65536 + 1  # MVR_NOALLOC_MAX_ROWS + 1
    with torch.cuda.stream(stream):
        dx = torch.zeros(n * 2, dtype=torch.float32, device="cuda")
        dcent = torch.zeros(8 * 2, dtype=torch.float32, device="cuda")
        dasg = torch.zeros(n, dtype=torch.int32, device="cuda")
    st, _, _ = _call_noalloc(lib, dx, n, 2, 8, 5, 1e-4, 1, dcent, dasg, stream)
    assert lib.mvr_status_name(st).decode() == "InvalidArgument"
    # and unsupported dims / k
    st, _, _ = _call_noalloc(lib, dx, 1000, 3, 8, 5, 1e-4, 1, dcent, dasg, stream)
    assert lib.mvr_status_name(st).decode() == "InvalidArgument"
