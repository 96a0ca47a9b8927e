"""Row-sharded pq.train on the GPU: the sharded entry point without a
communicator equals the one-GPU entry point, and (with two or more GPUs) a
torch.distributed run of tests/dist_worker.py gives every rank the one-GPU
codebooks byte for byte."""
import ctypes as C
import math
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from ir_multivector_retrieval_b200 import synth
from ir_multivector_retrieval_b200._lib import MvrError, PqTrainStats

THREADS = max(1, os.cpu_count() or 1)

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def test_sharded_entry_without_comm_is_the_one_gpu_path(ctx, orc):
    torch = pytest.importorskip("torch")
    x = synth.unit_rows(20_000, 64, seed=12)
    dx = torch.from_numpy(x).cuda()
    a = torch.empty(16 * 256 * 4, dtype=torch.float32, device="cuda")
    b = torch.empty_like(a)
    asg = torch.empty(16 * 20_000, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    ctx.check(ctx.lib.mvr_pq_train_device(ctx.handle, C.c_void_p(dx.data_ptr()), x.size, 64, 5, 1, 16, 6,
                                          C.c_float(-math.inf), C.c_void_p(a.data_ptr()), None))
    st = PqTrainStats()
    ctx.check(ctx.lib.mvr_pq_train_sharded_device(ctx.handle, C.c_void_p(dx.data_ptr()), 20_000, 0, 20_000, 64, 5,
                                                  1, 16, 6, C.c_float(-math.inf), C.c_void_p(b.data_ptr()),
                                                  C.c_void_p(asg.data_ptr()), C.byref(st)))
    assert a.cpu().numpy().tobytes() == b.cpu().numpy().tobytes()
    want = orc.pq_train(x, 64, 5, 16, n_threads=8, max_iters=6, tol=-math.inf)
    assert b.cpu().numpy().tobytes() == want.tobytes()
    with pytest.raises(MvrError) as e:
        ctx.check(ctx.lib.mvr_pq_train_sharded_device(ctx.handle, C.c_void_p(dx.data_ptr()), 10_000, 10_000,
                                                      20_000, 64, 5, 1, 16, 6, C.c_float(-math.inf),
                                                      C.c_void_p(b.data_ptr()), None, None))
    assert e.value.name == "InvalidArgument"


def test_serial_draws_mode_matches(ctx, orc):
    """Every draw through the reference's serial chain gives the same bytes."""
    x = synth.unit_rows(9_000, 32, seed=2)
    from ir_multivector_retrieval_b200 import pq

    st_fast, st_serial = {}, {}
    fast = pq.train(x, 32, 3, pq_m=16, max_iters=10, ctx=ctx, stats=st_fast)
    ctx.check(ctx.lib.mvr_ctx_set_serial_draws(ctx.handle, 1))
    try:
        serial = pq.train(x, 32, 3, pq_m=16, max_iters=10, ctx=ctx, stats=st_serial)
    finally:
        ctx.check(ctx.lib.mvr_ctx_set_serial_draws(ctx.handle, 0))
    assert st_serial["seed_fallbacks"] == 16 * 255 and st_fast["seed_fallbacks"] == 0
    assert fast.codebooks.tobytes() == serial.codebooks.tobytes()
    assert serial.codebooks.tobytes() == orc.pq_train(x, 32, 3, 16, n_threads=8, max_iters=10).tobytes()


def test_serial_draws_mode_matches_large_n(ctx, orc):
    """Above 2^18 rows an undecided draw runs the reference's sequential f64
    chain chunk by chunk (binade-exact steps for clean chunks, the weights one
    by one for the others): every draw through it gives the same bytes as
    the interval-bounded draws and the oracle, including data with many
    equal and zero weights and sums that cross many binades."""
    from ir_multivector_retrieval_b200 import pq

    rng = np.random.default_rng(5)
    x = synth.unit_rows(300_000, 16, seed=4)
    x[rng.integers(0, 300_000, 40_000)] = x[7]            # exact duplicates: zero weights
    x[::97] *= np.float32(1e-3)                              # small weights over many binades
    for fast_first in (True, False):
        st = {}
        ctx.check(ctx.lib.mvr_ctx_set_serial_draws(ctx.handle, 0 if fast_first else 1))
        try:
            got = pq.train(x, 16, 9, pq_m=4, max_iters=3, tol=-math.inf, ctx=ctx, stats=st)
        finally:
            ctx.check(ctx.lib.mvr_ctx_set_serial_draws(ctx.handle, 0))
        if not fast_first:
            assert st["seed_fallbacks"] == 4 * 255
        want = orc.pq_train(x, 16, 9, 4, n_threads=THREADS, max_iters=3, tol=-math.inf)
        assert got.codebooks.tobytes() == want.tobytes()


def test_sharded_training_on_several_gpus():
    torch = pytest.importorskip("torch")
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two or more GPUs")
    world = min(n, 4)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=str(ROOT))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr=127.0.0.1", "--master-port=29517", str(ROOT / "tests" / "dist_worker.py")]
    r = subprocess.run(["timeout", "-k", "30", "300", *cmd], env=env, capture_output=True, text=True)
    out = r.stdout + r.stderr
    print(out[-4000:])
    assert r.returncode == 0, out[-4000:]
    assert "[dist] FAIL" not in out


def test_second_device_context_with_two_groups(orc):
    """A context on the second GPU: pq.train's second subspace group runs on
    its own host thread, which must work on the context's device (a new
    thread starts on device 0). Same bytes as the oracle, with one group and
    with two."""
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two or more GPUs")
    from ir_multivector_retrieval_b200 import Context, pq

    x = synth.unit_rows(30_000, 32, seed=21)
    want = orc.pq_train(x, 32, 4, 8, n_threads=THREADS, max_iters=5, tol=-math.inf)
    before = torch.cuda.current_device()
    with Context(1) as ctx1:
        for groups in (2, 1):
            ctx1.check(ctx1.lib.mvr_ctx_set_pq_groups(ctx1.handle, groups))
            st = {}
            got = pq.train(x, 32, 4, pq_m=8, max_iters=5, tol=-math.inf, ctx=ctx1, stats=st)
            assert st["groups"] == groups
            assert got.codebooks.tobytes() == want.tobytes()
            assert torch.cuda.current_device() == before  # entry points restore the caller's device
    assert torch.cuda.current_device() == before
