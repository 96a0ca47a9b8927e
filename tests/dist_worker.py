"""Worker of the multi-GPU parity test (launched by tests/test_gpu_dist.py
under torch.distributed.run, one process per GPU).

Every rank trains PQ codebooks on its contiguous row shard through
``mvr_pq_train_sharded_device``; rank 0 also trains on the whole matrix with
the one-GPU entry point. The codebooks must be byte-identical on every rank
and equal to the one-GPU result; the local assignments must equal the
matching rows of the one-GPU assignments. Then every rank runs the
token-sharded clusterFlat; its outputs must equal the one-GPU call's on every
rank. Exit status 0 = pass.
"""
import ctypes as C
import datetime
import hashlib
import math
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
from ir_multivector_retrieval_b200 import Context, dist as mdist, synth, tac  # noqa: E402
from ir_multivector_retrieval_b200._lib import PqTrainStats  # noqa: E402


def reseed_data(trial: int, S: int):
    """Seeded data whose Lloyd iterations empty a cluster (found by search):
    pq.train with pq_m = 1, seed = trial, tol = 0."""
    rng = np.random.default_rng(trial)
    n = int(rng.integers(260, 2000))
    return (rng.uniform(-1, 1, size=(n, S)) ** 5).astype(np.float32)


def case_data(name):
    if name == "reseed4":
        return reseed_data(1247, 4), 4, 1
    if name == "reseed2":
        return reseed_data(2902, 2), 2, 1
    if name == "dup":  # heavy duplication: zero weights, ties, possible empty clusters
        rng = np.random.default_rng(3)
        base = synth.unit_rows(300, 32, seed=4)
        return base[rng.integers(0, 300, size=12_000)], 32, 16
    if name == "m3":  # three subspaces: uneven subspace ranges over 2 or 4 ranks
        return synth.unit_rows(20_000, 12, seed=5), 12, 3
    if name == "s2":
        return synth.unit_rows(30_001, 32, seed=9), 32, 16
    return synth.unit_rows(50_000, 64, seed=7), 64, 16


def main() -> int:
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    ctx = Context(local)
    mdist.init_comm(ctx)
    assert ctx.lib.mvr_ctx_comm_size(ctx.handle) == world
    failures = []
    # pq_m >= ranks: subspace-sharded; pq_m = 1 (the reseed data): row-sharded
    cases = [("s4", 8, -math.inf, False), ("s2", 25, 1e-4, False), ("dup", 25, 1e-4, False), ("m3", 10, 1e-4, False),
             ("reseed4", 25, 0.0, False), ("reseed2", 25, 0.0, False), ("s4", 3, -math.inf, True),
             ("reseed2", 4, -math.inf, True)]
    for name, iters, tol, serial in cases:
        x, dim, pq_m = case_data(name)
        n_total = x.shape[0]
        row0, nl = mdist.shard_rows(n_total, world, rank)
        d_rows = torch.from_numpy(np.ascontiguousarray(x[row0:row0 + nl])).cuda()
        cb_n = pq_m * 256 * (dim // pq_m)
        d_cb = torch.empty(cb_n, dtype=torch.float32, device="cuda")
        d_asg = torch.empty(pq_m * nl, dtype=torch.int32, device="cuda")
        ctx.check(ctx.lib.mvr_ctx_set_serial_draws(ctx.handle, 1 if serial else 0))
        torch.cuda.synchronize()
        seed = {"reseed4": 1247, "reseed2": 2902}.get(name, 11)
        st = mdist.train_sharded(ctx, d_rows.data_ptr(), nl, row0, n_total, dim, seed, pq_m=pq_m, max_iters=iters,
                                 tol=tol, d_codebooks_ptr=d_cb.data_ptr(), d_assign_ptr=d_asg.data_ptr())
        cb = d_cb.cpu().numpy()
        asg = d_asg.cpu().numpy().view(np.uint32).reshape(pq_m, nl)
        # every rank's codebooks to rank 0
        allcb = [None] * world
        dist.all_gather_object(allcb, mdist.codebook_digest(cb))
        allasg = [None] * world
        dist.all_gather_object(allasg, asg)
        if rank == 0:
            # the one-GPU run, on a context without a communicator
            ctx1 = Context(local)
            ctx1.check(ctx1.lib.mvr_ctx_set_serial_draws(ctx1.handle, 1 if serial else 0))
            d_full = torch.from_numpy(x).cuda()
            d_cb1 = torch.empty(cb_n, dtype=torch.float32, device="cuda")
            d_asg1 = torch.empty(pq_m * n_total, dtype=torch.int32, device="cuda")
            torch.cuda.synchronize()
            st1 = PqTrainStats()
            ctx1.check(ctx1.lib.mvr_pq_train_sharded_device(
                ctx1.handle, C.c_void_p(d_full.data_ptr()), n_total, 0, n_total, dim, seed, 1, pq_m, iters,
                C.c_float(tol), C.c_void_p(d_cb1.data_ptr()), C.c_void_p(d_asg1.data_ptr()), C.byref(st1)))
            cb1 = d_cb1.cpu().numpy()
            asg1 = d_asg1.cpu().numpy().view(np.uint32).reshape(pq_m, n_total)
            ctx1.close()
            if len(set(allcb)) != 1:
                failures.append(f"{name}: codebooks differ across ranks")
            if mdist.codebook_digest(cb1) != allcb[0]:
                failures.append(f"{name}: sharded codebooks != one-GPU codebooks")
            if not np.array_equal(np.concatenate(allasg, axis=1), asg1):
                failures.append(f"{name}: sharded assignments != one-GPU assignments")
            if name.startswith("reseed") and not (st["reseeds"] > 0 and st1.reseeds == st["reseeds"]):
                failures.append(f"{name}: expected the same non-zero reseed count")
            print(f"[dist] {name} world={world} iters={iters} tol={tol} serial={serial} "
                  f"fallbacks={st['seed_fallbacks']} reseeds={st['reseeds']} iters_run={st['iters_max']} "
                  f"one_gpu_fallbacks={st1.seed_fallbacks} one_gpu_reseeds={st1.reseeds} "
                  f"sharded_ms={st['total_ms']:.1f} one_gpu_ms={st1.total_ms:.1f}", flush=True)
        dist.barrier()
    ctx.check(ctx.lib.mvr_ctx_set_serial_draws(ctx.handle, 0))
    # clusterFlat split over the ranks by token: the full outputs on every
    # rank, equal to the one-GPU call (and, for the small case, the oracle)
    tac_cases = [(20_000, 64, 4096, 10, 8, False), (25_000, 24, 5000, 10, 3, True), (3_000, 8, 600, 2, 1, False)]
    for n, dim, kappa, theta, threads, with_oracle in tac_cases:
        c = synth.make_corpus(n, dim, n_anchors=50 if n == 3_000 else 19221, seed=n + dim)
        kw = dict(mu=8, tau=16, epsilon=2) if n == 3_000 else {}
        p = tac.ClusteringParams(kappa, 42, theta=theta, n_threads=threads, **kw)
        got = tac.cluster_flat(c.token_ids, c.vectors, dim, p, ctx=ctx, sharded=True)
        st = tac.last_stats(ctx)
        digest = hashlib.sha256(got.centroids.tobytes() + got.assignments.tobytes() +
                                got.kappa_per_token.tobytes() + np.float32(got.wcss_total).tobytes()).hexdigest()
        alld = [None] * world
        dist.all_gather_object(alld, (digest, st["problems"]))
        if rank == 0:
            ctx1 = Context(local)
            one = tac.cluster_flat(c.token_ids, c.vectors, dim, p, ctx=ctx1)
            st1 = tac.last_stats(ctx1)
            ctx1.close()
            d1 = hashlib.sha256(one.centroids.tobytes() + one.assignments.tobytes() +
                                one.kappa_per_token.tobytes() + np.float32(one.wcss_total).tobytes()).hexdigest()
            if len({d for d, _ in alld}) != 1:
                failures.append(f"tac {n}x{dim}: outputs differ across ranks")
            if d1 != alld[0][0]:
                failures.append(f"tac {n}x{dim}: sharded clusterFlat != one-GPU clusterFlat")
            if sum(q for _, q in alld) != st1["problems"]:
                failures.append(f"tac {n}x{dim}: problems split {[q for _, q in alld]} != {st1['problems']}")
            if with_oracle:
                from oracle import oracle as orc

                want = orc.tac_cluster_flat(c.token_ids, c.vectors, dim, kappa, 42, mu=p.mu, tau=p.tau,
                                            eps=p.epsilon, theta=p.theta, n_threads=threads)
                if not (np.array_equal(got.assignments, want.assignments) and
                        got.centroids.tobytes() == want.centroids.tobytes()):
                    failures.append(f"tac {n}x{dim}: sharded clusterFlat != oracle")
            print(f"[dist] tac {n}x{dim} kappa={kappa} world={world} problems={[q for _, q in alld]} "
                  f"sharded_ms={st['total_ms']:.1f} one_gpu_ms={st1['total_ms']:.1f}", flush=True)
        dist.barrier()
    ok = [not failures]
    dist.broadcast_object_list(ok, src=0)
    if rank == 0:
        for f in failures:
            print("[dist] FAIL", f, flush=True)
    ctx.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0 if ok[0] else 1


if __name__ == "__main__":
    sys.exit(main())
