"""Host logic of the row-sharded path on CPU: shard bounds, the NCCL id
hand-off over a torch group, and the Lloyd exchange protocol (running f32
sums carried rank to rank, counts summed) run by two gloo ranks against the
single serial loop of the reference; the token split and the exact merge of
the sharded clusterFlat."""
import os
import socket

import numpy as np
import pytest

from ir_multivector_retrieval_b200 import dist as mdist


def test_shard_rows_cover_contiguously():
    for n in (1, 2, 7, 256, 1_521_797):
        for world in (1, 2, 3, 4, 8):
            if n < world:
                continue
            nxt, sizes = 0, []
            for r in range(world):
                row0, nl = mdist.shard_rows(n, world, r)
                assert row0 == nxt and nl >= 1
                nxt += nl
                sizes.append(nl)
            assert nxt == n and max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        mdist.shard_rows(10, 2, 2)


def test_relay_order_equals_serial_sum():
    rng = np.random.default_rng(0)
    v = (rng.standard_normal(10_001) * 10.0 ** rng.integers(-6, 6, size=10_001)).astype(np.float32)
    serial = np.float32(0)
    for x in v:
        serial = np.float32(serial + x)
    for world in (1, 2, 3, 8):
        shards = [v[mdist.shard_rows(v.size, world, r)[0]:][: mdist.shard_rows(v.size, world, r)[1]]
                  for r in range(world)]
        assert mdist.relay_order(shards).tobytes() == serial.tobytes()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, ret):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        uid = mdist.exchange_unique_id(lambda: bytes(range(128)))
        ok_uid = uid == bytes(range(128))
        # one Lloyd exchange for K clusters of S coordinates over sharded rows
        rng = np.random.default_rng(42)
        n, K, S = 5_003, 16, 4
        rows = (rng.standard_normal((n, S)) * 100).astype(np.float32)
        asg = rng.integers(0, K, size=n)
        row0, nl = mdist.shard_rows(n, world, rank)
        # the engine's order: counts summed by all ranks, then the relay
        counts = torch.from_numpy(np.bincount(asg[row0:row0 + nl], minlength=K).astype(np.int64))
        dist.all_reduce(counts)
        sums = torch.zeros((K, S), dtype=torch.float32)
        if rank > 0:
            dist.recv(sums, src=rank - 1)
        acc = sums.numpy().copy()
        for i in range(row0, row0 + nl):
            acc[asg[i]] = (acc[asg[i]] + rows[i]).astype(np.float32)
        out = torch.from_numpy(acc)
        if rank + 1 < world:
            dist.send(out, dst=rank + 1)
        dist.broadcast(out, src=world - 1)
        if rank == 0:
            want = np.zeros((K, S), np.float32)
            for i in range(n):
                want[asg[i]] = (want[asg[i]] + rows[i]).astype(np.float32)
            ret.put((ok_uid, out.numpy().tobytes() == want.tobytes(),
                     np.array_equal(counts.numpy(), np.bincount(asg, minlength=K))))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_exchange_protocol():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    for p in procs:
        if p.exitcode is None:
            p.kill()
    assert all(p.exitcode == 0 for p in procs)
    ok_uid, ok_sums, ok_counts = q.get(timeout=10)
    assert ok_uid and ok_sums and ok_counts


def _lpt_model(freqs, kappa, world):
    """Longest-processing-time split restated in Python."""
    def work(n, k):
        if n == 0 or k == 0:
            return 0
        return n * (k + 1) if k < n else n

    owner = [0] * len(freqs)
    order = sorted((j for j in range(len(freqs)) if work(int(freqs[j]), int(kappa[j])) > 0),
                   key=lambda j: (-work(int(freqs[j]), int(kappa[j])), j))
    load = [0] * world
    for j in order:
        r = min(range(world), key=lambda q: (load[q], q))
        owner[j] = r
        load[r] += work(int(freqs[j]), int(kappa[j]))
    return np.array(owner, np.uint32), load


def test_partition_tokens_is_lpt():
    from ir_multivector_retrieval_b200 import tac

    rng = np.random.default_rng(3)
    for world in (1, 2, 3, 8):
        freqs = rng.zipf(1.3, size=500).astype(np.uint32)
        freqs[rng.integers(0, 500, size=40)] = 0
        kappa = np.minimum(freqs, rng.integers(0, 40, size=500)).astype(np.uint32)
        kappa[rng.integers(0, 500, size=10)] = 0
        got = tac.partition_tokens(freqs, kappa, world)
        want, load = _lpt_model(freqs, kappa, world)
        assert np.array_equal(got, want)
        assert int(got.max()) < world
        # LPT bound: no rank exceeds the mean load by more than the largest item
        biggest = max((int(f) * (int(k) + 1) if k < f else int(f)) for f, k in zip(freqs, kappa) if f and k)
        assert max(load) <= sum(load) / world + biggest
    assert tac.partition_tokens(np.zeros(0, np.uint32), np.zeros(0, np.uint32), 4).size == 0
    with pytest.raises(Exception):
        tac.partition_tokens([1, 2], [1, 1], 0)


def _tac_worker(rank, world, port, ret):
    """The sharded clusterFlat protocol on CPU: spreads and budgets on every
    rank, the per-token k-means of the owned tokens only (oracle restatement),
    outputs zero elsewhere, then one u32-sum all-reduce of the bit patterns."""
    import datetime

    import torch
    import torch.distributed as dist

    from ir_multivector_retrieval_b200 import synth, tac
    from oracle import oracle as orc

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        c = synth.make_corpus(4_000, 8, n_anchors=60, seed=11)
        dim, kappa_total, seed, kw = 8, 700, 5, dict(mu=8, tau=16, eps=2, theta=4)
        ids, vec = c.token_ids, c.vectors
        freqs, spreads = orc.tac_spreads(ids, vec, dim)
        kap = orc.tac_allocate_budgets(freqs, spreads, kappa_total, **kw)
        goffc = np.concatenate([[0], np.cumsum(kap.astype(np.int64))])
        owner = tac.partition_tokens(freqs, kap, world)
        cent = np.zeros(kappa_total * dim, np.float32)
        asg = np.zeros(ids.size, np.uint32)
        for j in np.flatnonzero((freqs > 0) & (kap > 0) & (owner == rank)):
            rows = np.flatnonzero(ids == j)
            r = orc.kmeans_fit(vec[rows], dim, int(kap[j]), seed ^ int(j))
            cent[goffc[j] * dim:(goffc[j] + kap[j]) * dim] = r.centroids
            asg[rows] = goffc[j] + r.assignments
        merged = torch.from_numpy(np.concatenate([cent.view(np.int32), asg.view(np.int32)]))
        dist.all_reduce(merged)  # int32 sum == u32 sum of bit patterns here (no carries)
        m = merged.numpy()
        if rank == 0:
            want = orc.tac_cluster_flat(ids, vec, dim, kappa_total, seed, **kw)
            got_c = m[: cent.size].view(np.float32)
            got_a = m[cent.size:].view(np.uint32)
            ret.put((got_c.tobytes() == want.centroids.tobytes(), np.array_equal(got_a, want.assignments),
                     len(set(owner[(freqs > 0) & (kap > 0)].tolist()))))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_cluster_flat_merge():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tac_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    for p in procs:
        if p.exitcode is None:
            p.kill()
    assert all(p.exitcode == 0 for p in procs)
    ok_c, ok_a, n_owners = q.get(timeout=10)
    assert ok_c and ok_a and n_owners == 2
