#!/usr/bin/env python3
"""Benchmark of the B200 PQ build path.

Workload (one "step"): ``pq.train`` over 1,521,797 x 64 f32 unit residuals,
M = 16 subspaces x 4 dims, 256 centroids each, k-means++ seeding plus 20
Lloyd iterations (tol = -inf), then ``pq.encode`` of all rows. Inputs are
seeded synthetic vectors (``synth.make_corpus``: normalize(anchor +
0.35 N(0, I)), anchors Zipf(1.1) over 19,221 token ids); the PQ input is each
vector's unit residual from its token anchor. The 389 MB input is larger
than L2 (126 MB), so no explicit L2 flush is needed between steps.

Metric: ``pq.train s/Lloyd-iter`` = device time of one full pq.train call
(seeding included) / 20; lower is better. ``e2e`` is the same metric through
the host-pointer C ABI (``mvr_pq_train``) with the rows copied from pinned
host memory every step. Encode throughput is reported beside it.

``--impl reference`` times the CPU restatement of the reference
(oracle/, multithreaded like the reference's work-stealing ``pq.train``) on
this host's cores: one whole pq.train (seeding + 20 Lloyd iterations, the GPU
value's basis) over a bounded row sample, scaled linearly to all rows. The
one-GPU line also checks the benched codebooks and codes against the
restatement run on all rows (``pq_bit_exact_vs_cpu``, after timing) and ends
with a short ``codebook_sha256`` line for comparing runs at different N.

``tac`` in the JSON line: ``tac.clusterFlat`` through the host-pointer C ABI
on the same 1,521,797-row corpus with kappa = 32,768 and the paper-strict
thresholds (mu 128, tau 256, eps 4, theta 39), with its device phases; and on
configs[0]'s 117,645-row corpus (kappa 12,288, theta 10) beside the CPU
restatement of the reference timed on one host core.

Multi-GPU (``--gpus N`` under torchrun, configs[2]): the same 1,521,797 rows
are split into N contiguous shards, one per GPU, and ``pq.train`` runs
sharded (``mvr_pq_train_sharded_device``): with 16 subspaces and N <= 16 each
GPU trains 16/N whole subspaces over all rows after one NCCL column exchange,
then the codebooks are gathered; codebooks are byte-identical to the one-GPU
run for any N (``codebook_sha256`` in the line lets runs at different N be
compared). ``pq.encode`` runs on each shard. Strong scaling: the total work
is fixed; times are the max over ranks.
"""
from __future__ import annotations

import argparse
import hashlib
import ctypes as C
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_ROWS = 1_521_797
DIM = 64
PQ_M = 16
K = 256
ITERS = 20
SEED = 42 + 0xA1B2C3D4  # storage.build passes params.seed +% 0xa1b2c3d4 to pq.train
METRIC = "pq.train s/Lloyd-iter"
UNIT = "s/iter"
WORKLOAD = "configs[1]: synthetic 1,521,797 x 64 f32, PQ M=16x4, 256 centroids, k-means++ + 20 Lloyd iters, + pq.encode"


def config_dict(world: int, rows_per_gpu: int | None = None) -> dict:
    """The workload description both arms print (same keys, same values)."""
    return {"workload": WORKLOAD, "rows": N_ROWS, "rows_per_gpu": rows_per_gpu or N_ROWS, "dim": DIM,
            "pq_m": PQ_M, "centroids": K, "lloyd_iters": ITERS,
            "parallelism": (("subspace-sharded" if PQ_M >= world else "row-sharded")
                            + f" over {world} GPUs (NCCL)") if world > 1 else "1gpu",
            "l2": "inputs (389 MB) > L2, no flush"}


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def make_corpus(n: int | None = None):
    from ir_multivector_retrieval_b200 import synth

    return synth.make_corpus(N_ROWS if n is None else n, DIM, seed=42)


def make_input(n: int | None = None) -> np.ndarray:
    from ir_multivector_retrieval_b200 import synth

    return synth.anchor_residuals(make_corpus(n))


def _hbm_peak() -> float:
    try:
        return float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["hbm_gbs"])
    except Exception:
        return 6650.0  # fallback copy bandwidth when the measured file is absent


HBM_PEAK = _hbm_peak()
TAC_KAPPA = 32_768
TAC_SMALL = (117_645, 12_288, 10)  # configs[0] rows, kappa (10,240 leaves no room for the tail), theta


def measure_tac(corpus, steps: int, cpu: bool, ctx=None, world: int = 1, reduce=None) -> dict:
    """clusterFlat through the host-pointer C ABI (e2e wall time with the
    inputs in page-locked host memory, device phases from mvr_tac_last_stats)
    on the full corpus and on configs[0].
    With world > 1 every rank calls the token-sharded entry point on the
    same inputs (a collective); times are the max over ranks (``reduce``)."""
    from ir_multivector_retrieval_b200 import synth, tac

    sharded = world > 1
    red = reduce or (lambda v: v)
    out = {"workload": (f"tac.clusterFlat {corpus.n:,} x {DIM}, kappa {TAC_KAPPA:,}, paper-strict "
                        "(mu 128, tau 256, eps 4, theta 39), 25 iters, tol 1e-4"),
           "parallelism": f"token-sharded over {world} GPUs (NCCL)" if sharded else "1gpu"}
    p = tac.ClusteringParams(kappa_total=TAC_KAPPA, seed=42)

    def call(ids, vec, prm):
        return tac.cluster_flat(ids, vec, DIM, prm, ctx=ctx, sharded=sharded)

    def pinned(a):  # inputs in page-locked host memory, like the pq.train e2e leg
        import torch

        return torch.from_numpy(np.ascontiguousarray(a)).pin_memory().numpy()

    ids_h, vec_h = pinned(corpus.token_ids), pinned(corpus.vectors)
    call(ids_h, vec_h, p)  # warm-up: grows buffers
    walls, stats, digests = [], [], set()
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        r = call(ids_h, vec_h, p)
        walls.append(time.perf_counter() - t0)
        stats.append(tac.last_stats(ctx))
        digests.add(hashlib.sha256(r.centroids.tobytes() + r.assignments.tobytes()).hexdigest())
    mid = sorted(range(len(walls)), key=walls.__getitem__)[len(walls) // 2]
    st = stats[mid]
    out.update({"e2e_ms": red(walls[mid] * 1e3),
                "device_ms": red(st["spread_ms"] + st["seed_ms"] + st["lloyd_ms"]),
                "phases_ms": {k: st[k] for k in ("host_ms", "h2d_ms", "spread_ms", "seed_ms", "lloyd_ms",
                                                 "d2h_ms")},
                "tokens": st["problems"], "iters_max": st["iters_max"], "gpu_launches": st["launches"],
                "filter": {"rows_rechecked": st["filter_rows_rechecked"], "violations": st["filter_violations"],
                           "rows_full_scan": st["filter_rows_full_scan"]},
                "wcss_total": r.wcss_total, "outputs_sha256": sorted(digests)[0],
                "repeatable": len(digests) == 1})
    out["_centroids"] = r.centroids
    if sharded:
        out["phases_ms_note"] = "phases and tokens of rank 0; e2e_ms and device_ms are the max over ranks"
    n0, k0, th0 = TAC_SMALL
    c0 = synth.make_corpus(n0, DIM, seed=42)
    p0 = tac.ClusteringParams(kappa_total=k0, seed=42, theta=th0)
    ids0, vec0 = pinned(c0.token_ids), pinned(c0.vectors)
    call(ids0, vec0, p0)
    w0 = []
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        r0 = call(ids0, vec0, p0)
        w0.append(time.perf_counter() - t0)
    small = {"workload": f"configs[0]: {n0:,} x {DIM}, kappa {k0:,}, theta {th0}",
             "e2e_ms": red(statistics.median(w0) * 1e3)}
    if cpu:
        from oracle import oracle

        oracle.build()
        t0 = time.perf_counter()
        rc = oracle.tac_cluster_flat(c0.token_ids, c0.vectors, DIM, k0, 42, theta=th0)
        small["cpu_baseline"] = {"value_ms": (time.perf_counter() - t0) * 1e3, "cores": 1, "kind": "port",
                                 "sample": "the whole configs[0] clusterFlat, single-threaded C restatement"}
        small["bit_exact_vs_cpu"] = bool(np.array_equal(rc.assignments, r0.assignments)
                                         and rc.centroids.tobytes() == r0.centroids.tobytes())
    out["small"] = small
    return out


def measure_hnsw(centroids, steps: int, cpu: bool, ctx=None) -> dict:
    """hnsw.build over the clusterFlat centroids as the storage layer runs it
    (storage.zig:404-424): the centroids normalised (vec.normalizeRowsInPlace,
    on the GPU), then the chunked deferred-commit build (the reference's
    10-thread path; the graph is the same for every thread count >= 2) with
    M 32, efConstruction 1500 and seed 42 +% 0xdeadbeef. e2e_ms: the host
    entry point (host centroids in, host CSR out); device_ms: the build's
    CUDA-event time. One GPU: the build does not shard."""
    from ir_multivector_retrieval_b200 import hnsw

    seed = (42 + hnsw.STORAGE_SEED_OFFSET) & (2**64 - 1)
    x = hnsw.normalize_rows(centroids, DIM, ctx=ctx)
    kappa = x.size // DIM
    hnsw.build(x[: DIM * 4096], DIM, seed, ctx=ctx)  # warm-up
    walls, devs, digests, g = [], [], set(), None
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        g = hnsw.build(x, DIM, seed, ctx=ctx)
        walls.append(time.perf_counter() - t0)
        devs.append(g.device_ms)
        digests.add(hashlib.sha256(b"".join(o.tobytes() + b.tobytes() for o, b in
                                            zip(g.layer_offsets, g.layer_neighbours))).hexdigest())
    out = {"workload": f"hnsw.build over the {kappa:,} clusterFlat centroids (dim {DIM}), M 32, efConstruction "
                       "1500, chunked deferred-commit path",
           "e2e_ms": statistics.median(walls) * 1e3, "device_ms": statistics.median(devs),
           "gpu_launches": g.kernel_launches, "max_level": g.max_level,
           "edges_per_layer": [int(b.size) for b in g.layer_neighbours],
           "graph_sha256": sorted(digests)[0], "repeatable": len(digests) == 1,
           "reference_published": {"value_s": 6.7, "note": "README: hnsw.build (parallel, 10 threads) on the "
                                                         "full Jira corpus, Apple M-series; other hardware"}}
    if cpu:
        from oracle import oracle

        oracle.build()
        cores = os.cpu_count() or 1
        t0 = time.perf_counter()
        o = oracle.hnsw_build(x, DIM, seed, n_threads=2, workers=cores)
        out["cpu_baseline"] = {"value_ms": (time.perf_counter() - t0) * 1e3, "cores": cores, "kind": "port",
                               "sample": "the whole build, the C restatement planning each chunk on every host "
                                         "core (like the reference's worker threads)"}
        out["bit_exact_vs_cpu"] = bool(o.entry_point == g.entry_point and all(
            np.array_equal(a, b) for a, b in zip(o.layer_offsets + o.layer_neighbours,
                                                 g.layer_offsets + g.layer_neighbours)))
    return out


# ---------------------------------------------------------------- clocks


class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons while running."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        # nvidia-smi needs a moment before its first sample: the timed region
        # starts only once sampling runs
        t0 = time.perf_counter()
        while not self.lines and time.perf_counter() - t0 < 10.0 and self.proc.poll() is None:
            time.sleep(0.01)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- CPU arm


def cpu_lloyd_seconds_per_iter(x: np.ndarray, threads: int, target_s: float = 15.0) -> dict:
    """One Lloyd iteration of every subspace (oracle, all host threads) on a
    row sample sized for ~target_s of CPU time, scaled linearly to N_ROWS
    (Lloyd cost is linear in the rows)."""
    from oracle import oracle

    oracle.build()
    n_probe = min(len(x), 20_000)
    cb0 = np.ascontiguousarray(
        x[np.linspace(0, len(x) - 1, K).astype(np.int64)].reshape(K, PQ_M, DIM // PQ_M).transpose(1, 0, 2)
    ).reshape(-1)
    t0 = time.perf_counter()
    oracle.pq_lloyd_iters(x[:n_probe], DIM, PQ_M, 1, threads, cb0)
    probe = time.perf_counter() - t0
    n_sample = int(min(len(x), max(n_probe, n_probe * target_s / max(probe, 1e-6))))
    t0 = time.perf_counter()
    oracle.pq_lloyd_iters(x[:n_sample], DIM, PQ_M, 1, threads, cb0)
    dt = time.perf_counter() - t0
    return {"s_per_iter": dt * N_ROWS / n_sample, "rows": n_sample, "wall_s": dt}


def cpu_train_seconds_per_iter(x: np.ndarray, threads: int, target_s: float = 15.0) -> dict:
    """The GPU value's basis on the host: one whole pq.train (k-means++
    seeding + ITERS Lloyd iterations, tol = -inf) by the C restatement on all
    host threads (work-stealing over the subspaces like pq.zig:192-284), on a
    row sample sized for ~target_s, scaled linearly to N_ROWS (seeding and
    Lloyd are both linear in the rows) and divided by ITERS."""
    from oracle import oracle

    oracle.build()
    n_probe = min(len(x), 10_000)
    t0 = time.perf_counter()
    oracle.pq_train(x[:n_probe], DIM, SEED, PQ_M, n_threads=threads, max_iters=ITERS, tol=-math.inf)
    probe = time.perf_counter() - t0
    n_sample = int(min(len(x), max(n_probe, n_probe * target_s / max(probe, 1e-6))))
    t0 = time.perf_counter()
    oracle.pq_train(x[:n_sample], DIM, SEED, PQ_M, n_threads=threads, max_iters=ITERS, tol=-math.inf)
    dt = time.perf_counter() - t0
    return {"s_per_iter": dt * N_ROWS / n_sample / ITERS, "rows": n_sample, "wall_s": dt,
            "sample": (f"one whole pq.train (k-means++ seeding + {ITERS} Lloyd iterations, all {PQ_M} subspaces) "
                       f"over the first {n_sample:,} rows (of {N_ROWS:,}), time scaled linearly to all rows "
                       f"and divided by {ITERS}; C restatement of pq.train on {threads} threads")}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = host_threads()
    x = make_input()
    # each timed step is a bounded sample; the whole run stays within a few minutes
    target = min(args.cpu_target_s, 150.0 / max(1, args.steps))
    for _ in range(args.warmup):
        cpu_train_seconds_per_iter(x, threads, target_s=1.0)
    vals, info = [], None
    for _ in range(args.steps):
        info = cpu_train_seconds_per_iter(x, threads, target_s=target)
        vals.append(info["s_per_iter"])
    v = statistics.median(vals)
    lloyd = cpu_lloyd_seconds_per_iter(x, threads, target_s=min(target, 10.0))
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": v * 1e3, "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(args.gpus, N_ROWS // max(1, args.gpus)),
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": info["sample"]},
        "lloyd_only_s_per_iter": lloyd["s_per_iter"],
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm


def run_b200(args) -> None:
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))

    from ir_multivector_retrieval_b200 import Context
    from ir_multivector_retrieval_b200._lib import PqTrainStats

    corpus = make_corpus(args.rows)
    from ir_multivector_retrieval_b200 import dist as mdist
    from ir_multivector_retrieval_b200 import synth

    x_all = synth.anchor_residuals(corpus)
    n_total = x_all.shape[0]
    row0, n = mdist.shard_rows(n_total, world, rank)
    x = np.ascontiguousarray(x_all[row0:row0 + n])
    x_pin = torch.from_numpy(x).pin_memory()
    dx = x_pin.to(f"cuda:{local}", non_blocking=False)
    dcb = torch.empty(PQ_M * K * (DIM // PQ_M), dtype=torch.float32, device=f"cuda:{local}")
    dcodes = torch.empty((n, PQ_M), dtype=torch.uint8, device=f"cuda:{local}")
    # A dedicated stream: the library and the timing events must share it
    # (torch's default stream has handle 0, which the C ABI reads as "the
    # context's own stream").
    stream = torch.cuda.Stream(device=f"cuda:{local}")
    torch.cuda.set_stream(stream)
    torch.cuda.synchronize()
    ctx = Context(local)
    ctx.set_stream(stream.cuda_stream)
    lib = ctx.lib
    if world > 1:
        mdist.init_comm(ctx)

    def train_dev(st):
        if world > 1:
            ctx.check(lib.mvr_pq_train_sharded_device(ctx.handle, C.c_void_p(dx.data_ptr()), n, row0, n_total, DIM,
                                                      SEED, 1, PQ_M, ITERS, C.c_float(-math.inf),
                                                      C.c_void_p(dcb.data_ptr()), None, C.byref(st)))
        else:
            ctx.check(lib.mvr_pq_train_device(ctx.handle, C.c_void_p(dx.data_ptr()), x.size, DIM, SEED, 1, PQ_M,
                                              ITERS, C.c_float(-math.inf), C.c_void_p(dcb.data_ptr()), C.byref(st)))

    def encode_dev():
        ctx.check(lib.mvr_pq_encode_device(ctx.handle, C.c_void_p(dcb.data_ptr()), DIM, PQ_M,
                                           C.c_void_p(dx.data_ptr()), n, C.c_void_p(dcodes.data_ptr())))

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        train_dev(PqTrainStats())
        encode_dev()
    barrier()

    clocks = ClockSampler(local)
    clocks.start()
    stats = []
    enc_ev = []
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for _ in range(args.steps):
        st = PqTrainStats()
        train_dev(st)
        stats.append(st)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        encode_dev()
        e1.record(stream)
        enc_ev.append((e0, e1))
    t_end.record(stream)
    barrier()
    clk = clocks.stop()
    step_ms = t_start.elapsed_time(t_end) / args.steps
    train_ms = statistics.mean(s.total_ms for s in stats)
    seed_ms = statistics.mean(s.seed_ms for s in stats)
    lloyd_ms = statistics.mean(s.lloyd_ms for s in stats)
    enc_ms = statistics.mean(a.elapsed_time(b) for a, b in enc_ev)
    assign_ms = sum(s.assign_ms for s in stats) / max(1, sum(s.assign_launches for s in stats))
    first_ms = statistics.mean(s.assign_first_ms for s in stats)
    rows_total = sum(s.lloyd_rows_total for s in stats)
    rows_exact = sum(s.lloyd_rows_exact for s in stats)
    launches = int(statistics.mean(s.launches for s in stats)) + 1

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    train_ms = max_over_ranks(train_ms)
    step_ms = max_over_ranks(step_ms)
    enc_ms = max_over_ranks(enc_ms)
    value = train_ms / 1e3 / ITERS

    # ---- e2e: host-pointer C ABI, rows copied from pinned memory each step
    cb_host = np.empty(PQ_M * K * (DIM // PQ_M), dtype=np.float32)
    codes_host = torch.empty((n, PQ_M), dtype=torch.uint8).pin_memory()
    e2e_train, e2e_enc = [], []
    for i in range(max(1, args.e2e_steps) + 1):
        barrier()
        t0 = time.perf_counter()
        if world > 1:  # the shard travels host -> device, codebooks come back
            dx.copy_(x_pin, non_blocking=True)
            train_dev(PqTrainStats())
            torch.cuda.current_stream().synchronize()
            cb_host[:] = dcb.cpu().numpy()
        else:
            ctx.check(lib.mvr_pq_train(ctx.handle, C.c_void_p(x_pin.data_ptr()), x.size, DIM, SEED, 1, PQ_M,
                                       ITERS, C.c_float(-math.inf), C.c_void_p(cb_host.ctypes.data), None))
        t1 = time.perf_counter()
        ctx.check(lib.mvr_pq_encode(ctx.handle, C.c_void_p(cb_host.ctypes.data), DIM, PQ_M,
                                    C.c_void_p(x_pin.data_ptr()), n, C.c_void_p(codes_host.data_ptr())))
        t2 = time.perf_counter()
        if i > 0:  # first call grows the staging buffers
            e2e_train.append(t1 - t0)
            e2e_enc.append(t2 - t1)
    e2e_value = max_over_ranks(statistics.median(e2e_train)) / ITERS
    e2e_enc_s = max_over_ranks(statistics.median(e2e_enc))
    assert np.array_equal(cb_host, dcb.cpu().numpy()), "host and device entry points disagree"
    if world == 1:
        encode_dev()
        torch.cuda.synchronize()
        assert np.array_equal(codes_host.numpy().reshape(-1), dcodes.cpu().numpy().reshape(-1)), \
            "host and device encodes disagree"

    # ---- encode through each assignment kernel (one GPU): the exact f32 scan
    # (the PQ default) and the tensor-core filter, both bit-identical; the
    # line reports both
    enc_paths = {}
    if world == 1:
        for name, on in (("exact_f32_scan", 0), ("tcgen05_filter", 1)):
            ctx.check(lib.mvr_ctx_set_pq_tensor_filter(ctx.handle, on))
            encode_dev()
            ts = []
            for _ in range(5):
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                encode_dev()
                e1.record(stream)
                ts.append((e0, e1))
            torch.cuda.synchronize()
            enc_paths[name] = statistics.median(a.elapsed_time(b) for a, b in ts)
            assert np.array_equal(codes_host.numpy().reshape(-1), dcodes.cpu().numpy().reshape(-1)), \
                f"encode through {name} differs"
        ctx.check(lib.mvr_ctx_set_pq_tensor_filter(ctx.handle, 0))  # the library default for PQ

    # ---- rooflines. (1) the k-means++ weight update: one HBM pass per step
    # over the subspace-major rows of this GPU's subspaces plus the weights
    # read (a weight is written back only where the new centroid lowers it:
    # those few writes are not counted); launches sampled with CUDA events
    # inside the engine (every 8th step). (2) the pruned Lloyd passes (iterations >= 1): exact
    # (row, centroid) distances actually computed x 12 flops (3 per
    # coordinate: subtract, square, add) against the measured f32x2 issue rate.
    # The line's "roofline" is the one with more device time per training.
    # The timed trainings run their subspaces as two groups side by side, so
    # one launch's duration there includes the other group's overlapping
    # kernels: the per-kernel rooflines come from one more training with all
    # subspaces in one group (same kernels, launched one after another).
    ctx.check(lib.mvr_ctx_set_pq_groups(ctx.handle, 1))
    st1 = PqTrainStats()
    train_dev(st1)
    barrier()
    ctx.check(lib.mvr_ctx_set_pq_groups(ctx.handle, 2))
    roof_stats = [st1]
    upd_samples = sum(s.seed_update_samples for s in roof_stats)
    upd_ms = sum(s.seed_update_ms_sampled for s in roof_stats) / max(1, upd_samples)
    m_local = PQ_M // world if (world > 1 and PQ_M >= world) else PQ_M
    n_rows = n_total if (world > 1 and PQ_M >= world) else n
    groups = max(1, max(int(s.groups) for s in roof_stats))  # 1: the roofline training runs one group
    m_launch = m_local / groups  # subspaces one update launch covers
    bytes_per_launch = int(n_rows * m_launch * ((DIM // PQ_M) * 4 + 4))
    achieved = bytes_per_launch / (max(upd_ms, 1e-9) / 1e3) / 1e9
    traffic_json = {}
    tfile = ROOT / "profiles" / "traffic.json"
    if tfile.exists():
        try:
            traffic_json = json.loads(tfile.read_text())
        except Exception:
            traffic_json = {}
    t = traffic_json.get("pq_seed_update_bytes_per_launch")
    traffic = t * (n_rows * m_launch) / (N_ROWS * PQ_M) if t else None
    sm_mhz = clk.get("sm_mhz") or 1965.0
    fp32_nominal = 148 * 128 * sm_mhz * 1e6 / 1e12  # scalar FP32 lanes x clock
    # measured packed f32x2 add/mul issue rate of this GPU (the exact distance
    # kernels' instructions; about twice the scalar rate on B200)
    rate = C.c_double(0.0)
    ctx.check(lib.mvr_measure_f32x2_rate(ctx.handle, C.byref(rate)))
    fp32_peak = rate.value / 1e12
    seed_upd_total_ms = upd_ms * (K - 1) * groups
    roof_hbm = {"kernel": (f"pq_seed_update_w_kernel<4> (k-means++ weight update, {(K - 1) * groups} launches per "
                           f"training of {m_launch:g} subspaces each)"),
                "bound": "hbm", "achieved": achieved, "peak": HBM_PEAK, "unit": "GB/s",
                "frac": achieved / HBM_PEAK, "traffic": traffic,
                "peak_source": "MEASURED_PEAKS.json hbm_gbs (copy bandwidth), of measured",
                "algorithmic_bytes_per_launch": bytes_per_launch, "avg_launch_ms": upd_ms,
                "sampled_launches": upd_samples, "device_ms_per_training": seed_upd_total_ms,
                "measured_on": "one extra training with the subspaces in one group (kernels not overlapped)"}
    list_launches = sum(s.list_launches for s in roof_stats)
    list_ms = sum(s.list_ms for s in roof_stats) / max(1, list_launches)
    list_dist = sum(s.list_distances for s in roof_stats) / max(1, list_launches)
    list_flops = list_dist * 3 * (DIM // PQ_M)
    list_tf = list_flops / (max(list_ms, 1e-9) / 1e3) / 1e12
    tl = traffic_json.get("pq_list_pass_bytes_per_launch")
    roof_fp32 = {"kernel": "pruned Lloyd pass (iterations >= 1: bound check + exact scans of the unsettled rows)",
                 "bound": "fp32", "achieved": list_tf, "peak": fp32_peak, "unit": "TFLOP/s",
                 "frac": list_tf / fp32_peak,
                 "traffic": tl * (n_rows * m_local) / (N_ROWS * PQ_M) if tl else None,
                 "peak_source": ("measured on this GPU in this run: packed f32x2 add/mul lane operations per "
                                 "second (mvr_measure_f32x2_rate; MEASURED_PEAKS.json has no FP32 figure), "
                                 "of measured; one algorithmic flop counted per lane operation"),
                 "scalar_fp32_nominal_tflops": fp32_nominal,
                 "algorithmic_flops_per_launch": list_flops, "distances_per_launch": list_dist,
                 "avg_launch_ms": list_ms, "launches": list_launches,
                 "device_ms_per_training": list_ms * max(1, list_launches) / max(1, len(roof_stats)),
                 "measured_on": "one extra training with the subspaces in one group (kernels not overlapped)"}
    if roof_fp32["device_ms_per_training"] > seed_upd_total_ms:
        roofline, roofline_other = roof_fp32, roof_hbm
    else:
        roofline, roofline_other = roof_hbm, roof_fp32
    enc_flops = n * K * 3 * DIM
    enc_bytes = n * (4 * DIM + PQ_M)
    encode_roofline = {
        "kernel": "pq.encode (default path)", "ms": enc_ms, "algorithmic_flops": enc_flops,
        "fp32_tflops": enc_flops / (enc_ms / 1e3) / 1e12, "fp32_frac": enc_flops / (enc_ms / 1e3) / 1e12 / fp32_peak,
        "hbm_bytes": enc_bytes, "hbm_gbs": enc_bytes / (enc_ms / 1e3) / 1e9,
        "hbm_frac": enc_bytes / (enc_ms / 1e3) / 1e9 / HBM_PEAK, "paths_ms": enc_paths}

    tac_line = None
    if not args.no_tac:  # collective when world > 1: every rank takes part
        tac_line = measure_tac(corpus, 3, cpu=(world == 1 and not args.no_cpu), ctx=ctx, world=world,
                               reduce=max_over_ranks)
    hnsw_line = None
    if tac_line is not None:
        cents = tac_line.pop("_centroids")
        if world == 1 and not args.no_hnsw:  # one GPU: the graph build does not shard
            hnsw_line = measure_hnsw(cents, 3, cpu=not args.no_cpu, ctx=ctx)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": False,
            "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(world, n),
            "codebook_sha256": mdist.codebook_digest(cb_host),
            "pq_train_ms": train_ms, "seed_ms": seed_ms, "lloyd_ms": lloyd_ms,
            "lloyd_only_s_per_iter": lloyd_ms / 1e3 / ITERS,
            "pq_encode_ms": enc_ms, "pq_encode_mvec_s": n_total / (enc_ms / 1e3) / 1e6,
            "seed_fallbacks": int(stats[-1].seed_fallbacks), "reseeds": int(stats[-1].reseeds),
            "gpu_launches": launches,
            "clocks": clk,
            "lloyd_assign": {"first_iteration_ms": first_ms, "mean_ms_per_iteration": assign_ms,
                             "rows_exact_fraction": rows_exact / max(1, rows_total),
                             "note": ("iterations after the first skip (row, subspace) pairs whose exact "
                                      "distance bounds prove the cluster unchanged")},
            "roofline": roofline, "roofline_secondary": roofline_other, "encode_roofline": encode_roofline,
            "pruned_passes": {"launches": list_launches, "avg_ms": list_ms, "distances_per_launch": list_dist},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(x.nbytes),
                    "d2h_bytes_per_step": int(cb_host.nbytes),
                    "encode_mvec_s": n_total / e2e_enc_s / 1e6},
        }
        if tac_line is not None:
            line["tac"] = tac_line
        if hnsw_line is not None:
            line["hnsw"] = hnsw_line
        if world == 1 and not args.no_cpu:
            threads = host_threads()
            cpu = cpu_train_seconds_per_iter(x, threads, target_s=args.cpu_target_s)
            lloyd = cpu_lloyd_seconds_per_iter(x, threads, target_s=min(args.cpu_target_s, 10.0))
            line["cpu_baseline"] = {"value": cpu["s_per_iter"], "unit": UNIT, "cores": threads, "kind": "port",
                                    "sample": cpu["sample"], "lloyd_only_s_per_iter": lloyd["s_per_iter"]}
        if world == 1 and not args.no_parity:
            # the benched codebooks and codes against the C restatement of the
            # reference on the same rows (after timing; all host threads)
            from oracle import oracle

            oracle.build()
            t0 = time.perf_counter()
            want_cb = oracle.pq_train(x, DIM, SEED, PQ_M, n_threads=host_threads(), max_iters=ITERS,
                                      tol=-math.inf)
            want_codes = oracle.pq_encode(want_cb, DIM, PQ_M, x, n_threads=host_threads())
            line["pq_bit_exact_vs_cpu"] = {
                "codebooks": bool(want_cb.tobytes() == cb_host.tobytes()),
                "codes": bool(np.array_equal(want_codes.reshape(-1), codes_host.numpy().reshape(-1))),
                "rows": int(n), "cpu_wall_s": time.perf_counter() - t0,
                "what": (f"oracle pq.train ({ITERS} Lloyd iterations, all rows) + PQ.encode of all rows vs "
                         "the benched codebooks and codes")}
        print(json.dumps(line), flush=True)
        # one short line that survives a tail: digests to compare across GPU counts
        print(f"codebook_sha256 {line['codebook_sha256']} n_gpus {world} value {value:.6g}", flush=True)
    ctx.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------- configs[4]

C4_ROWS, C4_DIM, C4_M, C4_ITERS = 50_000_000, 128, 32, 25
C4_WORKLOAD = ("configs[4]: synthetic 50,000,000 x 128 f32 (made on the GPU), PQ M=32x4, 256 centroids, "
               "k-means++ + 25 Lloyd iters, + pq.encode")


def run_configs4(args) -> None:
    """BASELINE configs[4]'s PQ stage: pq.train (M = 32 x 4, 25 iterations)
    and pq.encode of 50M x 128 rows made on the GPU (synth.device_residuals),
    at N GPUs: subspace-sharded training over NCCL, each rank encoding its
    row shard. Same metric as the default line; a row sample of the codes is
    checked against the oracle given the trained codebooks (one GPU)."""
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900))
    from ir_multivector_retrieval_b200 import Context
    from ir_multivector_retrieval_b200 import dist as mdist
    from ir_multivector_retrieval_b200 import synth
    from ir_multivector_retrieval_b200._lib import PqTrainStats

    n_total = args.rows or C4_ROWS
    row0, n = mdist.shard_rows(n_total, world, rank)
    dev = f"cuda:{local}"
    dx, _ids = synth.device_residuals(n_total, C4_DIM, seed=42, device=dev, row0=row0, n_rows=n)
    del _ids
    S = C4_DIM // C4_M
    dcb = torch.empty(C4_M * K * S, dtype=torch.float32, device=dev)
    dcodes = torch.empty((n, C4_M), dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    torch.cuda.synchronize()
    ctx = Context(local)
    ctx.set_stream(stream.cuda_stream)
    lib = ctx.lib
    if world > 1:
        mdist.init_comm(ctx)
    seed = SEED

    def train_dev(st):
        if world > 1:
            ctx.check(lib.mvr_pq_train_sharded_device(ctx.handle, C.c_void_p(dx.data_ptr()), n, row0, n_total, C4_DIM,
                                                      seed, 1, C4_M, C4_ITERS, C.c_float(-math.inf),
                                                      C.c_void_p(dcb.data_ptr()), None, C.byref(st)))
        else:
            ctx.check(lib.mvr_pq_train_device(ctx.handle, C.c_void_p(dx.data_ptr()), n * C4_DIM, C4_DIM, seed, 1,
                                              C4_M, C4_ITERS, C.c_float(-math.inf), C.c_void_p(dcb.data_ptr()),
                                              C.byref(st)))

    def encode_dev():
        ctx.check(lib.mvr_pq_encode_device(ctx.handle, C.c_void_p(dcb.data_ptr()), C4_DIM, C4_M,
                                           C.c_void_p(dx.data_ptr()), n, C.c_void_p(dcodes.data_ptr())))

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        train_dev(PqTrainStats())
        encode_dev()
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    stats, enc = [], []
    t0e = torch.cuda.Event(enable_timing=True)
    t1e = torch.cuda.Event(enable_timing=True)
    t0e.record(stream)
    for _ in range(args.steps):
        st = PqTrainStats()
        train_dev(st)
        stats.append(st)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        encode_dev()
        e1.record(stream)
        enc.append((e0, e1))
    t1e.record(stream)
    barrier()
    clk = clocks.stop()
    train_ms = max_over_ranks(statistics.mean(s.total_ms for s in stats))
    enc_ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in enc))
    step_ms = max_over_ranks(t0e.elapsed_time(t1e) / args.steps)
    cb_host = dcb.cpu().numpy()
    line = None
    if rank == 0:
        lst = stats[-1]
        line = {
            "metric": METRIC, "value": train_ms / 1e3 / C4_ITERS, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (generated on the GPU)",
            "config": {"workload": C4_WORKLOAD, "rows": n_total, "rows_per_gpu": n, "dim": C4_DIM, "pq_m": C4_M,
                       "centroids": K, "lloyd_iters": C4_ITERS,
                       "parallelism": f"subspace-sharded over {world} GPUs (NCCL)" if world > 1 else "1gpu",
                       "l2": "inputs (25.6 GB) > L2, no flush"},
            "codebook_sha256": mdist.codebook_digest(cb_host),
            "pq_train_ms": train_ms, "seed_ms": lst.seed_ms, "lloyd_ms": lst.lloyd_ms,
            "seed_fallbacks": int(lst.seed_fallbacks),
            "pq_encode_ms": enc_ms, "pq_encode_mvec_s": n_total / (enc_ms / 1e3) / 1e6,
            "pruned_passes": {"launches": lst.list_launches,
                              "avg_ms": lst.list_ms / max(1, lst.list_launches),
                              "distances_per_launch": lst.list_distances / max(1, lst.list_launches)},
            "clocks": clk,
        }
        if world == 1 and not args.no_cpu:
            from oracle import oracle

            oracle.build()
            threads = host_threads()
            xs = dx[: min(n, 4000)].cpu().numpy()
            t0 = time.perf_counter()
            oracle.pq_train(xs, C4_DIM, seed, C4_M, n_threads=threads, max_iters=C4_ITERS, tol=-math.inf)
            dt = time.perf_counter() - t0
            line["cpu_baseline"] = {
                "value": dt * n_total / xs.shape[0] / C4_ITERS, "unit": UNIT, "cores": threads, "kind": "port",
                "sample": (f"one whole pq.train (seeding + {C4_ITERS} Lloyd iterations, {C4_M} subspaces) over "
                           f"the first {xs.shape[0]:,} rows, time scaled linearly to {n_total:,} rows, / {C4_ITERS}")}
        if world == 1 and not args.no_parity:
            from oracle import oracle

            oracle.build()
            idx = torch.from_numpy(np.sort(np.random.default_rng(7).choice(n, 200_000, replace=False))).to(dev)
            xs = dx[idx].cpu().numpy()
            want = oracle.pq_encode(cb_host, C4_DIM, C4_M, xs, n_threads=host_threads())
            got = dcodes[idx].cpu().numpy()
            line["pq_encode_bit_exact_vs_cpu"] = {
                "codes": bool(np.array_equal(want.reshape(-1), got.reshape(-1))), "rows": 200_000,
                "what": "oracle PQ.encode of a seeded 200,000-row sample with the trained codebooks"}
            line["codebooks_finite"] = bool(np.isfinite(cb_host).all())
        print(json.dumps(line), flush=True)
        print(f"codebook_sha256 {line['codebook_sha256']} n_gpus {world} value {line['value']:.6g}", flush=True)
    ctx.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------- configs[3]

C3_ROWS, C3_DIM, C3_M, C3_ITERS, C3_SAMPLE = 600_000_000, 64, 16, 20, 10_000_000
C3_BLOCK = 1 << 24  # rows generated and encoded per block
C3_WORKLOAD = ("configs[3]: synthetic 600,000,000 x 64 f32 (made on the GPU block by block), PQ M=16x4 trained "
               "(k-means++ + 20 Lloyd iters) on the first 10,000,000 rows, pq.encode of all 600M rows")


def run_configs3(args) -> None:
    """BASELINE configs[3]'s PQ stage: pq.train on a seeded 10M-row sample
    (the corpus's first 10M rows; subspace-sharded over NCCL at N > 1) and
    pq.encode of all 600M rows, each rank encoding its contiguous shard
    block by block (rows made on the GPU by synth.device_residuals, the same
    rows whatever N). The anchor of each row's token stands in for its
    coarse (TAC) centroid, as in the default workload. Metric: pq.encode
    Mvec/s over the 600M rows (device time, max over ranks); the training
    figure is beside it. One GPU also streams the rows from page-locked host
    memory through the host-pointer encode (a bounded host buffer, refilled
    once and replayed, reported as e2e)."""
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900))
    from ir_multivector_retrieval_b200 import Context
    from ir_multivector_retrieval_b200 import dist as mdist
    from ir_multivector_retrieval_b200 import synth
    from ir_multivector_retrieval_b200._lib import PqTrainStats

    n_total = args.rows or C3_ROWS
    n_sample = min(C3_SAMPLE, n_total)
    dev = f"cuda:{local}"
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    ctx = Context(local)
    ctx.set_stream(stream.cuda_stream)
    lib = ctx.lib
    if world > 1:
        mdist.init_comm(ctx)
    S = C3_DIM // C3_M
    dcb = torch.empty(C3_M * K * S, dtype=torch.float32, device=dev)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- training on the sample (row shard of the first n_sample rows)
    s0, sn = mdist.shard_rows(n_sample, world, rank)
    xs, _ = synth.device_residuals(n_total, C3_DIM, seed=42, device=dev, row0=s0, n_rows=sn)

    def train(st):
        if world > 1:
            ctx.check(lib.mvr_pq_train_sharded_device(ctx.handle, C.c_void_p(xs.data_ptr()), sn, s0, n_sample, C3_DIM,
                                                      SEED, 1, C3_M, C3_ITERS, C.c_float(-math.inf),
                                                      C.c_void_p(dcb.data_ptr()), None, C.byref(st)))
        else:
            ctx.check(lib.mvr_pq_train_device(ctx.handle, C.c_void_p(xs.data_ptr()), sn * C3_DIM, C3_DIM, SEED, 1,
                                              C3_M, C3_ITERS, C.c_float(-math.inf), C.c_void_p(dcb.data_ptr()),
                                              C.byref(st)))

    for _ in range(max(1, args.warmup)):
        train(PqTrainStats())
    barrier()
    tst = PqTrainStats()
    train(tst)
    barrier()
    train_ms = max_over_ranks(tst.total_ms)
    cb_host = dcb.cpu().numpy()
    del xs
    ctx.check(lib.mvr_ctx_trim(ctx.handle))
    torch.cuda.empty_cache()

    # ---- encode this rank's shard, block by block (generation untimed)
    r0, rn = mdist.shard_rows(n_total, world, rank)
    codes = torch.empty((rn, C3_M), dtype=torch.uint8, device=dev)
    enc_ms = 0.0
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    for b0 in range(0, rn, C3_BLOCK):
        bn = min(C3_BLOCK, rn - b0)
        xb, _ = synth.device_residuals(n_total, C3_DIM, seed=42, device=dev, row0=r0 + b0, n_rows=bn)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        ctx.check(lib.mvr_pq_encode_device(ctx.handle, C.c_void_p(dcb.data_ptr()), C3_DIM, C3_M,
                                           C.c_void_p(xb.data_ptr()), bn, C.c_void_p(codes[b0].data_ptr())))
        e1.record(stream)
        e1.synchronize()
        enc_ms += e0.elapsed_time(e1)
        if b0 == 0 and world == 1 and not args.no_parity:
            keep_first = xb[:200_000].cpu().numpy()
        del xb
    barrier()
    clk = clocks.stop()
    enc_ms = max_over_ranks(enc_ms)

    # ---- one GPU: encode streamed from page-locked host memory
    e2e = None
    if world == 1 and not args.no_e2e_stream:
        hb = min(rn, 1 << 25)  # 33.5M rows, 8.6 GB page-locked
        xb, _ = synth.device_residuals(n_total, C3_DIM, seed=42, device=dev, row0=0, n_rows=hb)
        host = torch.empty((hb, C3_DIM), dtype=torch.float32, pin_memory=True)
        host.copy_(xb)
        del xb
        torch.cuda.empty_cache()
        codes_h = torch.empty((hb, C3_M), dtype=torch.uint8, pin_memory=True)
        passes = (n_total + hb - 1) // hb
        t0 = time.perf_counter()
        done = 0
        for _ in range(passes):
            bn = min(hb, n_total - done)
            ctx.check(lib.mvr_pq_encode(ctx.handle, C.c_void_p(cb_host.ctypes.data), C3_DIM, C3_M,
                                        C.c_void_p(host.data_ptr()), bn, C.c_void_p(codes_h.data_ptr())))
            done += bn
        wall = time.perf_counter() - t0
        same = bool(np.array_equal(codes_h[:100_000].numpy(), codes[:100_000].cpu().numpy()))
        e2e = {"value": n_total / wall / 1e6, "unit": "Mvec/s", "h2d_bytes_per_step": int(n_total * C3_DIM * 4),
               "d2h_bytes_per_step": int(n_total * C3_M),
               "note": (f"host-pointer pq.encode of {n_total:,} rows from a {hb:,}-row page-locked host buffer "
                        f"replayed {passes} times (copies overlapped with the encode in chunks); codes equal to the "
                        f"device path: {same}")}
        del host, codes_h
    if rank == 0:
        line = {
            "metric": "pq.encode Mvec/s", "value": n_total / (enc_ms / 1e3) / 1e6, "unit": "Mvec/s",
            "n_gpus": world, "steps": 1, "warmup": args.warmup, "ms_per_step": enc_ms + train_ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (generated on the GPU)",
            "config": {"workload": C3_WORKLOAD, "rows": n_total, "rows_per_gpu": rn, "dim": C3_DIM, "pq_m": C3_M,
                       "centroids": K, "lloyd_iters": C3_ITERS, "train_rows": n_sample,
                       "parallelism": f"row-sharded encode, subspace-sharded training over {world} GPUs (NCCL)"
                       if world > 1 else "1gpu", "l2": "inputs > L2, no flush"},
            "codebook_sha256": mdist.codebook_digest(cb_host),
            "pq_encode_ms": enc_ms, "pq_train_ms": train_ms, "pq_train_s_per_iter": train_ms / 1e3 / C3_ITERS,
            "seed_ms": tst.seed_ms, "lloyd_ms": tst.lloyd_ms, "seed_fallbacks": int(tst.seed_fallbacks),
            "clocks": clk,
        }
        if e2e is not None:
            line["e2e"] = e2e
        if world == 1 and not args.no_cpu:
            from oracle import oracle

            oracle.build()
            xc, _ = synth.device_residuals(n_total, C3_DIM, seed=42, device=dev, row0=0, n_rows=2_000_000)
            xc = xc.cpu().numpy()
            t0 = time.perf_counter()
            oracle.pq_encode(cb_host, C3_DIM, C3_M, xc, n_threads=host_threads())
            dt = time.perf_counter() - t0
            line["cpu_baseline"] = {"value": xc.shape[0] / dt / 1e6, "unit": "Mvec/s", "cores": host_threads(),
                                    "kind": "port", "sample": "PQ.encode of the first 2,000,000 rows by the C "
                                                              "restatement on all host threads"}
        if world == 1 and not args.no_parity:
            from oracle import oracle

            oracle.build()
            want = oracle.pq_encode(cb_host, C3_DIM, C3_M, keep_first, n_threads=host_threads())
            line["pq_encode_bit_exact_vs_cpu"] = {
                "codes": bool(np.array_equal(want.reshape(-1), codes[:200_000].cpu().numpy().reshape(-1))),
                "rows": 200_000, "what": "oracle PQ.encode of the first 200,000 rows with the trained codebooks"}
        print(json.dumps(line), flush=True)
        print(f"codebook_sha256 {line['codebook_sha256']} n_gpus {world} value {line['value']:.6g}", flush=True)
    ctx.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--cpu-target-s", type=float, default=15.0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the full-size check of the benched codebooks and codes against the oracle")
    ap.add_argument("--no-tac", action="store_true", help="skip the clusterFlat measurement")
    ap.add_argument("--no-hnsw", action="store_true", help="skip the hnsw.build measurement")
    ap.add_argument("--tac-only", action="store_true",
                    help="only the clusterFlat measurement (one GPU; for profiling captures)")
    ap.add_argument("--hnsw-only", action="store_true",
                    help="only clusterFlat and hnsw.build over its centroids (one GPU)")
    ap.add_argument("--workload", choices=["configs1", "configs3", "configs4"], default="configs1",
                    help="configs1 (default, the headline line), configs3 (600M x 64: train on 10M rows, encode "
                         "all) or configs4 (50M x 128, M=32, 25 iterations)")
    ap.add_argument("--no-e2e-stream", action="store_true",
                    help="configs3: skip the host-streamed encode leg")
    ap.add_argument("--rows", type=int, default=None,
                    help="rows of the workload (default 1,521,797; smaller only for profiling captures)")
    args = ap.parse_args()
    if args.tac_only or args.hnsw_only:
        t = measure_tac(make_corpus(args.rows), 1 if args.hnsw_only else args.steps,
                        cpu=not args.no_cpu and args.tac_only)
        cents = t.pop("_centroids")
        out = {"tac": t}
        if args.hnsw_only:
            out["hnsw"] = measure_hnsw(cents, args.steps, cpu=not args.no_cpu)
        print(json.dumps(out), flush=True)
        return 0
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "configs4":
        run_configs4(args)
    elif args.workload == "configs3":
        run_configs3(args)
    else:
        run_b200(args)
    return 0


if __name__ == "__main__":
    sys.exit(main())
