#!/usr/bin/env python
"""Benchmark: exact k-means assign throughput and train time on B200.

Workload: 200,000 x 768 f32 unit rows from a 4,096-component
Gaussian mixture (means N(0, I), noise sigma 0.5, Zipf(1.1) weights), k = 1024
centroids, squared-L2 metric, exact FP32 labels. The centroids are the result
of training on these rows with the engine's device loop (seed 0, the reference
schedule), so the assign sees trained geometry. One step = one full assign
pass over the 200,000 rows (``Device::top1`` preceded by the centroid norms,
as ``core::assign_on`` does). With N GPUs the rows are sharded over the ranks
(strong scaling: the total work is fixed), centroids replicated, and each
step ends with the labels and scores all-gathered to every rank (one kernel
pushing each rank's share into every peer's copy of the group's exchange
region over NVLink).

Reported:
- value: rows assigned per second (Grows/s), device-resident inputs, CUDA
  events on the engine's stream, max over ranks;
- e2e: the same through ``eb_assign`` (Assigner::assign), each rank on its
  shard, pinned host rows/centroids in and labels/scores out, copies inside
  the timed region;
- roofline of the dominant kernel (the tcgen05 screen) against the measured
  dense peak; parity of the timed run's labels and scores against the oracle
  (bit for bit, all rows); cpu_baseline (the C++ oracle port of the reference
  CPU kernel on this host's cores); train_s (C2 training) with its oracle
  baseline and objective delta, and at N > 1 the north-star training mode
  (partial sums exchanged once per step) beside the parity mode; the update
  ops' HBM throughput; internal scores; clocks.

``--impl reference`` times the reference CPU path (the oracle port; the Rust
reference cannot be built here) on the same workload and the same trained
centroids, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "assign Grows/s & k-means train s (200k×768 f32, k=1024) at 1/2/4/8 B200"
FALLBACK_PEAK_TFLOPS = 1590.0
# DRAM bytes (read + write) per row of one screen launch, from the ncu capture
# of k_screen on 65,536 C2 rows in profiles/k_screen_c2_65536rows.md (104.9 MB
# read + 7.8 MB written): the fixed-point rows (1,536 B/row) plus the centroid
# digits and the candidate lists.
SCREEN_DRAM_BYTES_PER_ROW = (104.9e6 + 7.8e6) / 65_536
TRAFFIC_SOURCE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one 65,536-row screen "
                  "launch (profiles/k_screen_c2_65536rows.md), scaled by rows")


def gen_rows(n, d, seed_rows, components=4096, sigma=0.5, zipf=1.1, seed_means=0):
    """Config-2 rows: Zipf-weighted Gaussian mixture, unit-normalised."""
    means = np.random.default_rng(seed_means).standard_normal((components, d), dtype=np.float32)
    w = 1.0 / np.arange(1, components + 1, dtype=np.float64) ** zipf
    rng = np.random.default_rng(1000 + seed_rows)
    comp = rng.choice(components, n, p=w / w.sum())
    x = means[comp]
    x += np.float32(sigma) * rng.standard_normal((n, d), dtype=np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    return np.ascontiguousarray(x, dtype=np.float32)


def hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        if "hbm_gbs" in j:
            return float(j["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (copy)"
    return 6650.0, "fallback 6.65 TB/s (no MEASURED_PEAKS.json)"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return j.get("bf16_tflops", FALLBACK_PEAK_TFLOPS), "MEASURED_PEAKS.json bf16_tflops (burst)"
    return FALLBACK_PEAK_TFLOPS, "fallback 1.59 PFLOP/s (no MEASURED_PEAKS.json)"


class Clocks:
    """nvidia-smi samples during the timed region."""

    Q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 6:
                self.rows.append(parts)

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4)
                          if r[2 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.rows)}


def dist_setup(gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != gpus:
        raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={world}: launch N>1 under torchrun")
    return world, rank, local


def shard(n, world, rank):
    """Rank `rank`'s rows [lo, hi) of n rows split into `world` contiguous
    shards of s = ceil(n / world) rows (the last ones shorter or empty)."""
    s = (n + world - 1) // world
    lo = min(rank * s, n)
    return lo, min(lo + s, n), s


def c2_config(args, world):
    """The workload both arms report (identical keys and values)."""
    return {"workload": f"C2 final assign: {args.n:,} x {args.d} f32 rows vs k={args.k} "
                        "centroids trained on C2 (seed 0, reference schedule), squared L2, "
                        "exact FP32 labels+scores; then k-means train s on C2",
            "rows": args.n, "d": args.d, "k": args.k, "metric": "L2",
            "centroids": "trained on the C2 rows, seed 0, nepochs 5 (bit-equal on both arms)",
            "l2_flush": "inputs larger than L2 (rows are 614 MB)",
            "parallelism": f"rows sharded over {world} GPU(s), centroids replicated; "
                           "labels and scores all-gathered to every rank (peer memory "
                           "over NVLink)"}


def cpu_assign(x, d, cent, budget_s):
    """The oracle port of the reference CPU kernel (cpu-fused order) on all
    host threads, over as many leading rows as fit in budget_s (all of C2 on
    the GPU box's host). Returns (timing dict, labels, scores)."""
    import oracle

    threads = os.cpu_count() or 1
    n = x.shape[0]
    labels = np.empty(n, np.uint32)
    scores = np.empty(n, np.float32)
    done, chunk, t0 = 0, 16384, time.perf_counter()
    while done < n and time.perf_counter() - t0 < budget_s:
        e = min(done + chunk, n)
        labels[done:e], scores[done:e] = oracle.top1(x[done:e].ravel(), d, cent.ravel(),
                                                     oracle.L2, threads=threads)
        done = e
    dt = time.perf_counter() - t0
    return ({"value": done / dt / 1e9, "unit": "Grows/s", "cores": threads, "kind": "port",
             "sample": f"first {done:,} of {n:,} rows (exact FP32 L2 top-1, k={cent.shape[0]}), "
                       f"{dt:.2f} s, oracle/oracle.cpp AVX2+FMA, {threads} threads"},
            labels[:done], scores[:done])


def cpu_train(x, d, k):
    """The reference training loop (oracle port, all host threads) on C2,
    timed like the reference's train_profile (rows already in memory)."""
    import oracle

    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    res = oracle.train(x, d, k, seed=0, threads=threads)
    return time.perf_counter() - t0, threads, res


def run_reference(args):
    """--impl reference: the reference CPU path (the oracle port; the Rust
    reference cannot be built here) on the host cores, rank 0 only: trains on
    C2 (timed, the train_s baseline), then assigns the C2 rows against those
    centroids, the same trained centroids the GPU arm assigns against."""
    world, rank, _ = dist_setup(args.gpus) if args.gpus > 1 else (1, 0, 0)
    if rank != 0:
        return
    import oracle

    n, d, k = args.n, args.d, args.k
    xtrain = gen_rows(200_000, d, 0)
    train_s, threads, tr = cpu_train(xtrain, d, k)
    cent = tr["centroids"].reshape(k, d)
    x = xtrain[:n] if n <= xtrain.shape[0] else gen_rows(n, d, 0)
    sample = min(args.ref_rows or n, n)
    for _ in range(args.warmup):
        oracle.top1(x[:sample].ravel(), d, cent.ravel(), oracle.L2, threads=threads)
    times = []
    for s in range(args.steps):
        lo = (s * sample) % (n - sample + 1)
        t0 = time.perf_counter()
        oracle.top1(x[lo:lo + sample].ravel(), d, cent.ravel(), oracle.L2, threads=threads)
        times.append(time.perf_counter() - t0)
    t = sum(times)
    v = sample * args.steps / t / 1e9
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "Grows/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * t / args.steps * n / sample, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": c2_config(args, world),
        "cpu_baseline": {"value": v, "unit": "Grows/s", "cores": threads, "kind": "port",
                         "sample": f"{sample:,} rows x {args.steps} steps against the trained "
                                   "centroids (oracle/oracle.cpp, the reference cpu-fused float "
                                   "order; the Rust reference is not buildable here: no cargo)"},
        "e2e": {"value": v, "unit": "Grows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "train_s": {"value": train_s, "unit": "s", "cores": threads, "kind": "port",
                    "steps": 65, "final_obj": tr["obj"][-1]},
    }), flush=True)


def _max_over_ranks(dist, vals):
    """Element-wise max of a list of floats over the ranks (float64)."""
    import torch

    if dist is None:
        return vals
    t = torch.tensor(vals, device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def run_ours(args):
    import torch

    world, rank, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    import emeans_b200 as eb

    n, d, k = args.n, args.d, args.k
    eng = eb.Engine(local)
    stream = torch.cuda.ExternalStream(eng.stream())
    if world > 1:
        eng.join_torch_group()

    # Centroids: train on the C2 rows (identical on every rank), always the
    # full 200,000 rows so that smaller --n runs see the same geometry.
    xtrain = gen_rows(200_000, d, 0)
    cfg = eb.Config(d=d, k=k, seed=0, spherical=False)
    train_s = train_red = tr = tr_red = None
    if args.load_cent:
        cent = np.load(args.load_cent).astype(np.float32)
    elif not args.no_train:
        # The rows go to the device once, outside the timer (Assigner::bind_data),
        # as the reference's train_profile does; training then reads them in place.
        eng.bind_data(xtrain, d)

        def timed_train():
            eng.train(xtrain, cfg)  # warm-up run
            if dist:
                dist.barrier()
            t0 = time.perf_counter()
            out = eng.train(xtrain, cfg)
            return time.perf_counter() - t0, out

        train_s, tr = timed_train()
        if world > 1:
            # North-star mode: the top-1 and the scatter-add split over the
            # ranks, partial sums exchanged once per step.
            eng.set_group_shard(3)
            train_red, tr_red = timed_train()
            eng.set_group_shard(0)
        train_s, train_red = _max_over_ranks(dist, [train_s, train_red or 0.0])
        cent = tr.centroids
    else:
        cent = xtrain[np.random.default_rng(0).permutation(xtrain.shape[0])[:k]]
    if args.save_cent and rank == 0:
        np.save(args.save_cent, cent)
    x = np.ascontiguousarray(xtrain[:n] if n <= xtrain.shape[0] else gen_rows(n, d, 0))
    lo, hi, s = shard(n, world, rank)

    # ---- device-resident assign: each rank binds its shard of the rows and
    # writes its labels and scores into its share of the group's exchange
    # region (share r = labels then scores of rows r s .. r s + s, each s4
    # words), which one all-gather per step, over NVLink peer memory, gives
    # to every rank.
    m = hi - lo
    xb = eng.bind(x[lo:hi], d)
    cb = eng.upload_f32(cent)
    cn = eng.zeros_f32(k)
    s4 = (s + 3) // 4 * 4
    res = eng.group_exchange(world * 2 * s4)
    xch_mapped, xch_why = eng.group_exchange_info()
    lab = eng.view(res, rank * 2 * s4, s4, eb.U32)
    sco = eng.view(res, rank * 2 * s4 + s4, s4, eb.F32)

    def step(ev=None):
        eng.row_norms(cb, k, d, cn)
        if ev:
            ev[0].record(stream)
        if m:
            eng.top1(xb, d, None, range(0, m), cb, cn, k, eb.L2, lab, sco)
        if ev:
            ev[1].record(stream)
        if world > 1:
            eng.group_allgather(res, 2 * s4)

    # The first call on fresh rows builds their fixed-point copy (kept for later
    # calls on the bound rows, as the reference keeps its per-buffer copy).
    eng.sync()
    t0 = time.perf_counter()
    step()
    eng.sync()
    cold_ms = (time.perf_counter() - t0) * 1e3
    for _ in range(args.warmup):
        step()
    eng.sync()
    if dist:
        dist.barrier()
    launches0 = eng.stats()["kernel_launches"]
    eng.set_kernel_timing(True)
    eng.screen_timing()  # reset
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        start.record(stream)
        for st in range(args.steps):
            step(kev[st])
        end.record(stream)
        end.synchronize()
    eng.sync()
    screen_ms, screen_launches, screen_rows = eng.screen_timing()
    eng.set_kernel_timing(False)
    launches = eng.stats()["kernel_launches"] - launches0
    ms = start.elapsed_time(end)
    top1_ms = statistics.mean(a.elapsed_time(b) for a, b in kev)
    stats = eng.stats()
    rank_ms = [ms / args.steps]
    if dist:
        mine = torch.tensor([ms / args.steps], device="cuda")
        every = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(every, mine)
        rank_ms = [float(v.item()) for v in every]
    ms, top1_ms, screen_ms, cold_ms = _max_over_ranks(dist, [ms, top1_ms, screen_ms, cold_ms])
    if dist:
        dist.barrier()
    # Every rank holds all rows' results.
    allres = res.read().reshape(world, 2 * s4)
    glab = np.ascontiguousarray(allres[:, :s]).ravel()[:n]
    gsco = np.ascontiguousarray(allres[:, s4:s4 + s]).ravel().view(np.float32)[:n]

    # ---- end to end through Assigner::assign (eb_assign): this rank's shard
    # from pinned host memory, labels and scores back into pinned host memory.
    hx = torch.from_numpy(x[lo:hi]).pin_memory()
    hc = torch.from_numpy(np.ascontiguousarray(cent)).pin_memory()
    hl = torch.empty(max(m, 1), dtype=torch.int32).pin_memory()
    hs = torch.empty(max(m, 1), dtype=torch.float32).pin_memory()

    def e2e_step():
        if m:
            eng.assign_ptr(hx.data_ptr(), m, d, hc.data_ptr(), k, eb.L2, hl.data_ptr(),
                           hs.data_ptr())

    for _ in range(max(1, args.warmup)):
        e2e_step()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e2e_s = _max_over_ranks(dist, [time.perf_counter() - t0])[0]
    if dist:
        dist.barrier()
    # The e2e labels must equal the device-resident ones.
    assert np.array_equal(hl.numpy()[:m].view(np.uint32), glab[lo:hi]), "e2e labels differ"

    # ---- the update ops over this rank's shard (HBM-bound): the scatter-add
    # of its rows into their centroids' sums (the reference's float order) and
    # one EMA step, timed by CUDA events.
    sums = eng.zeros_f32(k * d)
    counts = eng.zeros_u32(k)
    pos = eng.upload_f32(cent)
    usage = eng.upload_f32(np.full(k, 1.0 / k, np.float32))

    def upd_step():
        eng.scatter_add(xb, d, None, range(0, m), lab, k, sums, counts)
        eng.ema_update(pos, usage, sums, counts, k, d, 0.1)

    for _ in range(args.warmup):
        upd_step()
    eng.sync()
    u0 = torch.cuda.Event(enable_timing=True)
    u1 = torch.cuda.Event(enable_timing=True)
    u0.record(stream)
    for _ in range(args.steps):
        upd_step()
    u1.record(stream)
    u1.synchronize()
    eng.sync()
    upd_ms = _max_over_ranks(dist, [u0.elapsed_time(u1) / args.steps])[0]
    # Algorithmic bytes: rows and labels read, sums and counts written; the EMA
    # reads positions, sums, counts and masses and writes positions and masses.
    upd_bytes = m * d * 4 + m * 4 + k * d * 4 + k * 4 + 3 * k * d * 4 + 4 * k * 4

    # ---- internal scores of the final labels (metrics::internal_scores):
    # wall time of one call through the host API, after one warm-up call.
    met_ms = mres = None
    if rank == 0:
        eng.internal_scores(x, d, glab, k)
        t0 = time.perf_counter()
        mres = eng.internal_scores(x, d, glab, k)
        met_ms = (time.perf_counter() - t0) * 1e3

    c3 = c4 = c5 = None
    if not args.no_c3:
        c3 = c3_leg(eng, args, world, rank, local, dist)
    if not args.no_c4:
        c4 = c4_leg(eng, args, world, rank, dist)
    c5d = c5a = None
    if not args.no_c5 and world == 1:
        # BASELINE config 5's rows once: the sweep (auto_cluster's level 1) on
        # the first c5_n rows, the incremental add of the rest, dedup on all.
        x5 = gen_c5_rows(max(args.c5_n, args.c5_dedup_n), 768)
        best, c5 = c5_leg(eng, args, x5[:args.c5_n])
        if args.c5_dedup_n > args.c5_n:
            c5a = c5_add_leg(eng, x5[args.c5_n:args.c5_dedup_n], best)
        if args.c5_dedup_n:
            c5d = c5_dedup_leg(eng, args, x5[:args.c5_dedup_n])
        del x5

    if rank == 0:
        peak, peak_src = peaks()
        # The dominant kernel, the tcgen05 screen, timed by CUDA events around
        # each of its launches on the engine's stream: useful flops
        # 2 rows k d per launch over its mean duration.
        per_launch_ms = screen_ms / max(screen_launches, 1)
        rows_per_launch = screen_rows / max(screen_launches, 1)
        achieved = 2.0 * rows_per_launch * k * d / (per_launch_ms * 1e-3) / 1e12
        traffic = SCREEN_DRAM_BYTES_PER_ROW * rows_per_launch
        out = {
            "metric": METRIC,
            "value": n * args.steps / (ms * 1e-3) / 1e9,
            "unit": "Grows/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": c2_config(args, world),
            "engine": eng.name(),
            "exchange": {"peer_memory": xch_mapped, "why_not": xch_why} if world > 1 else None,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak, "traffic": traffic,
                         "kernel": "k_screen (tcgen05 kind::i8 screen on 16-bit fixed point in "
                                   "two int8 digits); achieved = useful 2*rows*k*d flops per "
                                   "launch / mean launch time (CUDA events), against the "
                                   "measured bf16 dense peak; executed tensor work is three "
                                   "int8 products (3x the useful ops), against an int8 peak "
                                   "taken as twice the measured bf16 one (the nominal dense "
                                   "ratio, 4.5 / 2.25 POPS)",
                         "launch_ms": per_launch_ms, "rows_per_launch": rows_per_launch,
                         "executed_int8_tops": 3.0 * achieved,
                         "executed_frac": 3.0 * achieved / (2.0 * peak),
                         "traffic_source": TRAFFIC_SOURCE,
                         "peak_source": peak_src, "top1_op_ms": top1_ms,
                         "top1_op_useful_tflops": 2.0 * (hi - lo) * k * d / (top1_ms * 1e-3)
                         / 1e12},
            "cache": {"fixed_point_rows": "built by the first call on the bound rows and kept "
                                          "for later calls (the timed steps reuse it)",
                      "cold_first_call_ms": cold_ms,
                      "cold_first_call_grows": n / (cold_ms * 1e-3) / 1e9},
            "e2e": {"value": n * args.steps / e2e_s / 1e9, "unit": "Grows/s",
                    "h2d_bytes_per_step": n * d * 4 + world * k * d * 4,
                    "d2h_bytes_per_step": n * 8,
                    "path": "eb_assign (Assigner::assign) per rank on its shard, pinned host "
                            "buffers, copies inside the timed region; results stay on each "
                            "rank's host (no gather)"},
            "update": {"op": f"scatter-add of {m:,} rows by their labels + one EMA step "
                             f"(k={k}) per rank, CUDA-event timed, rows resident",
                       "ms": upd_ms, "bytes": upd_bytes,
                       "achieved_gbs": upd_bytes / (upd_ms * 1e-3) / 1e9,
                       "peak_gbs": hbm_peak()[0],
                       "frac": upd_bytes / (upd_ms * 1e-3) / 1e9 / hbm_peak()[0],
                       "peak_source": hbm_peak()[1],
                       "bytes_source": "algorithmic: rows + labels read, sums + counts "
                                       "written; EMA 3 k d floats + 4 k"},
            "metrics": {"op": f"internal_scores (silhouette, Calinski-Harabasz, "
                              f"Davies-Bouldin, objective) of the {n:,} final labels, "
                              "wall time through the host API",
                        "ms": met_ms, "k_eff": mres["k_eff"],
                        "product_tflops": 2.0 * n * mres["k_eff"] * d / (met_ms * 1e-3) / 1e12,
                        "silhouette": mres["silhouette"],
                        "davies_bouldin": mres["davies_bouldin"]},
            "gpu_launches": launches,
            "rank_ms_per_step": rank_ms,
            "screen_stats": stats,
        }
        if tr is not None:
            out["train_s"] = {"value": train_s, "unit": "s", "n_gpus": world,
                              "timing": "wall time of Engine.train on rows bound beforehand "
                                        "(upload outside the timer, a warm-up run first), "
                                        "max over ranks",
                              "published_rtx3060_s": 0.16,
                              "mode": "group parity mode (eb_set_group_shard 0: equal to one "
                                      "GPU bit for bit)" if world > 1 else "one GPU",
                              "steps": tr.total_steps, "batch_size": tr.batch_size,
                              "final_obj": tr.obj[-1]}
            if tr_red is not None:
                dlt = abs(tr_red.obj[-1] - tr.obj[-1]) / abs(tr.obj[-1])
                out["train_s_reduce"] = {
                    "value": train_red, "unit": "s", "n_gpus": world,
                    "mode": "north-star (eb_set_group_shard 3): each rank top-1s and "
                            "scatter-adds its slice of the batch; one NCCL all-gather per step "
                            "of labels, scores and partial k x d sums + k counts, added in "
                            "rank order",
                    "final_obj": tr_red.obj[-1],
                    "obj_rel_delta_vs_parity": dlt,
                    "centroids_max_abs_diff": float(np.max(np.abs(tr_red.centroids -
                                                                  tr.centroids)))}
        if c3:
            out["c3"] = c3
        if c4:
            out["c4"] = c4
        if c5:
            out["c5_sweep"] = c5
        if c5a:
            out["c5_add"] = c5a
        if c5d:
            out["c5_dedup"] = c5d
        out["clocks"] = clk.summary()
        if not args.no_cpu:
            # Parity of the scored run: the oracle's labels and scores over the
            # rows it finishes in the budget (all 200,000 on the GPU box), bit
            # for bit against the gathered GPU results.
            cpu, ol, osc = cpu_assign(x, d, cent, budget_s=args.cpu_budget)
            r = ol.size
            out["parity"] = {"rows": r,
                             "labels_equal": bool(np.array_equal(glab[:r], ol)),
                             "scores_equal": bool(np.array_equal(gsco[:r].view(np.uint32),
                                                                 osc.view(np.uint32))),
                             "oracle": "oracle/oracle.cpp (reference cpu-fused order)"}
            if mres is not None:
                # The internal scores of the same labels by the oracle's
                # restatement (numpy, f64 sums, an f32 matrix product: the
                # reference agrees with it to rounding).
                from oracle import metrics as ometrics

                t0 = time.perf_counter()
                ores = ometrics.internal_scores(x, d, glab, k)
                o_s = time.perf_counter() - t0
                out["metrics"]["oracle"] = {
                    name: float(ores[name]) for name in
                    ("silhouette", "calinski_harabasz", "davies_bouldin", "objective")}
                out["metrics"]["rel_delta_vs_oracle"] = {
                    name: abs(float(mres[name]) - float(ores[name])) / max(abs(float(ores[name])),
                                                                           1e-300)
                    for name in ("silhouette", "calinski_harabasz", "davies_bouldin",
                                 "objective")}
                out["metrics"]["oracle_s"] = o_s
            if world == 1:
                out["cpu_baseline"] = cpu
            if tr is not None:
                cpu_s, threads, otr = cpu_train(xtrain, d, k)
                out["train_s"]["cpu_baseline"] = {
                    "value": cpu_s, "unit": "s", "cores": threads, "kind": "port",
                    "sample": "the whole C2 training (65 steps), oracle/oracle.cpp"}
                out["train_s"]["oracle_final_obj"] = otr["obj"][-1]
                out["train_s"]["obj_rel_delta_vs_oracle"] = \
                    abs(tr.obj[-1] - otr["obj"][-1]) / abs(otr["obj"][-1])
                out["train_s"]["centroids_equal_oracle"] = bool(np.array_equal(
                    tr.centroids.ravel().view(np.uint32), otr["centroids"].view(np.uint32)))
                if "train_s_reduce" in out:
                    out["train_s_reduce"]["obj_rel_delta_vs_oracle"] = \
                        abs(tr_red.obj[-1] - otr["obj"][-1]) / abs(otr["obj"][-1])
        print(json.dumps(out), flush=True)
    del xb, cb, cn, lab, sco, res, sums, counts, pos, usage
    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def gen_knn_rows(n, d, seed=4, components=10_000, sigma=0.4, dup_frac=0.05):
    """kNN self-join config rows: unit rows from a mixture (means N(0, I),
    noise sigma), with a fraction replaced by near-duplicates of random rows
    (plus N(0, 0.01^2 I), renormalised)."""
    rng = np.random.default_rng(seed)
    means = rng.standard_normal((components, d), dtype=np.float32)
    x = means[rng.integers(0, components, n)]
    x += np.float32(sigma) * rng.standard_normal((n, d), dtype=np.float32)
    nd = int(n * dup_frac)
    dup = rng.choice(n, nd, replace=False)
    x[dup] = x[rng.integers(0, n, nd)] + np.float32(0.01) * rng.standard_normal((nd, d),
                                                                                dtype=np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    return np.ascontiguousarray(x, dtype=np.float32)


def gen_c5_rows(n, d, seed=5, tops=64, subs=32, sub_sigma=0.3, row_sigma=0.2, dup_frac=0.02,
                dup_sigma=0.005):
    """Config-5 rows: a nested mixture (64 top means N(0, I), 32 sub-means per
    top = top + N(0, 0.3^2 I), rows = sub-mean + N(0, 0.2^2 I)), unit rows, with
    a fraction replaced by near-duplicates (a random row + N(0, 0.005^2 I),
    renormalised)."""
    rng = np.random.default_rng(seed)
    top = rng.standard_normal((tops, d), dtype=np.float32)
    sub = (np.repeat(top, subs, axis=0) +
           np.float32(sub_sigma) * rng.standard_normal((tops * subs, d), dtype=np.float32))
    x = sub[rng.integers(0, tops * subs, n)]
    # The row noise and the normalisation in row chunks (the generator's
    # stream is drawn in the same order: the same rows as one draw), so that
    # millions of rows need no full-size temporaries.
    step = 1 << 17
    for c0 in range(0, n, step):
        c1 = min(c0 + step, n)
        x[c0:c1] += np.float32(row_sigma) * rng.standard_normal((c1 - c0, d), dtype=np.float32)
    for c0 in range(0, n, step):
        c1 = min(c0 + step, n)
        x[c0:c1] /= np.linalg.norm(x[c0:c1], axis=1, keepdims=True)
    nd = int(n * dup_frac)
    dup = rng.choice(n, nd, replace=False)
    x[dup] = x[rng.integers(0, n, nd)] + np.float32(dup_sigma) * rng.standard_normal(
        (nd, d), dtype=np.float32)
    x[dup] /= np.linalg.norm(x[dup], axis=1, keepdims=True)
    return np.ascontiguousarray(x, dtype=np.float32)


def c3_rows(lo, hi, d, device, seed=3, chunk=65536):
    """Config-3 rows lo .. hi on the device: N(0, I) rows normalised, drawn in
    fixed 65,536-row chunks (chunk c from a generator seeded seed * 2^20 + c),
    so that any shard of the 10M rows is the same on any number of GPUs."""
    import torch

    out = torch.empty((hi - lo, d), dtype=torch.float32, device=device)
    g = torch.Generator(device=device)
    for c in range(lo // chunk, (hi + chunk - 1) // chunk if hi > lo else lo // chunk):
        g.manual_seed(seed * (1 << 20) + c)
        blk = torch.randn((chunk, d), generator=g, device=device, dtype=torch.float32)
        blk /= torch.linalg.vector_norm(blk, dim=1, keepdim=True)
        a, b = max(lo, c * chunk), min(hi, (c + 1) * chunk)
        out[a - lo:b - lo] = blk[a - c * chunk:b - c * chunk]
    return out


def c3_leg(eng, args, world, rank, local, dist):
    """assign-only throughput, 10M x 1024 unit rows vs
    k = 65,536 unit centroids (seed 1), inner product, label + score per row;
    rows sharded over the ranks (generated on the device), centroids
    replicated. Rank 0 checks its first rows against the oracle."""
    import torch

    import emeans_b200 as eb

    n, d, k = args.c3_n, 1024, 65536
    lo, hi, _ = shard(n, world, rank)
    m = hi - lo
    dev = torch.device("cuda", local)
    x = c3_rows(lo, hi, d, dev)
    g = torch.Generator(device=dev)
    g.manual_seed(1)
    cent = torch.randn((k, d), generator=g, device=dev, dtype=torch.float32)
    cent /= torch.linalg.vector_norm(cent, dim=1, keepdim=True)
    lab_t = torch.empty(max(m, 1), dtype=torch.int32, device=dev)
    sco_t = torch.empty(max(m, 1), dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    xb, cb, lab, sco = eng.wrap(x), eng.wrap(cent), eng.wrap(lab_t), eng.wrap(sco_t)
    stream = torch.cuda.ExternalStream(eng.stream())

    def step():
        if m:
            eng.top1(xb, d, None, range(0, m), cb, None, k, eb.IP, lab, sco)

    step()
    eng.sync()
    if dist:
        dist.barrier()
    eng.set_kernel_timing(True)
    eng.screen_timing()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.c3_steps):
        step()
    t1.record(stream)
    t1.synchronize()
    eng.sync()
    screen_ms, launches, srows = eng.screen_timing()
    eng.set_kernel_timing(False)
    ms = _max_over_ranks(dist, [t0.elapsed_time(t1) / args.c3_steps])[0]
    res = {"workload": f"C3 assign: {n:,} x {d} unit rows vs k={k} unit centroids (seed 1), "
                       "inner product, label u32 + score f32 per row, rows on the device",
           "rows": n, "d": d, "k": k, "n_gpus": world, "steps": args.c3_steps,
           "ms_per_pass": ms, "grows_per_s": n / (ms * 1e-3) / 1e9,
           "useful_tflops": 2.0 * n * k * d / (ms * 1e-3) / 1e12,
           "screen_useful_tflops_rank0": 2.0 * srows * k * d / max(screen_ms * 1e-3, 1e-12) / 1e12,
           "parallelism": f"rows sharded over {world} GPU(s), centroids replicated, results "
                          "stay on each rank"}
    if rank == 0 and m:
        import oracle

        chk = min(args.c3_check, m)
        xs = x[:chk].cpu().numpy()
        cs = cent.cpu().numpy()
        gl = lab_t[:chk].cpu().numpy().view(np.uint32)
        gs = sco_t[:chk].cpu().numpy()
        threads = os.cpu_count() or 1
        done, t = 0, time.perf_counter()
        ok_l = ok_s = True
        while done < chk and time.perf_counter() - t < args.cpu_budget:
            e = min(done + 4096, chk)
            ol, osc = oracle.top1(xs[done:e].ravel(), d, cs.ravel(), oracle.IP, threads=threads)
            ok_l &= bool(np.array_equal(ol, gl[done:e]))
            ok_s &= bool(np.array_equal(osc.view(np.uint32), gs[done:e].view(np.uint32)))
            done = e
        dt = time.perf_counter() - t
        res["parity"] = {"rows": done, "labels_equal": ok_l, "scores_equal": ok_s}
        res["cpu_baseline"] = {"value": done / dt / 1e9, "unit": "Grows/s", "cores": threads,
                               "kind": "port", "sample": f"first {done:,} rows, {dt:.1f} s"}
    del xb, cb, lab, sco, x, cent, lab_t, sco_t
    torch.cuda.empty_cache()
    return res


def c4_leg(eng, args, world, rank, dist):
    """exact kNN self-join, 1M x 384, kk = 10, inner
    product, self excluded, through the host-array API; with N GPUs the
    database is sharded, queries replicated, per-shard lists merged on the
    device (eb_topk_group). Rank 0 checks its first queries against the
    oracle's self-join."""
    n, d, kk = args.c4_n, 384, 10
    x = gen_knn_rows(n, d)
    lo, hi, _ = shard(n, world, rank)

    def call():
        if world > 1:
            return eng.topk_group(x, x[lo:hi], lo, n, d, kk, exclude_self=True)
        return eng.topk(x, x, d, kk, exclude_self=True)

    call()  # warm-up (screen scratch, the data's copy)
    times = []
    for _ in range(args.c4_steps):
        if dist:
            dist.barrier()
        t = time.perf_counter()
        ids, sims = call()
        times.append(time.perf_counter() - t)
    t = _max_over_ranks(dist, [statistics.median(times)])[0]
    res = {"workload": f"C4 kNN self-join: {n:,} x {d} unit rows (10,000-component mixture, "
                       "5% near-duplicates), kk=10, inner product, self excluded; host arrays "
                       "in and out (eb_topk / eb_topk_group)",
           "rows": n, "d": d, "kk": kk, "n_gpus": world, "steps": args.c4_steps,
           "s_per_join": t, "queries_per_s": n / t,
           "useful_tflops": 2.0 * n * n * d / t / 1e12,
           "parallelism": f"database sharded over {world} GPU(s), queries replicated, lists "
                          "all-gathered and merged on the device" if world > 1 else "one GPU"}
    if rank == 0:
        import oracle

        chk = min(args.c4_check, n)
        threads = os.cpu_count() or 1
        done, t0 = 0, time.perf_counter()
        ok_i = ok_s = True
        while done < chk and time.perf_counter() - t0 < args.cpu_budget:
            e = min(done + 1000, chk)
            oi, osm = oracle.topk_self_rows(x, d, done, e - done, kk, threads=threads)
            ok_i &= bool(np.array_equal(oi, ids[done * kk:e * kk]))
            ok_s &= bool(np.array_equal(osm.view(np.uint32), sims[done * kk:e * kk].view(np.uint32)))
            done = e
        dt = time.perf_counter() - t0
        res["parity"] = {"queries": done, "ids_equal": ok_i, "sims_equal": ok_s,
                         "oracle": "FMA-chain exact top-k (oracle/oracle.cpp)"}
        res["cpu_baseline"] = {"value": done / dt, "unit": "queries/s", "cores": threads,
                               "kind": "port", "sample": f"first {done:,} queries x all {n:,} "
                                                          f"rows, {dt:.1f} s"}
    return res


def c5_leg(eng, args, x):
    """BASELINE config 5's level-1 sweep path (auto::sweep, crates/emeans-cluster/
    src/auto.rs:455-505) on a C5-shaped sample, one GPU: the rows bound once,
    then for k in (32, 64, 128) two fits each (spherical training with
    AutoConfig's 5 epochs, inner-product assignment of every row), the better
    kept and scored by internal_scores. The oracle runs the first fit (train,
    assign, internal scores) on the host cores: the parity check and the CPU
    baseline of that fit."""
    import oracle
    from oracle import metrics as ometrics

    n, d = x.shape
    ks, restarts, nepochs, seed, salt = (32, 64, 128), 2, 5.0, 1234, 0
    eng.bind_data(x, d)
    eng.sweep(x, d, ks, nepochs, seed, salt, restarts=1)  # warm-up: every k's shapes
    eng.sync()
    t0 = time.perf_counter()
    res = eng.sweep(x, d, ks, nepochs, seed, salt, restarts=restarts)
    sweep_s = time.perf_counter() - t0
    t0 = time.perf_counter()
    tr, lab, sco = eng.fit(x, d, ks[0], nepochs, eb_seed_for(seed, salt, ks[0], 0))
    gmet = eng.internal_scores(x, d, lab, ks[0])
    fit_s = time.perf_counter() - t0
    eng.unbind_data()
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    want = oracle.train(x, d, ks[0], nepochs=nepochs, seed=eb_seed_for(seed, salt, ks[0], 0),
                        spherical=True, threads=threads)
    wl, ws = oracle.top1(x.ravel(), d, want["centroids"], oracle.IP, threads=threads)
    wmet = ometrics.internal_scores(x, d, wl, ks[0])
    cpu_s = time.perf_counter() - t0
    rel = {key: abs(gmet[key] - wmet[key]) / max(abs(wmet[key]), 1e-30)
           for key in ("silhouette", "calinski_harabasz", "davies_bouldin", "objective")}
    best = max(res, key=lambda r: r[1]["silhouette"])
    return best, {"workload": f"C5 level-1 sweep: {n:,} x {d} nested-mixture unit rows (64 x 32 "
                        "sub-means, 2% near-duplicates), k in (32, 64, 128), 2 fits each, "
                        "spherical, 5 epochs, rows bound once (SharedAssigner)",
            "rows": n, "d": d, "ks": list(ks), "restarts": restarts,
            "sweep_s": sweep_s, "fits": len(ks) * restarts,
            "chosen": [{"k": k, "objective": obj, "silhouette": sc["silhouette"],
                        "k_eff": sc["k_eff"]} for k, sc, _, _, _, obj in res],
            "one_fit_s": fit_s,
            "parity": {"fit": f"k={ks[0]}, restart 0",
                       "centroids_equal": bool(np.array_equal(
                           tr.centroids.ravel().view(np.uint32),
                           want["centroids"].view(np.uint32))),
                       "labels_equal": bool(np.array_equal(lab, wl)),
                       "scores_equal": bool(np.array_equal(sco.view(np.uint32),
                                                           ws.view(np.uint32))),
                       "internal_scores_max_rel_diff": max(rel.values())},
            "cpu_baseline": {"value": cpu_s, "unit": "s", "cores": threads, "kind": "port",
                             "sample": f"the first fit (k={ks[0]}: train, assign, internal "
                                       "scores) on the host, oracle/"}}


def c5_add_leg(eng, x_add, best):
    """BASELINE config 5's incremental add (Hierarchy::add's device work, the
    new rows' inner-product assignment to the chosen model's centroids) on the
    rows after the sweep's, through the host-array assign (eb_assign), after a
    warm-up call; the first rows checked against the oracle bit for bit."""
    import oracle
    import emeans_b200 as eb

    k, _, tr, _, _, _ = best
    m, d = x_add.shape
    cent = np.ascontiguousarray(tr.centroids, dtype=np.float32)
    eng.assign(x_add, d, cent, eb.IP)  # warm-up (the same shape)
    t0 = time.perf_counter()
    lab, sco = eng.assign(x_add, d, cent, eb.IP)
    add_s = time.perf_counter() - t0
    q = min(2000, m)
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    wl, ws = oracle.top1(x_add[:q].ravel(), d, cent.ravel(), oracle.IP, threads=threads)
    cpu_s = time.perf_counter() - t0
    return {"workload": f"C5 incremental add: {m:,} new rows assigned (inner product) to the "
                        f"chosen model's k={k} centroids, host arrays in and out (eb_assign)",
            "rows": m, "k": k, "s": add_s, "rows_per_s": m / add_s,
            "parity": {"rows": q, "labels_equal": bool(np.array_equal(lab[:q], wl)),
                       "scores_equal": bool(np.array_equal(sco[:q].view(np.uint32),
                                                           ws.view(np.uint32)))},
            "cpu_baseline": {"value": q / cpu_s, "unit": "rows/s", "cores": threads,
                             "kind": "port", "sample": f"the first {q:,} added rows"}}


def c5_dedup_leg(eng, args, x):
    """BASELINE config 5's dedup at full size on one GPU: 2,000,000 x 768 nested-
    mixture unit rows with 2% near-duplicates, dedup::dedup (crates/emeans-cluster/
    src/dedup.rs:160-183) at sim_threshold 0.97 and k 10 through the host-array
    API (the rows copied to the device, the exact kNN self-join on the engine,
    the grouping stages on the host), after a 50,000-row warm-up call. Parity:
    the nearest-neighbour similarity (self excluded) of the first rows, bit for
    bit against the oracle's exact self-join over all rows (the oracle's time
    on them is the CPU baseline)."""
    import oracle
    import emeans_b200 as eb

    n, d = x.shape
    kk = 10
    cfg = eb.DedupConfig(k=kk, sim_threshold=0.97)
    eng.dedup(x[:50_000], d, cfg=cfg)  # warm-up
    eng.sync()
    s0 = eng.stats()
    t0 = time.perf_counter()
    res = eng.dedup(x, d, cfg=cfg)
    dedup_s = time.perf_counter() - t0
    s1 = eng.stats()
    threads = os.cpu_count() or 1
    q = min(args.c5_dedup_check, n)
    t0 = time.perf_counter()
    _, wsims = oracle.topk_self_rows(x, d, 0, q, kk, threads=threads)
    cpu_s = time.perf_counter() - t0
    want = wsims.reshape(q, kk)[:, 0]
    return {"workload": f"C5 dedup: {n:,} x {d} nested-mixture unit rows (64 x 32 sub-means, "
                        "2% near-duplicates, sigma 0.005), sim_threshold 0.97, k 10, host "
                        "arrays in and out (eb_dedup)",
            "rows": n, "d": d, "k": kk, "sim_threshold": 0.97,
            "s_per_dedup": dedup_s,
            "self_join_useful_tflops": 2.0 * n * n * d / dedup_s / 1e12,
            "groups": res.n_groups(), "rows_in_groups_of_two_or_more":
                int(np.sum(res.sizes[res.sizes > 1])),
            "linked_pairs": res.linked_pairs,
            "largest_group": int(res.sizes.max()) if res.sizes.size else 0,
            "self_join_stats": {key: s1[key] - s0[key] for key in
                                ("screened_rows", "fallback_rows", "rescored_candidates",
                                 "exact_rows")},
            "parity": {"rows": q,
                       "nn_sim_equal": bool(np.array_equal(res.nn_sim[:q].view(np.uint32),
                                                           want.view(np.uint32))),
                       "oracle": "FMA-chain exact self-join (oracle/oracle.cpp)"},
            "cpu_baseline": {"value": q / cpu_s, "unit": "queries/s", "cores": threads,
                             "kind": "port",
                             "sample": f"the self-join of the first {q:,} rows against all "
                                       f"{n:,}, {cpu_s:.1f} s"}}


def eb_seed_for(seed, salt, k, restart):
    import emeans_b200 as eb

    return eb.seed_for(seed, salt, k, restart)


def run_knn(args):
    """--knn N: the kNN self-join config's shape on N rows (d 384, kk 10, inner
    product, self excluded) through eb_topk with host arrays; one JSON line."""
    import emeans_b200 as eb

    n, d, kk = args.knn, 384, 10
    x = gen_knn_rows(n, d)
    eng = eb.Engine(0)
    eng.topk(x[:2048], x, d, kk)  # warm-up
    times = []
    for _ in range(max(1, args.steps)):
        t0 = time.perf_counter()
        eng.topk(x, x, d, kk, exclude_self=True)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    print(json.dumps({"metric": "kNN self-join (d 384, kk 10, IP) queries/s", "value": n / t,
                      "unit": "queries/s", "n_gpus": 1, "steps": len(times),
                      "higher_is_better": True, "data": "synthetic",
                      "config": {"workload": f"kNN self-join config shape, {n} rows", "rows": n,
                                 "d": d, "kk": kk},
                      "s_per_join": t, "useful_tflops": 2.0 * n * n * d / t / 1e12,
                      "stats": eng.stats()}), flush=True)
    eng.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--n", type=int, default=200_000)
    ap.add_argument("--d", type=int, default=768)
    ap.add_argument("--k", type=int, default=1024)
    ap.add_argument("--ref-rows", type=int, default=0,
                    help="rows per reference step (default: all --n rows)")
    ap.add_argument("--cpu-budget", type=float, default=20.0,
                    help="seconds of host time for the oracle parity leg")
    ap.add_argument("--no-train", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--save-cent", default=None, help="write the trained centroids (.npy)")
    ap.add_argument("--load-cent", default=None, help="use these centroids instead of training")
    ap.add_argument("--no-c3", action="store_true", help="skip the config-3 assign leg")
    ap.add_argument("--no-c4", action="store_true", help="skip the config-4 kNN leg")
    ap.add_argument("--no-c5", action="store_true", help="skip the config-5 sweep leg")
    ap.add_argument("--c5-n", type=int, default=1_600_000,
                    help="rows of the config-5 sweep (the first rows of the config-5 set)")
    ap.add_argument("--c5-dedup-n", type=int, default=2_000_000,
                    help="rows of the config-5 set: the rows after the sweep's are added "
                         "(assigned to the chosen model), dedup runs on all (0: neither)")
    ap.add_argument("--c5-dedup-check", type=int, default=1000,
                    help="config-5 dedup rows whose nearest neighbour the oracle checks")
    ap.add_argument("--c3-n", type=int, default=10_000_000)
    ap.add_argument("--c3-steps", type=int, default=2)
    ap.add_argument("--c3-check", type=int, default=100_000,
                    help="config-3 rows checked against the oracle (time-bounded)")
    ap.add_argument("--c4-n", type=int, default=1_000_000)
    ap.add_argument("--c4-steps", type=int, default=2)
    ap.add_argument("--c4-check", type=int, default=10_000,
                    help="config-4 queries checked against the oracle (time-bounded)")
    ap.add_argument("--knn", type=int, default=0,
                    help="instead of the headline: the kNN self-join config's shape on this "
                         "many rows (one GPU)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.knn:
        run_knn(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
