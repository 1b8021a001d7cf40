#!/usr/bin/env python
"""Benchmark of the farthest-point-sampling engine (one JSON line on rank 0).

Metric: FPS samples/sec (whole box) at 1/2/4/8 B200; ms per
122,880 -> 16,384 scan.

Default workload: every rank samples one synthetic
64-beam LiDAR scan (122,880 points -> 16,384 samples, range x,y in [-80, 80],
z in [-3, 3], 32 x 32 x 8 blocks) per step, its own scan (seed = rank).  The
path shards whole clouds across GPUs with no collective, so scaling is weak:
`value` = samples of all ranks / the slowest rank's time.  `--workload c5`
runs the 256-scan batch split over the ranks instead (strong scaling).

  value   device-resident: the scan is in HBM before timing starts; each step
          is one nsfps_fps_device call (binning, sort, leaf build, sampling
          loop, epilogue) timed with CUDA events on the launching stream, with
          a 256 MiB L2 flush outside the timed window between steps.
  e2e     the same through nsfps_fps with HOST buffers: the H2D copy of the
          points and the D2H copy of the indices are inside the timed region.
  roofline  for the sampling-loop kernel: algorithmic bytes = 12 N + 20 sum_i
          u_i (u_i = points in the buckets the reference updates at step i,
          counted by the kernel itself) over the kernel's event-timed duration,
          against the measured HBM copy bandwidth.
  cpu_baseline  the reference's yuezu_fps() compiled from its own sources
          (oracle/_ref), timed on this host on a bounded sample.

  batch_c5  every line also carries the 256-scan batch (config 5) split over
          the ranks (strong scaling: 256 / N scans per rank): samples/s of the
          whole box over the slowest rank's device time, each rank's time,
          and the reference CPU on 16 threads (--no-batch-c5 skips it).

`--impl reference` times the reference CPU implementation alone on the same
workload with the host threads it can use (rank 0 only under torchrun).

`--path group [--radius R --nsample S]` measures the step after sampling
instead: the ball query around the c2 scan's 16,384 FPS samples (run_group).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from ns_fps_b200 import dist as D  # noqa: E402
from ns_fps_b200 import synthetic as S  # noqa: E402

METRIC = "FPS samples/sec (whole box) at 1/2/4/8 B200; ms per 122,880→16,384 scan"
L2_NOTE = "GPU arm: 256 MiB L2 flush between steps, outside the timed window"
# shared memory bytes per clock per SM (B200), for the sampling loop's SMEM figure
SMEM_BYTES_PER_CLK = 128


def config_dict(name: str, limit: int = 0):
    """The workload as both arms describe it (identical dicts)."""
    cfg = S.CONFIGS[name]
    clouds = min(cfg.clouds, limit) if limit > 0 else cfg.clouds
    return {"workload": name, "points": cfg.n, "k": cfg.k, "blocks": list(cfg.blocks),
            "range": list(cfg.rng), "clouds": clouds, "l2": L2_NOTE}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["c1", "c2", "c3", "c4", "c5"], default="c2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batch-c5", action="store_true",
                    help="skip the 256-scan batch sub-record")
    ap.add_argument("--c5-steps", type=int, default=2, help="timed steps of the batch_c5 record")
    ap.add_argument("--clouds", type=int, default=0,
                    help="c3/c5: sample only this many clouds of the batch (small cases "
                         "for profiling; the bench line then names the count)")
    ap.add_argument("--path", choices=["fps", "group"], default="fps",
                    help="fps: the sampler (default); group: the ball query after it")
    ap.add_argument("--radius", type=float, default=0.5, help="--path group: ball radius")
    ap.add_argument("--nsample", type=int, default=32, help="--path group: samples per ball")
    return ap.parse_args()


def workload_clouds(name: str, rank: int, world: int, limit: int = 0):
    """The clouds this rank samples every step, and a description."""
    cfg = S.CONFIGS[name]
    if name in ("c1", "c2", "c4"):
        clouds = S.make(name, seed=rank, count=1)  # weak scaling: one cloud per rank
        scaling = "weak"
        per = 1
    else:
        total = min(cfg.clouds, limit) if limit > 0 else cfg.clouds
        idx = D.shard_indices(total, rank, world)
        if name == "c3":
            clouds = [S.sphere_cube_cloud(cfg.n, seed=i) for i in idx]
        else:
            clouds = [S.lidar_scan(i) for i in idx]
        scaling = "strong"
        per = len(idx)
    return cfg, clouds, scaling, per


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None
        # wait (bounded) for the first sample, so that a timed region shorter
        # than the sampling period is still bracketed by samples
        t0 = time.time()
        while self.proc is not None and not self.lines and time.time() - t0 < 3.0:
            time.sleep(0.01)
        return self

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            n, t0 = len(self.lines), time.time()
            while len(self.lines) <= n and time.time() - t0 < 1.0:  # one sample after
                time.sleep(0.01)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx.append(float(f[1]))
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(max(mx)),
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def profiled_traffic(workload: str):
    """DRAM bytes of one sampling-loop launch from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "loop_kernel_traffic.json")
    try:
        with open(path) as f:
            t = json.load(f)
        return t.get(workload)
    except (OSError, ValueError):
        return None


def cpu_baseline(cfg, clouds, threads: int):
    """The reference's yuezu_fps() (oracle/_ref) on a bounded sample: one
    whole cloud per thread, `threads` threads (1 for a single cloud)."""
    import oracle
    if not oracle.have_ref():
        sample = clouds[: max(1, threads)]
        t0 = time.perf_counter()
        n = 0
        for c in sample:
            n += len(oracle.fps(c, cfg.k, cfg.rng, cfg.blocks))
        dt = time.perf_counter() - t0
        return {"value": n / dt, "unit": "samples/s", "cores": 1, "kind": "port",
                "sample": f"{len(sample)} cloud(s) of {cfg.n} points -> {cfg.k} samples, "
                          f"{dt:.2f} s"}
    sample = clouds[: max(1, threads)]
    outs, secs = oracle.ref_fps_many(sample, cfg.k, cfg.rng, cfg.blocks, threads=len(sample))
    n = sum(len(o) for o in outs)
    return {"value": n / secs, "unit": "samples/s", "cores": len(sample), "kind": "reference",
            "sample": f"{len(sample)} whole cloud(s) of {cfg.n} points -> {cfg.k} samples "
                      f"on {len(sample)} thread(s), {secs:.2f} s"}


def run_reference(args):
    """--impl reference: the reference CPU implementation alone."""
    rank, _, world = D.env_rank()
    if rank != 0:
        return 0
    import oracle
    cfg, clouds, scaling, per = workload_clouds(args.workload, 0, 1, args.clouds)
    if args.workload in ("c3", "c5"):
        clouds = clouds[: max(1, min(len(clouds), os.cpu_count() or 1))]
    threads = len(clouds)
    times, n_samples = [], 0
    for s in range(args.warmup + args.steps):
        if oracle.have_ref():
            outs, secs = oracle.ref_fps_many(clouds, cfg.k, cfg.rng, cfg.blocks, threads=threads)
            kind = "reference"
        else:
            t0 = time.perf_counter()
            outs = [oracle.fps(c, cfg.k, cfg.rng, cfg.blocks) for c in clouds]
            secs = time.perf_counter() - t0
            kind, threads = "port", 1
        if s >= args.warmup:
            times.append(secs)
            n_samples += sum(len(o) for o in outs)
    total = sum(times)
    value = n_samples / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "samples/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total / args.steps * 1e3, "higher_is_better": True, "scaling": scaling,
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(args.workload, args.clouds), "clouds_per_step": len(clouds),
        "cpu_baseline": {"value": value, "unit": "samples/s", "cores": threads, "kind": kind,
                         "sample": f"{len(clouds)} whole cloud(s) per step, {threads} thread(s)"},
        "e2e": {"value": value, "unit": "samples/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def batch_c5(args, rank: int, world: int, dev, capi, flush, stream):
    """The 256-scan batch (config 5) split over the ranks, strong scaling:
    rank r samples scans r, r + N, ... as one nsfps_fps_device call per step,
    timed with CUDA events (warm-up 1, args.c5_steps timed steps, the L2 flush
    between steps).  Every rank takes the same collective steps.  Returns the
    record on rank 0, None elsewhere."""
    import torch
    cfg, clouds, _, per = workload_clouds("c5", rank, world)
    offsets = np.zeros(len(clouds) + 1, dtype=np.int64)
    offsets[1:] = np.cumsum([c.shape[0] for c in clouds])
    d_xyz = torch.from_numpy(np.concatenate(clouds, axis=0)).to(dev)
    d_out = torch.empty(len(clouds) * cfg.k, dtype=torch.int64, device=dev)

    def step():
        return capi.fps_device(d_xyz.data_ptr(), offsets, cfg.k, (cfg.rng, cfg.blocks), False,
                               d_out.data_ptr(), stream.cuda_stream)

    step()
    torch.cuda.synchronize(dev)
    D.barrier(dev.index)
    samples, ms = 0, 0.0
    capi.set_profiling(True)
    with ClockSampler(dev.index) as clk:
        for _ in range(max(1, args.c5_steps)):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            samples += sum(step())
            b.record(stream)
            b.synchronize()
            ms += a.elapsed_time(b)
    prof = capi.last_profile()
    steps = max(1, args.c5_steps)
    mine = np.zeros(world)
    mine[rank] = ms / steps
    rank_ms = D.sum_over_ranks(list(mine), device=dev)
    total = D.sum_over_ranks([samples], device=dev)[0]
    del d_xyz, d_out
    if rank != 0:
        return None
    slow, fast = max(rank_ms), min(rank_ms)
    rec = {"workload": "c5", "value": total / steps / (slow / 1e3), "unit": "samples/s",
           "scaling": "strong", "scans": cfg.clouds, "scans_per_gpu": per,
           "ms_per_step": slow, "rank_ms": rank_ms, "slowest_over_fastest": slow / fast,
           "steps": steps, "warmup": 1,
           "layout": {"mode": "grid groups" if prof.mode == 3 else "clusters",
                      "ctas_per_scan": int(prof.ctas_per_cloud)},
           "clocks": clk.summary()}
    # roofline of the batch's sampling-loop launch on rank 0 (the last step):
    # algorithmic bytes 12 N + 20 sum_i u_i over its scans, over the launch's
    # event-timed duration; DRAM traffic scaled from the committed capture of
    # 9 scans (each scan's part is read once, so traffic grows with the scans)
    n_pts = float(offsets[-1])
    alg = 12.0 * n_pts + 20.0 * float(prof.ref_points_updated)
    peak, peak_kind = measured_peaks()
    t9 = profiled_traffic("c5x9")
    achieved = alg / (prof.loop_ms / 1e3) / 1e9
    rec["roofline"] = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                       "frac": achieved / peak, "peak_source": peak_kind,
                       "traffic": t9 * len(clouds) / 9.0 if t9 else None,
                       "kernel": "fps_rounds_cluster (batch groups)" if prof.mode == 3
                                 else "fps_rounds_cluster (clusters)",
                       "algorithmic_bytes_per_launch": alg,
                       "kernel_ms_per_launch": float(prof.loop_ms),
                       "operative_bound": "latency and worker throughput: each scan's serial "
                                          "step chain; the scans are shared-memory resident"}
    if not args.no_cpu_baseline:
        import oracle
        threads = min(16, os.cpu_count() or 1)
        sample = clouds[:threads] if len(clouds) >= threads else \
            [S.lidar_scan(i) for i in range(threads)]
        if oracle.have_ref():
            outs, secs = oracle.ref_fps_many(sample, cfg.k, cfg.rng, cfg.blocks, threads=threads)
            kind = "reference"
        else:
            t0 = time.perf_counter()
            outs = [oracle.fps(c, cfg.k, cfg.rng, cfg.blocks) for c in sample[:1]]
            secs, kind, threads = time.perf_counter() - t0, "port", 1
        rec["reference_cpu"] = {"value": sum(len(o) for o in outs) / secs, "unit": "samples/s",
                                "cores": threads, "kind": kind,
                                "sample": f"{len(outs)} whole scan(s) on {threads} thread(s), "
                                          f"{secs:.2f} s"}
    return rec


def run_ours(args):
    import torch
    rank, local, world = D.env_rank()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    D.init("nccl", timeout_s=300)
    from ns_fps_b200 import capi

    cfg, clouds, scaling, per = workload_clouds(args.workload, rank, world, args.clouds)
    k = cfg.k
    offsets = np.zeros(len(clouds) + 1, dtype=np.int64)
    offsets[1:] = np.cumsum([c.shape[0] for c in clouds])
    packed = np.ascontiguousarray(np.concatenate(clouds, axis=0).astype(np.float32))
    d_xyz = torch.from_numpy(packed).to(dev)
    d_out = torch.empty(len(clouds) * k, dtype=torch.int64, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    ranges = (cfg.rng, cfg.blocks)

    def step():
        return capi.fps_device(d_xyz.data_ptr(), offsets, k, ranges, False, d_out.data_ptr(),
                               stream.cuda_stream)

    capi.set_profiling(True)
    for _ in range(args.warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize(dev)
    D.barrier(local)
    torch.cuda.synchronize(dev)

    # ---- device-resident timed region
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    loop_ms, ref_pts, evals, launches, samples, loop_mode = 0.0, 0, 0, 0, 0, 0
    with ClockSampler(local) as clk:
        for s in range(args.steps):
            flush.zero_()  # L2 flush outside the timed window
            ev[s][0].record(stream)
            lens = step()
            ev[s][1].record(stream)
            prof = capi.last_profile()
            loop_ms += prof.loop_ms
            ref_pts += prof.ref_points_updated
            evals += prof.points_evaluated
            launches += prof.launches
            loop_mode = prof.mode
            samples += sum(lens)
        torch.cuda.synchronize(dev)
    step_ms = [a.elapsed_time(b) for a, b in ev]
    my_ms = float(sum(step_ms))
    D.barrier(local)

    # ---- end to end through the C ABI with host buffers
    host = [np.ascontiguousarray(c) for c in clouds]
    pinned = [torch.from_numpy(c).pin_memory() for c in host]
    e2e_times = []
    for s in range(max(1, args.steps // 2) + 1):
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        if len(pinned) == 1:
            out = capi.fps(pinned[0].numpy(), k, cfg.rng, cfg.blocks, device=local)
            e2e_n = len(out)
        else:
            outs = capi.fps_batched([p.numpy() for p in pinned], k, cfg.rng, cfg.blocks,
                                    devices=(local,))
            e2e_n = sum(len(o) for o in outs)
        dt = time.perf_counter() - t0
        if s > 0:
            e2e_times.append(dt)
    e2e_s = float(np.mean(e2e_times))

    # ---- the 256-scan batch over the ranks (all ranks, same collectives)
    batch = None
    if not args.no_batch_c5 and args.workload != "c5":
        batch = batch_c5(args, rank, world, dev, capi, flush, stream)

    # ---- aggregate over ranks (max of times, sum of work)
    mx = D.max_over_ranks([my_ms, e2e_s], device=dev)
    sm = D.sum_over_ranks([samples, e2e_n, ref_pts, len(clouds)], device=dev)
    total_ms, e2e_max = mx
    all_samples, all_e2e, _, _ = sm

    result = None
    if rank == 0:
        value = all_samples / (total_ms / 1e3)
        e2e_value = all_e2e / e2e_max
        # roofline of the sampling loop kernel on this rank
        n_pts = int(offsets[-1])
        alg_bytes = 12.0 * n_pts * args.steps + 20.0 * ref_pts
        achieved = alg_bytes / (loop_ms / 1e3) / 1e9
        peak, peak_kind = measured_peaks()
        traffic = profiled_traffic(args.workload)
        iters = samples / max(len(clouds), 1) / args.steps
        clocks = clk.summary()
        # the loop keeps the cloud in shared memory: its operative bound is the
        # serial step chain (us_per_iteration); for scale, the same algorithmic
        # bytes against the shared-memory bandwidth of the SMs it occupies
        sm_used = min(148, int(prof.ctas_per_cloud) * len(clouds))
        mhz = clocks.get("sm_mhz") or 1965.0
        smem_peak = sm_used * SMEM_BYTES_PER_CLK * mhz * 1e6 / 1e9
        result = {
            "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(args.workload, args.clouds), "clouds_per_gpu": len(clouds),
            "ms_per_scan": my_ms / args.steps / max(len(clouds), 1) if per == 1 else None,
            "us_per_iteration": (loop_ms / args.steps) * 1e3 / max(iters, 1),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "peak_source": peak_kind,
                         "kernel": "fps_rounds_cluster" if loop_mode in (2, 3) else "fps_loop_cluster",
                         "algorithmic_bytes_per_launch": alg_bytes / args.steps,
                         "kernel_ms_per_launch": loop_ms / args.steps,
                         "points_evaluated_per_launch": evals / args.steps,
                         "operative_bound": "latency: the serial step chain (us_per_iteration); "
                                            "the cloud is shared-memory resident",
                         "smem": {"achieved": achieved, "peak": smem_peak, "unit": "GB/s",
                                  "frac": achieved / smem_peak, "sms": sm_used,
                                  "peak_basis": f"{SMEM_BYTES_PER_CLK} B/clk/SM x {sm_used} SMs "
                                                f"x {mhz:.0f} MHz"}},
            "e2e": {"value": e2e_value, "unit": "samples/s",
                    "h2d_bytes_per_step": int(12 * n_pts),
                    "d2h_bytes_per_step": int(8 * k * len(clouds) + 8 * len(clouds))},
            "gpu_launches": int(launches),
            "clocks": clocks,
        }
        if batch is not None:
            result["batch_c5"] = batch
        if not args.no_cpu_baseline:
            cfgc = S.CONFIGS[args.workload]
            threads = 1 if per == 1 else min(len(clouds), os.cpu_count() or 1)
            result["cpu_baseline"] = cpu_baseline(cfgc, clouds, threads)
    D.barrier(local)
    D.finalize()
    if result is not None:
        print(json.dumps(result), flush=True)
    return 0


def run_group(args):
    """--path group: the ball query after sampling (one GPU, rank 0 of N
    replicas).  Workload: the c2 scan, its 16,384 FPS samples as centres
    (computed once, untimed), radius --radius, --nsample per ball.  A step is
    one nsfps_ball_query_device call (grid build + query); `e2e` is
    nsfps_ball_query with host buffers (points and centres in, indices and
    hit counts out).  The reference has no ball query, so there is no
    reference arm; cpu_baseline is the brute-force restatement (oracle, one
    thread) on the first 1,024 centres."""
    import torch
    rank, local, world = D.env_rank()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    D.init("nccl", timeout_s=300)
    from ns_fps_b200 import capi
    cfg = S.CONFIGS["c2"]
    cloud = S.lidar_scan(seed=rank)
    d_xyz = torch.from_numpy(cloud).to(dev)
    d_s = torch.empty(cfg.k, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev)
    n_s = capi.fps_device(d_xyz.data_ptr(), [0, cfg.n], cfg.k, (cfg.rng, cfg.blocks), False,
                          d_s.data_ptr(), stream.cuda_stream)[0]
    centers = d_xyz[d_s[:n_s]].contiguous()
    m, S_, radius = int(n_s), int(args.nsample), float(args.radius)
    d_idx = torch.empty((m, S_), dtype=torch.int64, device=dev)
    d_hits = torch.empty(m, dtype=torch.int32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def step():
        capi.ball_query_device(d_xyz.data_ptr(), [0, cfg.n], centers.data_ptr(), [0, m], radius,
                               S_, d_idx.data_ptr(), d_hits.data_ptr(), stream.cuda_stream)

    capi.set_profiling(True)
    for _ in range(args.warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize(dev)
    D.barrier(local)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    q_ms, g_ms, launches = 0.0, 0.0, 0
    with ClockSampler(local) as clk:
        for s in range(args.steps):
            flush.zero_()
            ev[s][0].record(stream)
            step()
            ev[s][1].record(stream)
            prof = capi.last_profile()
            q_ms += prof.loop_ms
            g_ms += prof.setup_ms
            launches += prof.launches
        torch.cuda.synchronize(dev)
    my_ms = float(sum(a.elapsed_time(b) for a, b in ev))
    D.barrier(local)
    host_pts, host_c = cloud, centers.cpu().numpy()
    e2e = []
    for s in range(max(1, args.steps // 2) + 1):
        t0 = time.perf_counter()
        capi.ball_query(host_pts, host_c, radius, S_, device=local)
        if s:
            e2e.append(time.perf_counter() - t0)
    e2e_s = float(np.mean(e2e))
    total_ms, e2e_max = D.max_over_ranks([my_ms, e2e_s], device=dev)
    result = None
    if rank == 0:
        # algorithmic bytes of the query kernel: points (12 B) and centres
        # (12 B) read once, the index rows (8 B per slot) and hit counts written
        alg = 12.0 * cfg.n + 12.0 * m + 8.0 * m * S_ + 4.0 * m
        q_launch_ms = q_ms / args.steps
        achieved = alg / (q_launch_ms / 1e3) / 1e9
        peak, peak_kind = measured_peaks()
        result = {
            "metric": "ball queries/s after FPS (c2 scan, 16,384 centres)", "path": "group",
            "value": world * m / (total_ms / 1e3 / args.steps), "unit": "queries/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "c2 + ball query", "points": cfg.n, "centres": m,
                       "radius": radius, "nsample": S_,
                       "l2": "256 MiB flush between steps, outside the timed window"},
            "grid_build_ms": g_ms / args.steps, "query_kernel_ms": q_launch_ms,
            "mean_hits": float(d_hits.float().mean().item()),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": None, "peak_source": peak_kind,
                         "kernel": "ball_query", "algorithmic_bytes_per_launch": alg,
                         "kernel_ms_per_launch": q_launch_ms},
            "e2e": {"value": world * m / e2e_max, "unit": "queries/s",
                    "h2d_bytes_per_step": int(12 * cfg.n + 12 * m),
                    "d2h_bytes_per_step": int(8 * m * S_ + 4 * m)},
            "gpu_launches": int(launches),
            "clocks": clk.summary(),
        }
        if not args.no_cpu_baseline:
            import oracle
            t0 = time.perf_counter()
            oracle.ball_query(host_pts, host_c[:1024], radius, S_)
            dt = time.perf_counter() - t0
            result["cpu_baseline"] = {"value": 1024 / dt, "unit": "queries/s", "cores": 1,
                                      "kind": "port",
                                      "sample": f"brute-force restatement, first 1024 centres, "
                                                f"{dt:.2f} s"}
    D.barrier(local)
    D.finalize()
    if result is not None:
        print(json.dumps(result), flush=True)
    return 0


def main():
    args = parse()
    if args.path == "group":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "path": "group",
                              "unavailable": "the reference has no ball query"}), flush=True)
            return 0
        return run_group(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
