"""Benchmark of the exact flat-search hot path on B200 (one JSON line on stdout).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mflat|reference]
                  [--config 1..5]

Default workload = BASELINE config 3 (the north-star target): flat L2, fp32
exact (3xTF32 screen + fp64 re-rank), database N = 10,000,000 x d = 128,
Q = 10,000 queries, k = 10, values uniform [0,1) from seed 1, row-sharded
across the ranks.  One step = one search of all Q queries.  The other BASELINE
configs are available with --config (parity cases elsewhere; measured here for
the record):
  1  L2 fp32, N = 100k x 128, Q = 1000, k = 10, N(0,1) seed 0
  2  IP fp16, N = 1M x 768, Q = 10k, k = 100, 1000-component mixture
     (centres N(0,1), sigma 0.3, L2-normalised), seed 3
  4  k-means assignment step: 10M points x 128 from a 65,536-component mixture
     (centres N(0,1), sigma 0.3), centroids = centres + N(0, 0.05), seed 4;
     sharded by points; unit = points assigned / s
  5  L2 bf16, N = 100M x 128, Q = 16,384, k = 1024, N(0,1) seed 2
Seeded synthetic data (no public dataset is used): database row block b of 1M
rows comes from np.random.default_rng([seed, b]), queries from
np.random.default_rng([seed, 10**6]), mixture centres from
np.random.default_rng([seed, 10**7]).

Timing: `value` = Q*K / max-over-ranks device time (queries already in HBM;
device-pointer C-ABI call on torch's stream, CUDA events); `e2e` = the same
through the host-pointer C-ABI call mflat_flat_search (pinned host queries in,
results out into pinned buffers reused across steps, copies inside the timed
region).  N > 1 runs under torchrun: rank
r holds rows [r*N/P, (r+1)*N/P), the library all-gathers the per-rank top-k
over NCCL and merges on the device.  --impl reference times the CPU baseline
(oracle/cpu_baseline.py: multithreaded BLAS sgemm + partial top-k with the
reference's semantics; the reference's own search runs only on Apple Metal)
on a bounded query sample of the same workload.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "metal-flat_b200", "python"))

METRIC = "exact flat top-k queries/sec at 1/2/4/8 B200; % of GEMM/HBM roofline"
BLOCK = 1_000_000

CONFIGS = {
    1: dict(name="C1: flat L2 fp32 exact, N=100k x d=128, Q=1000, k=10, N(0,1)", n=100_000,
            dim=128, q=1000, k=10, metric="l2", storage="fp32", seed=0, dist="normal"),
    2: dict(name="C2: flat IP fp16, N=1M x d=768, Q=10k, k=100, 1000-comp mixture, normalised",
            n=1_000_000, dim=768, q=10_000, k=100, metric="ip", storage="fp16", seed=3,
            dist="mixture", comps=1000, sigma=0.3, normalise=True),
    3: dict(name="C3: flat L2 fp32 exact (3xTF32 screen + fp64 re-rank), N=10M x d=128, Q=10k, k=10",
            n=10_000_000, dim=128, q=10_000, k=10, metric="l2", storage="fp32", seed=1,
            dist="uniform"),
    4: dict(name="C4: k-means assignment step, 10M points x 128, 65,536 centroids, top-1 L2 bit-exact",
            n=10_000_000, dim=128, q=65_536, k=1, metric="l2", storage="fp32", seed=4,
            dist="mixture", comps=65_536, sigma=0.3, normalise=False, kmeans=True),
    5: dict(name="C5: flat L2 bf16, N=100M x d=128, Q=16,384, k=1024", n=100_000_000, dim=128,
            q=16_384, k=1024, metric="l2", storage="bf16", seed=2, dist="normal"),
}


class Workload:
    def __init__(self, cfg, n_override=None, q_override=None):
        self.cfg = dict(cfg)
        if n_override:
            self.cfg["n"] = n_override
        if q_override:
            self.cfg["q"] = q_override
        c = self.cfg
        self.n, self.dim, self.nq, self.k = c["n"], c["dim"], c["q"], c["k"]
        self._centres = None

    def centres(self):
        if self._centres is None:
            c = self.cfg
            self._centres = np.random.default_rng([c["seed"], 10**7]).standard_normal(
                (c["comps"], self.dim), dtype=np.float32)
        return self._centres

    def _draw(self, rng, rows):
        c = self.cfg
        if c["dist"] == "uniform":
            return rng.random((rows, self.dim), dtype=np.float32)
        if c["dist"] == "normal":
            return rng.standard_normal((rows, self.dim), dtype=np.float32)
        comp = rng.integers(0, c["comps"], size=rows)
        x = self.centres()[comp] + np.float32(c["sigma"]) * rng.standard_normal(
            (rows, self.dim), dtype=np.float32)
        if c.get("normalise"):
            x /= np.linalg.norm(x, axis=1, keepdims=True)
        return x.astype(np.float32, copy=False)

    def rows(self, lo, hi):
        """Database rows (or k-means points) [lo, hi)."""
        out = np.empty((hi - lo, self.dim), np.float32)
        b = lo // BLOCK
        while b * BLOCK < hi:
            blk = self._draw(np.random.default_rng([self.cfg["seed"], b]), BLOCK)
            a0, a1 = max(lo, b * BLOCK), min(hi, (b + 1) * BLOCK)
            out[a0 - lo:a1 - lo] = blk[a0 - b * BLOCK:a1 - b * BLOCK]
            b += 1
        return out

    def queries(self):
        """Queries, or for k-means the centroids (centres + N(0, 0.05))."""
        c = self.cfg
        rng = np.random.default_rng([c["seed"], 10**6])
        if c.get("kmeans"):
            return (self.centres() + np.float32(0.05) * rng.standard_normal(
                self.centres().shape, dtype=np.float32)).astype(np.float32)
        return self._draw(rng, self.nq)


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p.get("bf16_tflops"), p.get("hbm_gbs"), "measured"
    return 1590.0, 6650.0, "fallback"


def profiled_traffic(cfg_id):
    """Per-launch DRAM bytes of the screen kernel from a committed ncu summary."""
    path = os.path.join(ROOT, "profiles", f"screen_traffic_c{cfg_id}.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f).get("dram_bytes_per_launch")
    return None


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def config_dict(wl, cfg_id, world):
    c = wl.cfg
    return {"workload": c["name"], "config_id": cfg_id, "n": wl.n, "dim": wl.dim,
            "queries": wl.nq, "k": wl.k, "metric": c["metric"], "storage": c["storage"],
            "global_batch": wl.nq if not c.get("kmeans") else wl.n,
            "l2_flush": "inputs larger than L2 (database >= 51 MB streamed per step; "
                        "config 3: 10.24 GB hi/lo planes)" if wl.n * wl.dim * 4 > 126e6
                        else "database fits L2 (config 1: 51 MB); no flush between steps",
            "parallelism": (f"row-shard x{world} + NCCL all-gather merge" if world > 1 else "1 GPU")
            if not c.get("kmeans") else (f"point-shard x{world}, no collective" if world > 1 else "1 GPU")}


def cpu_metric(c):
    from_metric = {"l2": 0, "ip": 1}
    return from_metric[c["metric"]]


def cpu_baseline_run(wl, sample, repeats=1):
    """Time the CPU port on `sample` queries (or k-means points) against the full data."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import cpu_baseline as B
    c = wl.cfg
    db = wl.rows(0, wl.n) if not c.get("kmeans") else wl.queries()
    q = wl.queries()[:sample] if not c.get("kmeans") else wl.rows(0, sample)
    metric = cpu_metric(c)
    dn = np.einsum("ij,ij->i", db, db, dtype=np.float64).astype(np.float32) if metric == 0 else None
    B.search(db, q[:max(1, sample // 8)], wl.k, metric, dnorm=dn)
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        B.search(db, q, wl.k, metric, dnorm=dn)
        times.append(time.perf_counter() - t0)
    return times


def run_reference(args, wl, cfg_id, rank, world):
    """CPU baseline arm: rank 0 only, a bounded query sample per step."""
    if rank != 0:
        return
    sample = args.ref_sample
    times = cpu_baseline_run(wl, sample, repeats=args.steps + args.warmup)[args.warmup:]
    tot = sum(times)
    value = sample * len(times) / tot
    unit = "queries/s" if not wl.cfg.get("kmeans") else "points/s"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * tot / len(times), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": f"synthetic (seed {wl.cfg['seed']})", "config": config_dict(wl, cfg_id, world),
        "cpu_baseline": {"value": value, "unit": unit, "cores": os.cpu_count() or 1, "kind": "port",
                         "sample": f"{sample} queries per step against the full database "
                                   "(BLAS sgemm + partial top-k, all host threads)"},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's search path is Metal/MPS (Apple only): unavailable on this box; "
                "the timed baseline is the CPU port of its semantics",
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mflat", choices=["mflat", "reference"])
    ap.add_argument("--config", type=int, default=3, choices=sorted(CONFIGS))
    ap.add_argument("--ref-sample", type=int, default=32)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--n-db", type=int, default=None,
                    help="profiling only: smaller database (rows) for ncu captures")
    ap.add_argument("--n-q", type=int, default=None, help="profiling only: fewer queries")
    ap.add_argument("--k", type=int, default=None, help="profiling only: other k")
    args = ap.parse_args()
    wl = Workload(CONFIGS[args.config], args.n_db, args.n_q)
    if args.k:
        wl.k = wl.cfg["k"] = args.k
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, wl, args.config, rank, world)
        return

    import torch
    import torch.distributed as dist
    import mflat_b200 as M

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=900))
    c = wl.cfg
    kmeans = bool(c.get("kmeans"))
    lo, hi = rank * wl.n // world, (rank + 1) * wl.n // world
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world > 1:
            t = torch.tensor([x], dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t[0])
        return x

    qh = wl.queries()
    if kmeans:
        pts_h = wl.rows(lo, hi)
        d_pts = torch.from_numpy(pts_h).cuda()
        d_cent = torch.from_numpy(qh).cuda()
        d_out = torch.empty(hi - lo, dtype=torch.int32, device="cuda")
        L = M.lib()

        def step():
            st = L.mflat_kmeans_assign_device(d_pts.data_ptr(), hi - lo, d_cent.data_ptr(),
                                              qh.shape[0], wl.dim, d_out.data_ptr(), local, sp)
            if st != 0:
                raise M.MflatError(st, "kmeans_assign_device")
        units_per_step, idx = wl.n, None
    else:
        idx = M.FlatIndex(wl.dim, c["metric"], c["storage"], device=local)
        for a in range(lo, hi, BLOCK):
            idx.add(wl.rows(a, min(hi, a + BLOCK)))
        if world > 1:
            obj = [M.comm_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(obj, src=0)
            idx.set_shard(rank, world, obj[0], lo)
        d_q = torch.from_numpy(qh).cuda()
        d_ids = torch.empty((wl.nq, wl.k), dtype=torch.int32, device="cuda")
        d_dist = torch.empty((wl.nq, wl.k), dtype=torch.float32, device="cuda")

        def step():
            idx.search_device(d_q.data_ptr(), wl.nq, wl.k, d_ids.data_ptr(), d_dist.data_ptr(), sp)
        units_per_step = wl.nq

    for _ in range(max(3, args.warmup)):
        step()
    barrier()

    # ---- device-resident timed region (value) with live per-kernel timing
    if idx is not None:
        idx.set_timing(True)
    screen_ms, total_ms, launches = [], [], 0
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        ev0.record(stream)
        for _ in range(args.steps):
            step()
            if idx is not None:
                t = idx.last_timing()
                screen_ms.append(t.screen_ms)
                total_ms.append(t.total_ms)
                launches += t.launches
            else:
                launches += 4
        ev1.record(stream)
        barrier()
    if idx is not None:
        idx.set_timing(False)
    dev_s = max_over_ranks(ev0.elapsed_time(ev1) / 1000.0)
    value = units_per_step * args.steps / dev_s
    unit = "queries/s" if not kmeans else "points/s"

    # ---- end-to-end through the host-pointer C ABI (pinned host buffers)
    barrier()
    if kmeans:
        pts_p = torch.from_numpy(pts_h).pin_memory().numpy()
        cent_p = torch.from_numpy(qh).pin_memory().numpy()
        asg_p = torch.empty(pts_p.shape[0], dtype=torch.int32, pin_memory=True).numpy()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            out = M.kmeans_assign(pts_p, cent_p, device=local, out=asg_p)
        barrier()
        e2e_s = max_over_ranks(time.perf_counter() - t0)
        e2e = {"value": wl.n * args.steps / e2e_s, "unit": unit,
               "h2d_bytes_per_step": int(pts_p.nbytes + cent_p.nbytes),
               "d2h_bytes_per_step": int(out.nbytes)}
    else:
        qp = torch.from_numpy(qh).pin_memory().numpy()
        # result buffers: page-locked and reused across steps, as a serving
        # caller would hold them (the C ABI writes into caller-owned buffers)
        ids_p = torch.empty(wl.nq * wl.k, dtype=torch.int32, pin_memory=True).numpy()
        dist_p = torch.empty(wl.nq * wl.k, dtype=torch.float32, pin_memory=True).numpy()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            ids_h, dist_h = idx.search(qp, wl.k, out=(ids_p, dist_p))
        barrier()
        e2e_s = max_over_ranks(time.perf_counter() - t0)
        e2e = {"value": wl.nq * args.steps / e2e_s, "unit": unit,
               "h2d_bytes_per_step": int(qp.nbytes),
               "d2h_bytes_per_step": int(ids_h.nbytes + dist_h.nbytes)}

    # ---- roofline of the dominant kernel on this rank
    bf16_peak, hbm_peak, src = measured_peaks()
    n_local = hi - lo
    fp32 = c["storage"] == "fp32"
    passes = 3.0 if fp32 else 1.0
    peak = bf16_peak / 2.0 if fp32 else bf16_peak
    if kmeans:
        flops = passes * 2.0 * n_local * qh.shape[0] * wl.dim
        t_s = dev_s / args.steps
        what = "whole assignment step (screen + exact re-check), CUDA events"
    else:
        flops = passes * 2.0 * wl.nq * n_local * wl.dim
        large = wl.k > (21 if fp32 else 16)
        t_s = statistics.mean(total_ms if large else screen_ms) / 1000.0
        what = ("whole search incl. floor pre-pass and select (large k)" if large
                else "screen kernel alone") + ", CUDA events on the launching stream"
    achieved = flops / t_s / 1e12
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "traffic": profiled_traffic(args.config),
                "kernel": "screen_tf32x3_kernel" if fp32 else "screen_f16_kernel",
                "note": (f"{'tf32-equivalent: 3 x ' if fp32 else ''}2*Q*N*d per launch "
                         f"(Q={wl.nq if not kmeans else n_local}, N={n_local if not kmeans else qh.shape[0]}, "
                         f"d={wl.dim}); peak = {src} bf16 dense{' / 2 (kind::tf32 rate)' if fp32 else ''}"
                         f" = of {src}; time = {what}: {1000 * t_s:.3f} ms")}

    line = {
        "metric": METRIC, "value": value, "unit": unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * dev_s / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32" if fp32 else c["storage"].replace("fp", "f"),
        "data": f"synthetic (BASELINE config {args.config}, seed {c['seed']})",
        "config": config_dict(wl, args.config, world), "roofline": roofline, "e2e": e2e,
        "gpu_launches": launches, "clocks": clk.summary(),
    }
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        sample = {1: 64, 2: 16, 3: 64, 4: 20000, 5: 4}[args.config]
        t = cpu_baseline_run(wl, sample)[0]
        line["cpu_baseline"] = {
            "value": sample / t, "unit": unit, "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"{sample} {'points' if kmeans else 'queries'} against the full "
                      f"{'centroid set' if kmeans else 'database'} (BLAS sgemm + partial top-k, "
                      "all host threads), scaled to per-second"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if idx is not None:
        idx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
