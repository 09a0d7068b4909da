"""Benchmark of the exact flat-search hot path on B200 (one JSON line on stdout).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mflat|reference]
                  [--config 1..5]

Default workload = BASELINE config 3 (the north-star target): flat L2, fp32
exact (3 x bf16 split screen on the tensor cores + proof + fp64 re-rank),
database N = 10,000,000 x d = 128,
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
device-pointer C-ABI call on torch's stream, CUDA events; the library's
per-search timing events are only recorded during the loop and read after it,
so nothing waits on the host between steps); `e2e` = the same through the
host-pointer C-ABI call mflat_flat_search (pinned host queries in, results out
into pinned buffers reused across steps, copies inside the timed region).
N > 1 runs under torchrun: rank r holds rows [r*N/P, (r+1)*N/P), the library
all-gathers the per-rank top-k over NCCL and merges on the device.

Parity (outside the timed region): a subsample of the queries (config 4: of
the points) is checked against the exact oracle (oracle/scale.py: fp64 top-k,
ties to the lowest id; sequential-fp32 k-means argmin), which each rank feeds
with the rows it ingests; rank 0 merges the ranks' oracle pools and compares
with the search's own result, so every multi-GPU run also checks the NCCL
merge.  The line carries "parity": ids that differ outside 1e-6 relative
near-ties and the largest relative distance error (fp32 configs), recall@k
(16-bit configs), or mismatched assignments (config 4).

--impl reference times the CPU baseline (oracle/cpu_baseline.py: a
multithreaded BLAS sgemm + top-k brute force with the reference's semantics;
the reference's own search runs only on Apple Metal) on a sample of the same
workload's queries against the full database, on rank 0.
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
    3: dict(name="C3: flat L2 fp32 exact, N=10M x d=128, Q=10k, k=10, U[0,1)",
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

    def _block(self, b):
        return self._draw(np.random.default_rng([self.cfg["seed"], b]), BLOCK)

    def blocks(self, lo, hi, threads=None):
        """Yield (row0, rows) covering [lo, hi) in order, in pieces of at most
        BLOCK rows; the generator blocks are drawn on a thread pool ahead of
        the consumer (numpy's generators release the GIL)."""
        from concurrent.futures import ThreadPoolExecutor
        b0, b1 = lo // BLOCK, (hi + BLOCK - 1) // BLOCK
        threads = threads or min(16, os.cpu_count() or 1)
        if hi <= lo:
            return
        self.centres() if self.cfg["dist"] == "mixture" else None
        with ThreadPoolExecutor(threads) as ex:
            futs = {}
            nxt = b0
            for b in range(b0, b1):
                while nxt < b1 and nxt < b + threads:
                    futs[nxt] = ex.submit(self._block, nxt)
                    nxt += 1
                blk = futs.pop(b).result()
                a0, a1 = max(lo, b * BLOCK), min(hi, (b + 1) * BLOCK)
                yield a0, blk[a0 - b * BLOCK:a1 - b * BLOCK]

    def rows(self, lo, hi):
        """Database rows (or k-means points) [lo, hi)."""
        out = np.empty((max(0, hi - lo), self.dim), np.float32)
        for a0, r in self.blocks(lo, hi):
            out[a0 - lo:a0 - lo + r.shape[0]] = r
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


def profiled_traffic(cfg_id, kernel):
    """Per-launch DRAM bytes of `kernel` on this config from a committed ncu
    summary (None when no capture of this kernel exists)."""
    path = os.path.join(ROOT, "profiles", f"screen_traffic_c{cfg_id}.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        if d.get("kernel") == kernel:
            return d.get("dram_bytes_per_launch")
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
                        "config 3: 10.24 GB of screen planes)" if wl.n * wl.dim * 4 > 126e6
                        else "database fits L2 (config 1: 51 MB); no flush between steps",
            "parallelism": (f"row-shard x{world} + NCCL all-gather merge" if world > 1 else "1 GPU")
            if not c.get("kmeans") else (f"point-shard x{world}, no collective" if world > 1 else "1 GPU")}


ORACLE_METRIC = {"l2": 0, "ip": 1, "cosine": 2}
CPU_SAMPLE = {1: 1000, 2: 1000, 3: 1000, 4: 16384, 5: 256}   # queries (config 4: points)
PARITY_SAMPLE = {1: 1000, 2: 256, 3: 256, 4: 100, 5: 256}    # config 4: every 100th point


def cpu_baseline_run(wl, sample, warm=0):
    """Time the CPU brute force (all host threads) on `sample` queries (config 4:
    points) against the full database (centroid set).  Only the search itself
    is timed: the database blocks are generated (or drawn from memory) between
    the timed pieces.  Returns (seconds, algorithmic GFLOP)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import cpu_baseline as B
    c = wl.cfg
    if c.get("kmeans"):
        cents = wl.queries()
        pts = wl.rows(0, sample)
        if warm:
            B.kmeans_assign(pts[:warm], cents)
        t0 = time.perf_counter()
        B.kmeans_assign(pts, cents)
        dt = time.perf_counter() - t0
        return dt, 2.0 * sample * cents.shape[0] * wl.dim / 1e9
    metric = ORACLE_METRIC[c["metric"]]
    q = wl.queries()[:sample]
    if metric == 2:
        import oracle as O
        q = O.normalize_rows(q)
    topk = B.TopK(q, wl.k, 0 if metric == 0 else 1)
    dt = 0.0
    for a0, rows in wl.blocks(0, wl.n):
        if metric == 2:
            rows = O.normalize_rows(rows)
        if warm and a0 == 0:
            B.TopK(q[:warm], wl.k, 0 if metric == 0 else 1).add(rows[:65536], 0)
        for j in range(0, rows.shape[0], 65536):
            t0 = time.perf_counter()
            topk.add(rows[j:j + 65536], a0 + j)
            dt += time.perf_counter() - t0
    t0 = time.perf_counter()
    topk.result()
    dt += time.perf_counter() - t0
    return dt, 2.0 * sample * wl.n * wl.dim / 1e9


class ReferenceDB:
    """The full database held once in host memory for the reference arm's
    repeated steps (configs 1-4; config 5 streams its blocks instead)."""

    def __init__(self, wl):
        self.wl = wl
        self.db = None if wl.n > 20_000_000 or wl.cfg.get("kmeans") else wl.rows(0, wl.n)

    def step(self, sample, warm=False):
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import cpu_baseline as B
        wl = self.wl
        if self.db is None:
            return cpu_baseline_run(wl, sample)
        metric = ORACLE_METRIC[wl.cfg["metric"]]
        q = wl.queries()[:sample]
        db = self.db
        if metric == 2:
            import oracle as O
            q, db = O.normalize_rows(q), O.normalize_rows(db)
        t0 = time.perf_counter()
        B.search(db, q, wl.k, 0 if metric == 0 else 1)
        return time.perf_counter() - t0, 2.0 * sample * wl.n * wl.dim / 1e9


def run_reference(args, wl, cfg_id, rank, world):
    """CPU baseline arm: rank 0 only, a sample of the queries per step."""
    if rank != 0:
        return
    sample = args.ref_sample or CPU_SAMPLE[cfg_id]
    if not wl.cfg.get("kmeans"):
        sample = min(sample, wl.nq)
    ref = ReferenceDB(wl)
    for _ in range(args.warmup):      # warm-up steps: a small sample (untimed)
        ref.step(max(1, min(sample, 64)))
    times, gflop = [], 0.0
    for _ in range(args.steps):
        t, g = ref.step(sample)
        times.append(t)
        gflop = g
    tot = sum(times)
    value = sample * len(times) / tot
    unit = "queries/s" if not wl.cfg.get("kmeans") else "points/s"
    what = "points" if wl.cfg.get("kmeans") else "queries"
    cores = os.cpu_count() or 1
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * tot / len(times), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": f"synthetic (seed {wl.cfg['seed']})", "config": config_dict(wl, cfg_id, world),
        "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": "port",
                         "sample": f"{sample} {what} per step against the full "
                                   f"{'centroid set' if wl.cfg.get('kmeans') else 'database'} "
                                   "(BLAS sgemm + top-k, all host threads)",
                         "gflops": gflop * len(times) / tot},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's search path is Metal/MPS (Apple only): unavailable on this box; "
                "the timed baseline is the CPU port of its semantics",
    }
    print(json.dumps(line), flush=True)


class Parity:
    """Oracle side of the parity check, fed with the rows this rank ingests."""

    def __init__(self, wl, cfg_id, rank, world, lo, hi, enabled):
        self.enabled = enabled
        self.wl, self.cfg_id, self.rank, self.world = wl, cfg_id, rank, world
        self.lo, self.hi = lo, hi
        self.se = None
        if not enabled:
            return
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import scale as S
        self.S = S
        c = wl.cfg
        if c.get("kmeans"):
            self.stride = PARITY_SAMPLE[cfg_id]
        else:
            self.nchk = min(PARITY_SAMPLE[cfg_id], wl.nq)
            self.se = S.StreamingExact(wl.queries()[:self.nchk], wl.k, ORACLE_METRIC[c["metric"]])

    def feed(self, a0, rows):
        if self.se is not None:
            self.se.add(rows, a0)

    def check_search(self, dist, got_ids, got_dist):
        """Rank 0 compares got_* (first nchk queries) with the merged oracle."""
        if not self.enabled:
            return None
        import oracle as O
        pools = [self.se.pools()]
        if self.world > 1:
            gathered = [None] * self.world if self.rank == 0 else None
            dist.gather_object(self.se.pools(), gathered, dst=0)
            pools = gathered
        if self.rank != 0:
            return None
        ref_i, ref_d = self.se.result(self.S.merge_pools(pools))
        c = self.wl.cfg
        out = {"checked": int(self.nchk), "oracle": "exact fp64 top-k over the fp32 rows "
               "(oracle/scale.py: fp32 BLAS screen + proven margin + fp64 re-score)"}
        if c["storage"] == "fp32":
            bad = O.exact_ids_match(got_ids, got_dist, ref_i, ref_d, rel=1e-6)
            fin = np.isfinite(ref_d)
            rel = np.abs(got_dist[fin] - ref_d[fin]) / np.maximum(np.abs(ref_d[fin]), 1e-30)
            out.update(bad_ids=int(bad), max_rel_dist_err=float(rel.max()) if rel.size else 0.0,
                       criterion="ids equal outside 1e-6 relative near-ties; distances within 1e-5")
            out["ok"] = bool(bad == 0 and out["max_rel_dist_err"] <= 1e-5)
        else:
            hits = sum(len(np.intersect1d(got_ids[i], ref_i[i][ref_i[i] >= 0]))
                       for i in range(self.nchk))
            total = int((ref_i >= 0).sum())
            out.update(recall=hits / max(total, 1), criterion="recall@k >= 0.99")
            out["ok"] = bool(out["recall"] >= 0.99)
        return out

    def check_kmeans(self, dist, pts, got):
        """Every stride-th global point this rank holds; counts gathered to rank 0."""
        if not self.enabled:
            return None
        first = (self.lo + self.stride - 1) // self.stride * self.stride
        sel = np.arange(first, self.hi, self.stride) - self.lo
        ref = self.S.kmeans_assign_screened(pts[sel], self.wl.queries())
        counts = [int(sel.size), int((ref != got[sel]).sum())]
        if self.world > 1:
            t = __import__("torch").tensor(counts, dtype=__import__("torch").int64)
            dist.all_reduce(t)
            counts = [int(t[0]), int(t[1])]
        if self.rank != 0:
            return None
        return {"checked": counts[0], "mismatched": counts[1], "ok": counts[1] == 0,
                "oracle": "sequential fp32 sqL2 argmin, lowest index on ties "
                          "(oracle/scale.py kmeans_assign_screened)",
                "criterion": "assignments bit-exact"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mflat", choices=["mflat", "reference"])
    ap.add_argument("--config", type=int, default=3, choices=sorted(CONFIGS))
    ap.add_argument("--ref-sample", type=int, default=0,
                    help="reference arm: queries (config 4: points) per step (default: per config)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle check (profiling)")
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
    parity = Parity(wl, args.config, rank, world, lo, hi, not args.no_parity)

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
        for a0, rows in wl.blocks(lo, hi):
            idx.add(rows)
            parity.feed(a0, rows)
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

    # ---- device-resident timed region (value).  The library's timing events
    # are recorded per search and read after the loop (no host wait inside).
    if idx is not None:
        idx.set_timing(True)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        barrier()
    dev_s = max_over_ranks(ev0.elapsed_time(ev1) / 1000.0)
    value = units_per_step * args.steps / dev_s
    unit = "queries/s" if not kmeans else "points/s"
    if idx is not None:
        tsum, n_timed = idx.timing_sum()
        idx.set_timing(False)
        launches = tsum.launches
        screen_ms_mean = tsum.screen_ms / max(n_timed, 1)
        total_ms_mean = tsum.total_ms / max(n_timed, 1)
        fallback_queries = tsum.fallback_queries
    else:
        launches = 4 * args.steps
        fallback_queries = None

    # ---- parity of the timed search's own output (outside the timed region)
    if kmeans:
        par = parity.check_kmeans(dist, pts_h, d_out.cpu().numpy())
    else:
        nchk = parity.nchk if parity.enabled else 0
        par = parity.check_search(dist, d_ids[:nchk].cpu().numpy(), d_dist[:nchk].cpu().numpy())

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
    # fp32 storage: the distance GEMM runs as 3 bf16 products per element
    # (q_h x_h + q_l x_h + q_h x_l) at the bf16 tensor rate
    passes = 3.0 if fp32 else 1.0
    peak = bf16_peak
    kernel = "screen_kernel"
    if kmeans:
        flops = passes * 2.0 * n_local * qh.shape[0] * wl.dim
        t_s = dev_s / args.steps
        what = "whole assignment step (screen + exact re-check), CUDA events"
    else:
        flops = passes * 2.0 * wl.nq * n_local * wl.dim
        large = wl.k > (21 if fp32 else 16)
        t_s = (total_ms_mean if large else screen_ms_mean) / 1000.0
        what = ("whole search incl. floor pre-pass and select (large k)" if large
                else "screen kernel alone") + (", CUDA events on the launching stream, "
                                               f"mean over the {args.steps} timed searches")
    achieved = flops / t_s / 1e12
    # The screen streams its rows (the database, or the centroids for k-means)
    # once per launch: the bf16 planes (fp32 storage: two) plus 16 B of bias
    # parts per row.  With few query tiles that stream, not the tensor core,
    # bounds the launch; the line reports whichever bound is nearer.
    d_pad = (wl.dim + 63) // 64 * 64
    rows_streamed = qh.shape[0] if kmeans else n_local
    alg_bytes = rows_streamed * ((4 if fp32 else 2) * d_pad + 16)
    achieved_gbs = alg_bytes / t_s / 1e9
    # the committed DRAM capture belongs to the config's own workload only
    traffic = (profiled_traffic(args.config, kernel)
               if not (args.n_db or args.n_q or args.k) else None)
    flop_note = (f"{'3 bf16 products per element (fp32 split): 3 x ' if fp32 else ''}2*Q*N*d "
                 f"per launch (Q={wl.nq if not kmeans else n_local}, "
                 f"N={n_local if not kmeans else qh.shape[0]}, d={wl.dim})")
    byte_note = (f"algorithmic bytes = rows streamed x ({4 if fp32 else 2} x d_pad + 16) = "
                 f"{alg_bytes / 1e9:.3f} GB per launch")
    if achieved_gbs / hbm_peak > achieved / peak:
        roofline = {"bound": "hbm", "achieved": achieved_gbs, "peak": hbm_peak, "unit": "GB/s",
                    "frac": achieved_gbs / hbm_peak, "traffic": traffic, "kernel": kernel,
                    "note": (f"{byte_note}; peak = {src} HBM copy bandwidth = of {src}; "
                             f"time = {what}: {1000 * t_s:.3f} ms; tensor side {achieved:.1f} TFLOP/s "
                             f"= {achieved / peak:.3f} of {src} bf16 dense")}
    else:
        roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak, "traffic": traffic, "kernel": kernel,
                    "note": (f"{flop_note}; peak = {src} bf16 dense (kind::f16) = of {src}; "
                             f"time = {what}: {1000 * t_s:.3f} ms; {byte_note}")}

    line = {
        "metric": METRIC, "value": value, "unit": unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * dev_s / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32" if fp32 else c["storage"].replace("fp", "f"),
        "data": f"synthetic (BASELINE config {args.config}, seed {c['seed']})",
        "config": config_dict(wl, args.config, world), "roofline": roofline, "e2e": e2e,
        "gpu_launches": launches, "clocks": clk.summary(),
    }
    if par is not None:
        line["parity"] = par
    if fallback_queries is not None:
        line["fallback_queries"] = fallback_queries
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        sample = CPU_SAMPLE[args.config] if kmeans else min(CPU_SAMPLE[args.config], wl.nq)
        t, gflop = cpu_baseline_run(wl, sample, warm=8)
        line["cpu_baseline"] = {
            "value": sample / t, "unit": unit, "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"{sample} {'points' if kmeans else 'queries'} against the full "
                      f"{'centroid set' if kmeans else 'database'} (BLAS sgemm + top-k, "
                      "all host threads), scaled to per-second",
            "gflops": gflop / t}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if idx is not None:
        idx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
