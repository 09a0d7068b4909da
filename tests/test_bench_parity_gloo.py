"""bench.py's parity leg across ranks, on the CPU with gloo (world size 2).

Each rank feeds the screened oracle (oracle/scale.py) with only the rows of its
shard, exactly as a multi-GPU bench run does while ingesting; rank 0 gathers the
ranks' pools and compares a search result with the merged oracle.  Here the
"search result" is the plain fp64 oracle over all rows, so the check must pass
with no bad ids; a result with one id swapped must be caught.  The k-means leg
sums the per-rank counts of checked and mismatched points.
"""
import os
import socket
import sys

import numpy as np
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, out):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import bench
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    res = {}
    # config 3 semantics (L2, U[0,1)), shrunk: 30k rows, 300 queries (256 checked)
    wl = bench.Workload(bench.CONFIGS[3], 30_000, 300)
    lo, hi = rank * wl.n // world, (rank + 1) * wl.n // world
    par = bench.Parity(wl, 3, rank, world, lo, hi, True)
    for a0, rows in wl.blocks(lo, hi):
        par.feed(a0, rows)
    db = wl.rows(0, wl.n)
    q = wl.queries()[: par.nchk]
    ids, d = O.flat_search_f64(db, q, wl.k, O.L2)
    res["good"] = par.check_search(dist, ids, d)
    bad = ids.copy()
    bad[3, 0], bad[3, 1] = bad[3, 1], bad[3, 0]        # a swapped pair, not a near-tie
    res["bad"] = par.check_search(dist, bad, d)
    # config 4 semantics, shrunk: 20k points against the 65,536 centroids
    wk = bench.Workload(bench.CONFIGS[4], 20_000)
    lo, hi = rank * wk.n // world, (rank + 1) * wk.n // world
    pk = bench.Parity(wk, 4, rank, world, lo, hi, True)
    pts = wk.rows(lo, hi)
    got = O.kmeans_assign_f32(pts, wk.queries())
    res["kmeans"] = pk.check_kmeans(dist, pts, got)
    out[rank] = res
    dist.destroy_process_group()


def test_parity_leg_two_ranks():
    world = 2
    with mp.Manager() as man:
        out = man.dict()
        mp.spawn(_rank_main, args=(world, _free_port(), out), nprocs=world, join=True)
        r0, r1 = out[0], out[1]
    assert r1["good"] is None and r1["kmeans"] is None      # rank 0 reports
    assert r0["good"]["checked"] == 256 and r0["good"]["bad_ids"] == 0 and r0["good"]["ok"]
    assert r0["bad"]["bad_ids"] >= 1 and not r0["bad"]["ok"]
    assert r0["kmeans"]["checked"] == 200 and r0["kmeans"]["mismatched"] == 0
