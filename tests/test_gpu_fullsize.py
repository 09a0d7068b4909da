"""Parity at the sizes the benchmark times (full size, the
same seeded data bench.py generates), through the C ABI on one B200:

  config 3  fp32 exact L2, 10M x 128 U[0,1), Q = 10,000, k = 10: the first 256
            queries of the timed batch have ids equal to the fp64 oracle's
            outside 1e-6 relative near-ties and distances within 1e-5;
  config 4  k-means step, 10M points x 65,536 centroids: every 100th point
            (100,000) is assigned bit-exactly like the sequential-fp32 oracle;
  config 5  bf16 L2, 100M x 128 N(0,1), Q = 16,384, k = 1024: recall@1024 of
            256 queries >= 0.99 against the exact oracle over the fp32 rows;
  config 2  fp16 IP, 1M x 768 normalised mixture, Q = 10,000, k = 100:
            recall@100 of 256 queries >= 0.99.

The oracle at these sizes is oracle/scale.py (screened, proven equal to the
plain oracle in tests/test_oracle_scale.py), fed block by block while the
index ingests the same blocks.
"""
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def _search_config(cfg_id):
    import torch
    import bench
    import mflat_b200 as M
    wl = bench.Workload(bench.CONFIGS[cfg_id])
    c = wl.cfg
    par = bench.Parity(wl, cfg_id, 0, 1, 0, wl.n, True)
    idx = M.FlatIndex(wl.dim, c["metric"], c["storage"], device=0)
    try:
        for a0, rows in wl.blocks(0, wl.n):
            idx.add(rows)
            par.feed(a0, rows)
        assert idx.size == wl.n
        # the whole query batch, as the benchmark times it
        d_q = torch.from_numpy(wl.queries()).cuda()
        d_ids = torch.empty((wl.nq, wl.k), dtype=torch.int32, device="cuda")
        d_dist = torch.empty((wl.nq, wl.k), dtype=torch.float32, device="cuda")
        idx.search_device(d_q.data_ptr(), wl.nq, wl.k, d_ids.data_ptr(), d_dist.data_ptr(),
                          torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        n = par.nchk
        res = par.check_search(None, d_ids[:n].cpu().numpy(), d_dist[:n].cpu().numpy())
        # every query of the batch got a full, sorted, duplicate-free list
        ids = d_ids.cpu().numpy()
        dist = d_dist.cpu().numpy()
    finally:
        idx.close()
    assert (ids >= 0).all() and (ids < wl.n).all()
    srt = np.sort(ids, axis=1)
    assert (np.diff(srt, axis=1) != 0).all()
    if c["metric"] == "l2":
        assert (np.diff(dist, axis=1) >= 0).all()
    else:
        assert (np.diff(dist, axis=1) <= 0).all()
    return res


def test_config3_full_size_exact_ids():
    res = _search_config(3)
    print(res)
    assert res["checked"] == 256
    assert res["bad_ids"] == 0 and res["max_rel_dist_err"] <= 1e-5, res


def test_config5_full_size_recall():
    res = _search_config(5)
    print(res)
    assert res["checked"] == 256 and res["recall"] >= 0.99, res


def test_config2_full_size_recall():
    res = _search_config(2)
    print(res)
    assert res["checked"] == 256 and res["recall"] >= 0.99, res


def test_config4_full_size_bit_exact_assignment():
    import bench
    import mflat_b200 as M
    wl = bench.Workload(bench.CONFIGS[4])
    par = bench.Parity(wl, 4, 0, 1, 0, wl.n, True)
    pts = wl.rows(0, wl.n)
    got = M.kmeans_assign(pts, wl.queries(), device=0)
    res = par.check_kmeans(None, pts, got)
    print(res)
    assert res["checked"] == 100_000 and res["mismatched"] == 0, res
