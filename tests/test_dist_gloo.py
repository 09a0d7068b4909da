"""Row-sharded search across two ranks, on the CPU with the gloo backend.

Each rank holds rows [r*N/P, (r+1)*N/P) (the split bench.py and
mflat_flat_set_shard use), computes its exact top-k with global ids, the ranks
all-gather the (id, distance) lists and merge them nearest-first / lowest id
first -- the same exchange the library runs over NCCL on GPUs.  The merged
result must equal the single-shard oracle exactly, including cross-shard ties.
A second test checks that a rank which dies before the exchange surfaces as an
error on the survivor (short process-group timeout) rather than a hang.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _data(metric):
    rng = np.random.default_rng(17)
    db = rng.standard_normal((1201, 24)).astype(np.float32)
    db[1000] = db[10]                        # duplicate across the shard boundary
    q = rng.standard_normal((13, 24)).astype(np.float32)
    q[0] = db[10]
    return db, q


def _rank_main(rank, world, port, metric, k, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    db, q = _data(metric)
    n = db.shape[0]
    lo, hi = rank * n // world, (rank + 1) * n // world
    ids, d = O.flat_search_f64(db[lo:hi], q, k, metric)
    ids = np.where(ids >= 0, ids + lo, -1).astype(np.int32)
    gi = [torch.empty(ids.shape, dtype=torch.int32) for _ in range(world)]
    gd = [torch.empty(d.shape, dtype=torch.float32) for _ in range(world)]
    dist.all_gather(gi, torch.from_numpy(ids))
    dist.all_gather(gd, torch.from_numpy(d))
    mi, md = O.merge_shards(np.stack([t.numpy() for t in gi]), np.stack([t.numpy() for t in gd]), metric)
    out[rank] = (mi, md)
    dist.destroy_process_group()


@pytest.mark.parametrize("metric", [O.L2, O.IP])
def test_two_rank_shard_merge_equals_single(metric):
    world, k = 2, 9
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_rank_main, args=(world, _free_port(), metric, k, out), nprocs=world, join=True)
    db, q = _data(metric)
    ref_i, ref_d = O.flat_search_f64(db, q, k, metric)
    for r in range(world):
        mi, md = out[r]
        assert np.array_equal(mi, ref_i)
        assert np.array_equal(md, ref_d)


def _dying_main(rank, world, port, out):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        os._exit(0)                           # leaves between steps, no exchange
    try:
        dist.all_gather([torch.empty(4) for _ in range(world)], torch.ones(4))
        out[rank] = "completed"
    except Exception as e:                    # noqa: BLE001 - any error is the point
        out[rank] = "error:" + type(e).__name__


def test_dead_rank_is_reported_not_hung():
    mgr = mp.Manager()
    out = mgr.dict()
    ctx = mp.start_processes(_dying_main, args=(2, _free_port(), out), nprocs=2, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=60)
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    assert out.get(0, "").startswith("error:")
