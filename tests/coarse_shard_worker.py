"""One rank of the sharded k-means training GPU test (launched by
tests/test_gpu_coarse.py under torchrun).  Rank r holds a contiguous block of
the points on GPU r; all ranks train collectively and every rank checks its
centroids and global CSR against the oracle's sharded restatement."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "metal-flat_b200", "python"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import mflat_b200 as M  # noqa: E402
import oracle as O  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    rc = 0
    # (n, dim, nlist, iters): subsampled training, full training, many empty cells
    for n, dim, nlist, iters, dup in ((20000, 16, 50, 5, False), (3001, 40, 24, 4, False),
                                     (2500, 12, 32, 3, True)):
        rng = np.random.default_rng(n + dim)
        if dup:
            base = rng.standard_normal((10, dim)).astype(np.float32)
            data = base[rng.integers(0, 10, n)]
        else:
            centres = rng.standard_normal((max(4, nlist // 3), dim)).astype(np.float32)
            data = (centres[rng.integers(0, centres.shape[0], n)] +
                    0.3 * rng.standard_normal((n, dim))).astype(np.float32)
        offsets = np.array([r * n // world for r in range(world)] + [n], np.int64)
        lo, hi = offsets[rank], offsets[rank + 1]
        uid = [M.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        cq = M.CoarseQuantizer(dim, device=local)
        cq.set_shard(rank, world, uid[0], offsets)
        cq.train(data[lo:hi], nlist, iters)
        c = cq.centroids()
        s, r = cq.csr()
        c_ref, _, s_ref, r_ref = O.kmeans_train_sharded(data, nlist, iters, offsets)
        ok = (np.array_equal(c.view(np.uint32), c_ref.view(np.uint32)) and np.array_equal(s, s_ref)
              and np.array_equal(r, r_ref) and cq.size == n)
        q = data[:17] + 0.01
        cells = cq.probe(q, 3)
        ref_i, ref_d = O.flat_search_f64(c_ref, q, 4, O.L2)
        dd = ((q[:, None, :].astype(np.float64) - c_ref[cells].astype(np.float64)) ** 2).sum(-1)
        ok = ok and O.exact_ids_match(cells, dd.astype(np.float32), ref_i, ref_d, rel=1e-6) == 0
        print(f"rank {rank}: n={n} nlist={nlist} world={world} match={ok}", flush=True)
        if not ok:
            rc = 1
        cq.close()
        dist.barrier()
    dist.destroy_process_group()
    sys.exit(rc)


if __name__ == "__main__":
    main()
