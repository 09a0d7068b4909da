"""One rank of the sharded-search GPU test (launched by tests/test_gpu_shard.py
under torchrun).  Rank r holds rows [r*N/P, (r+1)*N/P) on GPU r; every rank
searches all queries collectively and rank 0 checks the merged global result
against the fp64 oracle."""
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
    for metric, n, dim, m, k in (("l2", 30011, 64, 300, 10), ("ip", 20000, 128, 129, 21),
                                 ("cosine", 5003, 33, 77, 7)):
        rng = np.random.default_rng(7 + dim)
        db = rng.standard_normal((n, dim)).astype(np.float32)
        db[n - 3] = db[5]                    # a duplicate that crosses shards
        q = rng.standard_normal((m, dim)).astype(np.float32)
        q[0] = db[5]
        lo, hi = rank * n // world, (rank + 1) * n // world
        idx = M.FlatIndex(dim, metric, device=local)
        idx.add(db[lo:hi])
        uid = [M.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        idx.set_shard(rank, world, uid[0], lo)
        ids, d = idx.search(q, k)
        # device-pointer variant too
        dq = torch.from_numpy(q).cuda()
        di = torch.empty((m, k), dtype=torch.int32, device="cuda")
        dd = torch.empty((m, k), dtype=torch.float32, device="cuda")
        idx.search_device(dq.data_ptr(), m, k, di.data_ptr(), dd.data_ptr(),
                          torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        same = np.array_equal(di.cpu().numpy(), ids)
        if rank == 0:
            ref_i, ref_d = O.flat_search_f64(db, q, k + 1, {"l2": 0, "ip": 1, "cosine": 2}[metric])
            bad = O.exact_ids_match(ids, d, ref_i, ref_d, rel=1e-6)
            err = np.max(np.abs(d - ref_d[:, :k]) / np.maximum(np.abs(ref_d[:, :k]), 1e-20))
            print(f"{metric}: bad ids {bad}, max rel dist err {err:.2e}, device api same {same}")
            if bad or err > 1e-5 or not same:
                rc = 1
        idx.close()
        dist.barrier()
    dist.destroy_process_group()
    sys.exit(rc)


if __name__ == "__main__":
    main()
