"""One rank of the dead-rank GPU test (tests/test_gpu_shard.py, 2 ranks under
torchrun, NCCL_NVLS_ENABLE=0, short MFLAT_NCCL_TIMEOUT_S).  Both ranks run one
sharded search; then rank 1 leaves between steps (nothing of it in flight:
its index and communicator are closed after a host barrier) and rank 0 runs
the next search, whose all-gather can no longer complete.  The library's
watchdog must abort the communicator and return MFLAT_ERR_DEVICE within the
timeout; rank 0 prints the outcome and exits without further collectives."""
import datetime
import os
import sys
import time

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "metal-flat_b200", "python"))

import mflat_b200 as M  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    rng = np.random.default_rng(5)
    n, dim = 20000, 32
    db = rng.standard_normal((n, dim)).astype(np.float32)
    q = rng.standard_normal((64, dim)).astype(np.float32)
    lo, hi = rank * n // world, (rank + 1) * n // world
    idx = M.FlatIndex(dim, "l2", device=torch.cuda.current_device())
    idx.add(db[lo:hi])
    uid = [M.comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    idx.set_shard(rank, world, uid[0], lo)
    ids, _ = idx.search(q, 5)                  # a healthy collective step
    ok_first = bool((ids >= 0).all())
    dist.barrier()                             # everything of step 1 has completed
    if rank == 1:
        idx.close()                            # leaves between steps
        print("rank 1 left", flush=True)
        os._exit(0)
    time.sleep(2.0)
    t0 = time.time()
    try:
        idx.search(q, 5)
        status = 0
    except M.MflatError as e:
        status = e.status
    took = time.time() - t0
    print(f"rank 0: first step ok {ok_first}, second step status {status} after {took:.1f} s",
          flush=True)
    # after the abort the index is local again and still answers
    ids2, _ = idx.search(q, 5)
    local_ok = bool((ids2 >= lo).all() and (ids2 < hi).all())
    print(f"rank 0: local search after abort ok {local_ok}", flush=True)
    idx.close()
    os._exit(0 if (ok_first and status == 6 and took < 60 and local_ok) else 1)


if __name__ == "__main__":
    main()
