"""One rank of the dead-rank GPU test (tests/test_gpu_shard.py, 2 ranks under
torchrun, NCCL_NVLS_ENABLE=0, short MFLAT_NCCL_TIMEOUT_S).  Both ranks run one
sharded search; then rank 1 stops taking part between steps: nothing of it is in
flight (a host barrier follows the first step), and it neither searches again
nor tears down its communicator -- its process and its NCCL buffers stay alive,
so no peer ever touches freed memory.  Rank 0 runs the next search, whose
all-gather can no longer complete; the library's watchdog must abort the
communicator and return MFLAT_ERR_DEVICE within the timeout.  Rank 0 then
checks that the index answers for its own rows, writes the flag file named by
MFLAT_TEST_DONE_FLAG, and only then does rank 1 exit (bounded wait)."""
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
    flag = os.environ["MFLAT_TEST_DONE_FLAG"]
    if rank == 1:
        # stops taking part between steps; stays alive (communicator and its
        # buffers intact) until rank 0 has finished, at most 180 s
        print("rank 1 stopped taking part", flush=True)
        t_end = time.time() + 180.0
        while not os.path.exists(flag) and time.time() < t_end:
            time.sleep(0.2)
        os._exit(0)
    time.sleep(2.0)
    print("rank 0: second step starts", flush=True)
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
    with open(flag, "w") as f:
        f.write("done")
    os._exit(0 if (ok_first and status == 6 and took < 60 and local_ok) else 1)


if __name__ == "__main__":
    main()
