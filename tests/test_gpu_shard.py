"""Row-sharded exact search over NCCL on 2+ GPUs (one process per GPU), checked
against the fp64 oracle.  Skipped when fewer than two GPUs are visible."""
import os
import subprocess
import sys
import tempfile

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:                                  # noqa: BLE001
        return 0


@pytest.mark.skipif(_gpus() < 2, reason="needs at least two GPUs")
def test_sharded_search_matches_oracle():
    world = min(_gpus(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MFLAT_NCCL_TIMEOUT_S="120")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", "29533",
           os.path.join(ROOT, "tests", "shard_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0


@pytest.mark.skipif(_gpus() < 2, reason="needs at least two GPUs")
def test_dead_rank_reports_device_error():
    """Rank 1 stops taking part between steps (alive, its communicator intact);
    rank 0's next sharded search ends with MFLAT_ERR_DEVICE after the library's
    NCCL watchdog aborts the communicator (MFLAT_NCCL_TIMEOUT_S), instead of
    hanging.  NVLS off, plain NCCL."""
    flag = os.path.join(tempfile.mkdtemp(prefix="mflat_dead_rank_"), "rank0_done")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MFLAT_NCCL_TIMEOUT_S="5", MFLAT_TEST_DONE_FLAG=flag)
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", "29541",
           os.path.join(ROOT, "tests", "dead_rank_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert "second step status 6" in r.stdout
    assert "local search after abort ok True" in r.stdout
