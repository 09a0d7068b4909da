"""Failure detection without a GPU fault: a screen launch whose bounded wait runs
out ends through its error path (error word set, copies and MMAs drained, TMEM
freed), the host reports MFLAT_ERR_DEVICE, and the same index serves the next
search correctly.

The stall is a test hook of the fp32 screen (MFLAT_TEST_STALL_SCREEN=1 at
index creation, one shot): its MMA warp first waits on a barrier that nothing
arrives at, with the wait limit shortened by MFLAT_WAIT_LIMIT_MS.  Nothing is
read or written out of bounds and no wait is unbounded.  The search that
follows the failed screen skips its select (the lists are not valid) and
returns the error instead of results."""
import time

import numpy as np
import pytest

import mflat_b200 as M
import oracle as O

pytestmark = pytest.mark.gpu


def _stalling_index(monkeypatch, dim, rows):
    monkeypatch.setenv("MFLAT_TEST_STALL_SCREEN", "1")
    monkeypatch.setenv("MFLAT_WAIT_LIMIT_MS", "50")
    idx = M.FlatIndex(dim, "l2")          # both variables are read at creation
    monkeypatch.delenv("MFLAT_TEST_STALL_SCREEN")
    monkeypatch.delenv("MFLAT_WAIT_LIMIT_MS")
    idx.add(rows)
    return idx


def test_wait_timeout_host_search(monkeypatch):
    rng = np.random.default_rng(31)
    db = rng.standard_normal((200_000, 64)).astype(np.float32)
    q = rng.standard_normal((300, 64)).astype(np.float32)
    idx = _stalling_index(monkeypatch, 64, db)
    t0 = time.time()
    with pytest.raises(M.MflatError) as e:
        idx.search(q, 10)
    assert e.value.status == 6                    # MFLAT_ERR_DEVICE
    assert time.time() - t0 < 30
    # the index works afterwards: exact results again
    ids, dist = idx.search(q, 10)
    ref_i, ref_d = O.flat_search_f64(db, q, 11, O.L2)
    assert O.exact_ids_match(ids, dist, ref_i, ref_d, rel=1e-6) == 0
    idx.close()


def test_wait_timeout_device_search_reported_by_next_call(monkeypatch):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(32)
    db = rng.standard_normal((100_000, 32)).astype(np.float32)
    q_host = rng.standard_normal((128, 32)).astype(np.float32)
    idx = _stalling_index(monkeypatch, 32, db)
    q = torch.from_numpy(q_host).cuda()
    ids = torch.empty((128, 5), dtype=torch.int32, device="cuda")
    dist = torch.empty((128, 5), dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    # device-pointer calls only enqueue: the failure surfaces at the next call
    idx.search_device(q.data_ptr(), 128, 5, ids.data_ptr(), dist.data_ptr(), st)
    torch.cuda.synchronize()
    with pytest.raises(M.MflatError) as e:
        idx.search_device(q.data_ptr(), 128, 5, ids.data_ptr(), dist.data_ptr(), st)
    assert e.value.status == 6
    idx.search_device(q.data_ptr(), 128, 5, ids.data_ptr(), dist.data_ptr(), st)
    torch.cuda.synchronize()
    ref_i, ref_d = O.flat_search_f64(db, q_host, 6, O.L2)
    assert O.exact_ids_match(ids.cpu().numpy(), dist.cpu().numpy(), ref_i, ref_d, rel=1e-6) == 0
    idx.close()
