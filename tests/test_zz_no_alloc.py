"""mflat_flat_search_noalloc: the allocation-free search entry point.

It exists for callers that cannot call cudaMalloc -- a serving process whose
device memory is already held by a framework's caching allocator, or a
latency-critical loop that cannot take the device-wide synchronisation of
cudaMalloc / cudaFree.  Its scratch is a fixed array inside the library, so
it is limited to 128 queries, dim <= 128 and k <= 21 per call.

Checked here through the C ABI:
  * two calls in a row (128 then 100 queries, so the second call starts from
    the first call's leftovers in the shared array) return the fp64 oracle's
    ids (outside 1e-6 relative near-ties) and distances (1e-5 relative), and
    the same as mflat_flat_search_device;
  * duplicated rows that defeat the exactness proof (the exact fallback scan,
    whose lists also live in the shared array), and fewer rows than k;
  * a first call on a fresh index leaves the device's free memory unchanged
    (a regular first search on a fresh index, by contrast, allocates);
  * sizes past the limits are rejected with MFLAT_ERR_BAD_ARG.
This file is collected last on purpose."""
import numpy as np
import pytest

import mflat_b200 as M
import oracle as O

pytestmark = pytest.mark.gpu

REL = 1e-5
METRIC = {"l2": O.L2, "ip": O.IP, "cosine": O.COSINE}


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _both(torch, idx, q_host, k, stream):
    """(noalloc ids, dist), (search_device ids, dist) for the same queries."""
    m = q_host.shape[0]
    q = _dev(torch, q_host)
    ref_i = torch.empty((m, k), dtype=torch.int32, device="cuda")
    ref_d = torch.empty((m, k), dtype=torch.float32, device="cuda")
    got_i = torch.full((m, k), -7, dtype=torch.int32, device="cuda")
    got_d = torch.full((m, k), -7.0, dtype=torch.float32, device="cuda")
    assert idx.search_noalloc(q.data_ptr(), m, k, got_i.data_ptr(), got_d.data_ptr(), stream) == k
    assert idx.search_device(q.data_ptr(), m, k, ref_i.data_ptr(), ref_d.data_ptr(), stream) == k
    torch.cuda.synchronize()
    return (got_i.cpu().numpy(), got_d.cpu().numpy()), (ref_i.cpu().numpy(), ref_d.cpu().numpy())


def _check(got, same, db, q, k, metric, what):
    gi, gd = got
    oi, od = O.flat_search_f64(db, q, k + 1, METRIC[metric])
    assert O.exact_ids_match(gi, gd, oi, od, rel=1e-6) == 0, what
    fin = np.isfinite(od[:, :k])
    assert np.array_equal(np.isfinite(gd), fin), what
    assert np.all(np.abs(gd[fin] - od[:, :k][fin]) <= REL * np.maximum(np.abs(od[:, :k][fin]), 1e-20)), what
    si, sd = same
    assert np.array_equal(gi, si), what
    fin = np.isfinite(sd)
    assert np.array_equal(gd[~fin], sd[~fin]), what
    assert np.all(np.abs(gd[fin] - sd[fin]) <= REL * np.maximum(np.abs(sd[fin]), 1e-20)), what


@pytest.mark.parametrize("metric,dim", [("l2", 128), ("ip", 64), ("cosine", 100)])
def test_noalloc_matches_oracle_twice(metric, dim):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(123 + dim)
    db = rng.standard_normal((50_000, dim)).astype(np.float32)
    idx = M.FlatIndex(dim, metric)
    idx.add(db)
    stream = torch.cuda.current_stream().cuda_stream
    k = 10
    for call, m in enumerate((128, 100)):
        q = rng.standard_normal((m, dim)).astype(np.float32)
        got, same = _both(torch, idx, q, k, stream)
        _check(got, same, db, q, k, metric, f"call {call}")
    idx.close()


def test_noalloc_fallback_scan_and_short_database():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(9)
    dim, k = 48, 21
    db = rng.standard_normal((20_000, dim)).astype(np.float32)
    db[1000:1060] = db[17]          # 61 equal rows: more than the 32 candidates
    q = rng.standard_normal((40, dim)).astype(np.float32)
    q[:10] = db[17] + np.float32(1e-3)
    idx = M.FlatIndex(dim, "l2")
    idx.add(db)
    stream = torch.cuda.current_stream().cuda_stream
    got, same = _both(torch, idx, q, k, stream)
    _check(got, same, db, q, k, "l2", "ties")
    idx.close()
    small = M.FlatIndex(dim, "ip")
    small.add(db[:5])
    got, same = _both(torch, small, q[:7], 10, stream)
    assert (got[0][:, 5:] == -1).all() and np.isneginf(got[1][:, 5:]).all()
    _check(got, same, db[:5], q[:7], 10, "ip", "n < k")
    small.close()


def test_noalloc_first_call_allocates_nothing():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(4)
    dim, m, k = 128, 128, 10
    db = rng.standard_normal((30_000, dim)).astype(np.float32)
    q_host = rng.standard_normal((m, dim)).astype(np.float32)
    stream = torch.cuda.current_stream().cuda_stream
    q = _dev(torch, q_host)
    ids = torch.empty((m, k), dtype=torch.int32, device="cuda")
    dist = torch.empty((m, k), dtype=torch.float32, device="cuda")
    # one call elsewhere first: the library's one-time set-up on this device
    warm = M.FlatIndex(dim, "l2")
    warm.add(db[:1000])
    warm.search_noalloc(q.data_ptr(), m, k, ids.data_ptr(), dist.data_ptr(), stream)
    torch.cuda.synchronize()

    fresh = M.FlatIndex(dim, "l2")
    fresh.add(db)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    assert fresh.search_noalloc(q.data_ptr(), m, k, ids.data_ptr(), dist.data_ptr(), stream) == k
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    assert free1 == free0, f"no-alloc call changed free device memory by {free0 - free1} bytes"
    oi, od = O.flat_search_f64(db, q_host, k + 1, O.L2)
    assert O.exact_ids_match(ids.cpu().numpy(), dist.cpu().numpy(), oi, od, rel=1e-6) == 0

    # control: the regular entry's first search on a fresh index takes scratch
    # (several MB for 8192 queries), which the same reading does see
    other = M.FlatIndex(dim, "l2")
    other.add(db)
    big_q = _dev(torch, rng.standard_normal((8192, dim)).astype(np.float32))
    big_i = torch.empty((8192, k), dtype=torch.int32, device="cuda")
    big_d = torch.empty((8192, k), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    free2 = torch.cuda.mem_get_info()[0]
    other.search_device(big_q.data_ptr(), 8192, k, big_i.data_ptr(), big_d.data_ptr(), stream)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] < free2
    for ix in (warm, fresh, other):
        ix.close()


def test_noalloc_rejects_sizes_past_the_limit():
    torch = pytest.importorskip("torch")
    idx = M.FlatIndex(32, "l2")
    idx.add(np.random.default_rng(1).standard_normal((1000, 32)).astype(np.float32))
    stream = torch.cuda.current_stream().cuda_stream
    q = torch.zeros((129, 32), dtype=torch.float32, device="cuda")
    ids = torch.empty((129, 32), dtype=torch.int32, device="cuda")
    dist = torch.empty((129, 32), dtype=torch.float32, device="cuda")
    with pytest.raises(M.MflatError) as e:
        idx.search_noalloc(q.data_ptr(), 129, 10, ids.data_ptr(), dist.data_ptr(), stream)
    assert e.value.status == 2
    with pytest.raises(M.MflatError) as e:
        idx.search_noalloc(q.data_ptr(), 8, 22, ids.data_ptr(), dist.data_ptr(), stream)
    assert e.value.status == 2
    wide = M.FlatIndex(129, "l2")
    wide.add(np.zeros((10, 129), np.float32))
    with pytest.raises(M.MflatError) as e:
        wide.search_noalloc(q.data_ptr(), 8, 10, ids.data_ptr(), dist.data_ptr(), stream)
    assert e.value.status == 2
