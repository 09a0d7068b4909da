"""mflat_flat_search_noalloc: the allocation-free search entry point.

It exists for callers that cannot call cudaMalloc -- a serving process whose
device memory is already held by a framework's caching allocator, or a
latency-critical loop that cannot take the device-wide synchronisation of
cudaMalloc / cudaFree.  Its scratch is a fixed array inside the library, so
it is limited to 128 queries, dim <= 128 and k <= 21 per call.

Checked here through the C ABI: two calls in a row (different queries, so the
second call starts from the first call's leftovers in the shared array) give
the same results as mflat_flat_search_device, and sizes past the limits are
rejected with MFLAT_ERR_BAD_ARG.  This file is collected last on purpose."""
import numpy as np
import pytest

import mflat_b200 as M

pytestmark = pytest.mark.gpu

REL = 1e-5


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("metric,dim", [("l2", 128), ("ip", 64), ("cosine", 100)])
def test_noalloc_matches_search_device_twice(metric, dim):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(123 + dim)
    db = rng.standard_normal((50_000, dim)).astype(np.float32)
    idx = M.FlatIndex(dim, metric)
    idx.add(db)
    stream = torch.cuda.current_stream().cuda_stream
    k = 10
    for call in range(2):
        m = 100 if call == 0 else 128
        q = _dev(torch, rng.standard_normal((m, dim)).astype(np.float32))
        ref_i = torch.empty((m, k), dtype=torch.int32, device="cuda")
        ref_d = torch.empty((m, k), dtype=torch.float32, device="cuda")
        got_i = torch.full((m, k), -7, dtype=torch.int32, device="cuda")
        got_d = torch.full((m, k), -7.0, dtype=torch.float32, device="cuda")
        assert idx.search_device(q.data_ptr(), m, k, ref_i.data_ptr(), ref_d.data_ptr(), stream) == k
        assert idx.search_noalloc(q.data_ptr(), m, k, got_i.data_ptr(), got_d.data_ptr(), stream) == k
        torch.cuda.synchronize()
        gi, gd = got_i.cpu().numpy(), got_d.cpu().numpy()
        ri, rd = ref_i.cpu().numpy(), ref_d.cpu().numpy()
        assert np.array_equal(gi, ri), f"call {call}"
        assert np.all(np.abs(gd - rd) <= REL * np.maximum(np.abs(rd), 1e-20)), f"call {call}"


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
