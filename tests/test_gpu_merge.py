"""The on-device merge of a sharded search (comm.cu merge_ranks_kernel), run on
one GPU through mflat_cu_merge_ranks on synthetic gathered lists and compared
bit for bit with the oracle's merge (oracle.merge_shards): nearer first, then
lower id, including ties across shards, padded (short) lists, rank counts that
are not powers of two and k up to 1024."""
import ctypes

import numpy as np
import pytest

import mflat_b200 as M
import oracle as O

pytestmark = pytest.mark.gpu


def _lib():
    L = ctypes.CDLL(M.CUDA_LIB_PATH)
    vp, ci = ctypes.c_void_p, ctypes.c_int
    L.mflat_cu_merge_ranks.argtypes = [vp, vp, ci, ci, ci, ci, vp, vp, vp]
    L.mflat_cu_merge_ranks.restype = ci
    return L


def make_lists(rng, world, m, k, metric, short_every=3):
    """Per-rank sorted lists with global ids (rank r owns ids r, r+world, ...)
    and planted cross-shard ties."""
    ids = np.full((world, m, k), -1, np.int32)
    dist = np.full((world, m, k), np.inf if metric == O.L2 else -np.inf, np.float32)
    for p in range(world):
        for q in range(m):
            n = k if (q + p) % short_every else max(0, k - 1 - (q % (k + 1)))
            d = rng.integers(0, 4 * k + 8, size=n).astype(np.float32) * np.float32(0.25)
            gid = (rng.choice(max(4 * k, n + 1), size=n, replace=False) * world + p).astype(np.int32)
            order = np.lexsort((gid, d if metric == O.L2 else -d))
            ids[p, q, :n] = gid[order]
            dist[p, q, :n] = d[order]
    return ids, dist


@pytest.mark.parametrize("world,k", [(2, 10), (3, 7), (5, 100), (8, 10), (8, 1024), (16, 64), (1, 5)])
@pytest.mark.parametrize("metric", [O.L2, O.IP])
def test_merge_matches_oracle(world, k, metric):
    import torch
    rng = np.random.default_rng(world * 1000 + k + metric)
    m = 37
    ids, dist = make_lists(rng, world, m, k, metric)
    ref_i, ref_d = O.merge_shards(ids, dist, metric)
    gi = torch.from_numpy(ids).cuda()
    gd = torch.from_numpy(dist).cuda()
    oi = torch.full((m, k), 7, dtype=torch.int32, device="cuda")
    od = torch.zeros((m, k), dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = _lib().mflat_cu_merge_ranks(gi.data_ptr(), gd.data_ptr(), world, m, k, metric,
                                     oi.data_ptr(), od.data_ptr(), st)
    assert rc == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(oi.cpu().numpy(), ref_i)
    np.testing.assert_array_equal(od.cpu().numpy(), ref_d)


def test_merge_rejects_oversized_fan_in():
    import torch
    gi = torch.zeros(1, dtype=torch.int32, device="cuda")
    gd = torch.zeros(1, dtype=torch.float32, device="cuda")
    # 64 ranks x k = 1024 needs 768 KB of shared memory: refused, nothing launched
    assert _lib().mflat_cu_merge_ranks(gi.data_ptr(), gd.data_ptr(), 64, 1, 1024, 0,
                                       gi.data_ptr(), gd.data_ptr(), None) != 0
