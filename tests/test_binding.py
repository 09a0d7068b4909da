"""Host logic of the Python binding (metal-flat_b200/python/mflat_b200.py), on CPU.

The search wrapper's handling of caller-owned result buffers is exercised
against a stand-in for the C ABI that writes a known pattern, so no device is
needed; the real library is exercised by the GPU tests.
"""
import ctypes
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                "metal-flat_b200", "python"))
import mflat_b200 as M  # noqa: E402


class FakeLib:
    """mflat_flat_search stand-in: k_used = min(k, 7); ids = q*100 + j, dist = j / 2."""

    def __init__(self):
        self.calls = []

    def mflat_flat_search(self, h, q, m, k, ids, dist, used):
        ku = min(k, 7)
        self.calls.append((m, k, ctypes.addressof(ids.contents), ctypes.addressof(dist.contents)))
        for i in range(m):
            for j in range(ku):
                ids[i * ku + j] = i * 100 + j
                dist[i * ku + j] = j / 2
        used._obj.value = ku
        return 0

    def mflat_flat_free(self, h):
        pass


def fake_index():
    idx = M.FlatIndex.__new__(M.FlatIndex)
    idx._h, idx._lib, idx.metric = 1, FakeLib(), 0
    return idx


def expected(m, ku):
    return (np.arange(m)[:, None] * 100 + np.arange(ku)[None, :]).astype(np.int32), \
        np.tile(np.arange(ku, dtype=np.float32) / 2, (m, 1))


def test_search_allocates_and_packs_at_k_used():
    idx = fake_index()
    ids, dist = idx.search(np.zeros((3, 4), np.float32), 10)
    ei, ed = expected(3, 7)
    assert ids.shape == (3, 7) and np.array_equal(ids, ei) and np.array_equal(dist, ed)


def test_search_into_caller_buffers():
    idx = fake_index()
    out_i = np.full(5 * 10, -9, np.int32)
    out_d = np.full(5 * 10, -9, np.float32)
    ids, dist = idx.search(np.zeros((5, 4), np.float32), 10, out=(out_i, out_d))
    ei, ed = expected(5, 7)
    assert np.array_equal(ids, ei) and np.array_equal(dist, ed)
    assert np.shares_memory(ids, out_i) and np.shares_memory(dist, out_d)
    # the C ABI got the caller's buffers, and packed the results at stride k_used
    _, _, pi, pd = idx._lib.calls[-1]
    assert pi == out_i.ctypes.data and pd == out_d.ctypes.data
    assert np.all(out_i[5 * 7:] == -9)
    # reused on the next call
    idx.search(np.zeros((2, 4), np.float32), 3, out=(out_i, out_d))
    assert idx._lib.calls[-1][2] == out_i.ctypes.data
    assert np.array_equal(out_i[:6].reshape(2, 3), expected(2, 3)[0])


def test_search_accepts_two_dimensional_buffers():
    idx = fake_index()
    out_i = np.empty((4, 10), np.int32)
    out_d = np.empty((4, 10), np.float32)
    ids, _ = idx.search(np.zeros((4, 2), np.float32), 10, out=(out_i, out_d))
    assert ids.shape == (4, 7) and np.shares_memory(ids, out_i)


@pytest.mark.parametrize("bad", [
    (np.empty(49, np.int32), np.empty(50, np.float32)),         # too small
    (np.empty(50, np.int64), np.empty(50, np.float32)),         # wrong dtype
    (np.empty(50, np.int32), np.empty(50, np.float64)),
    (np.empty(100, np.int32)[::2], np.empty(50, np.float32)),   # not contiguous
    ([0] * 50, np.empty(50, np.float32)),                       # not an array
])
def test_search_rejects_unusable_buffers(bad):
    idx = fake_index()
    with pytest.raises(ValueError):
        idx.search(np.zeros((5, 4), np.float32), 10, out=bad)
    assert idx._lib.calls == []


def test_search_rejects_read_only_buffers():
    idx = fake_index()
    out_i = np.empty(50, np.int32)
    out_i.flags.writeable = False
    with pytest.raises(ValueError):
        idx.search(np.zeros((5, 4), np.float32), 10, out=(out_i, np.empty(50, np.float32)))


class FakeKmeansLib:
    """mflat_kmeans_assign stand-in: point i -> centroid i % c."""

    def mflat_kmeans_assign(self, p, n, c, nc, dim, out, device):
        for i in range(n):
            out[i] = i % nc
        return 0


def test_kmeans_assign_into_caller_buffer(monkeypatch):
    monkeypatch.setattr(M, "lib", lambda: FakeKmeansLib())
    pts = np.zeros((10, 3), np.float32)
    cen = np.zeros((4, 3), np.float32)
    got = M.kmeans_assign(pts, cen)
    assert np.array_equal(got, np.arange(10) % 4)
    buf = np.full(16, -1, np.int32)
    got = M.kmeans_assign(pts, cen, out=buf)
    assert got.shape == (10,) and np.shares_memory(got, buf)
    assert np.array_equal(buf[:10], np.arange(10) % 4) and np.all(buf[10:] == -1)
    with pytest.raises(ValueError):
        M.kmeans_assign(pts, cen, out=np.empty(9, np.int32))
    with pytest.raises(ValueError):
        M.kmeans_assign(pts, cen, out=np.empty(10, np.int64))
