"""ctypes wrapper over oracle/_ref/libmflat_oracle.so.

TEST INFRASTRUCTURE ONLY: the checker for tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline legs.  The product library never imports this module.
Semantics are documented in oracle/mflat_oracle.h (restating the reference's
src/Distance.h, src/FlatIndex.mm cpuSearch and src/CoarseQuantizer.mm).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
L2, IP, COSINE = 0, 1, 2

_lib = None


def build() -> None:
    """Compile the oracle (and, where the reference tree exists, its goldens lib)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = os.path.join(REF_DIR, "libmflat_oracle.so")
        if not os.path.exists(path):
            build()
        _lib = ctypes.CDLL(path)
        f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
        i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
        i64 = ctypes.c_int64
        ci = ctypes.c_int
        _lib.mfo_row_sq_norms.argtypes = [f32p, i64, ci, f32p]
        _lib.mfo_normalize_rows.argtypes = [f32p, i64, ci]
        _lib.mfo_sq_l2_f32.argtypes = [f32p, f32p, ci]
        _lib.mfo_sq_l2_f32.restype = ctypes.c_float
        _lib.mfo_dot_f32.argtypes = [f32p, f32p, ci]
        _lib.mfo_dot_f32.restype = ctypes.c_float
        for fn in (_lib.mfo_flat_search_f64, _lib.mfo_flat_search_cpusearch):
            fn.argtypes = [f32p, i64, ci, ci, f32p, i64, ci, ci, i32p, f32p]
            fn.restype = ci
        _lib.mfo_kmeans_assign_f32.argtypes = [f32p, i64, f32p, ci, ci, i32p]
        _lib.mfo_merge_shards.argtypes = [i32p, f32p, ci, i64, ci, ci, i32p, f32p]
        _lib.mfo_kmeans_train.argtypes = [f32p, i64, ci, ci, ci, ci, f32p, i32p, i32p, i32p]
        _lib.mfo_kmeans_train.restype = ci
        _lib.mfo_kmeans_seed_permutation.argtypes = [i64, ctypes.c_uint32, i32p]
        _lib.mfo_kmeans_train_sharded.argtypes = [f32p, i64, ci, ci, ci, ci, ci,
                                                  np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS"),
                                                  f32p, i32p, i32p, i32p]
        _lib.mfo_kmeans_train_sharded.restype = ci
        i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
        f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
        _lib.mfo_score_pairs_f64.argtypes = [f32p, ci, ci, f32p, i64p, i64p, i64, f64p]
        _lib.mfo_kmeans_assign_cand.argtypes = [f32p, i64, f32p, ci, i64p, i32p, i32p]
    return _lib


def _c(a, dt=np.float32):
    return np.ascontiguousarray(a, dtype=dt)


def row_sq_norms(v: np.ndarray) -> np.ndarray:
    v = _c(v)
    out = np.empty(v.shape[0], np.float32)
    lib().mfo_row_sq_norms(v, v.shape[0], v.shape[1], out)
    return out


def normalize_rows(v: np.ndarray) -> np.ndarray:
    v = _c(v).copy()
    lib().mfo_normalize_rows(v, v.shape[0], v.shape[1])
    return v


def flat_search_f64(db, q, k, metric=L2, kmax=1024):
    """Exact fp64 brute force (ties to lowest id).  For COSINE the rows are
    normalised first, exactly as the index stores them."""
    db, q = _c(db), _c(q)
    if metric == COSINE:
        db, q = normalize_rows(db), normalize_rows(q)
    m, dim = q.shape
    kk = max(1, min(k, kmax))
    ids = np.empty((m, kk), np.int32)
    dist = np.empty((m, kk), np.float32)
    n = db.shape[0] if db.size else 0
    dbp = db if db.size else np.zeros((1, dim), np.float32)
    lib().mfo_flat_search_f64(dbp, n, dim, metric, q, m, k, kmax, ids, dist)
    return ids, dist


def flat_search_cpusearch(db, q, k, metric=L2, kmax=1024):
    """The reference's cpuSearch semantics (fp32 Distance.h score)."""
    db, q = _c(db), _c(q)
    if metric == COSINE:
        db, q = normalize_rows(db), normalize_rows(q)
    m, dim = q.shape
    kk = max(1, min(k, kmax))
    ids = np.empty((m, kk), np.int32)
    dist = np.empty((m, kk), np.float32)
    n = db.shape[0] if db.size else 0
    dbp = db if db.size else np.zeros((1, dim), np.float32)
    lib().mfo_flat_search_cpusearch(dbp, n, dim, metric, q, m, k, kmax, ids, dist)
    return ids, dist


def kmeans_assign_f32(points, cents) -> np.ndarray:
    points, cents = _c(points), _c(cents)
    out = np.empty(points.shape[0], np.int32)
    lib().mfo_kmeans_assign_f32(points, points.shape[0], cents, cents.shape[0],
                                points.shape[1], out)
    return out


def kmeans_train(data, nlist: int, iters: int = 12, max_points_per_centroid: int = 256):
    """CoarseQuantizer::train restated (see mflat_oracle_kmeans.cpp):
    returns (centroids, assign, cell_start, reordered_ids)."""
    data = _c(data)
    n, dim = data.shape
    nl = min(nlist, n)
    cents = np.empty((nl, dim), np.float32)
    assign = np.empty(n, np.int32)
    start = np.empty(nl + 1, np.int32)
    reord = np.empty(n, np.int32)
    got = lib().mfo_kmeans_train(data, n, dim, nlist, iters, max_points_per_centroid, cents, assign,
                                 start, reord)
    assert got == nl
    return cents, assign, start, reord


def kmeans_train_sharded(data, nlist: int, iters: int, offsets, max_points_per_centroid: int = 256):
    """kmeans_train over row shards [offsets[r], offsets[r+1]) (per-rank sums added in rank order)."""
    data = _c(data)
    n, dim = data.shape
    off = np.ascontiguousarray(offsets, dtype=np.int64)
    nl = min(nlist, n)
    cents = np.empty((nl, dim), np.float32)
    assign = np.empty(n, np.int32)
    start = np.empty(nl + 1, np.int32)
    reord = np.empty(n, np.int32)
    got = lib().mfo_kmeans_train_sharded(data, n, dim, nlist, iters, max_points_per_centroid,
                                         len(off) - 1, off, cents, assign, start, reord)
    assert got == nl
    return cents, assign, start, reord


def kmeans_seed_permutation(n: int, seed: int = 12345) -> np.ndarray:
    out = np.empty(n, np.int32)
    lib().mfo_kmeans_seed_permutation(n, seed, out)
    return out


def merge_shards(ids, dist, metric=L2):
    """ids/dist: (P, m, k) per-shard lists with global ids -> (m, k)."""
    ids, dist = _c(ids, np.int32), _c(dist)
    p, m, k = ids.shape
    oi = np.empty((m, k), np.int32)
    od = np.empty((m, k), np.float32)
    lib().mfo_merge_shards(ids, dist, p, m, k, metric, oi, od)
    return oi, od


def exact_ids_match(got_ids, got_dist, ref_ids, ref_dist, rel=1e-6):
    """North-star id criterion: returned ids must equal the oracle's except
    where the oracle's adjacent distances differ by less than `rel` relative
    (inside such a near-tie run the order is not pinned).  `ref_ids` /
    `ref_dist` may carry extra columns past k (pass k+1 to also check the
    boundary).  Returns the number of positions j < k whose id differs and is
    not explained by a near-tie with a neighbouring oracle position."""
    got_ids = np.asarray(got_ids)
    ref_ids = np.asarray(ref_ids)
    ref_dist = np.asarray(ref_dist, np.float64)
    m, k = got_ids.shape
    kr = ref_ids.shape[1]
    bad = 0
    for i in range(m):
        if np.array_equal(got_ids[i], ref_ids[i, :k]):
            continue
        d = ref_dist[i]
        for j in range(k):
            if got_ids[i, j] == ref_ids[i, j]:
                continue
            scale = max(abs(d[j]), 1e-30)
            near = (j > 0 and abs(d[j] - d[j - 1]) <= rel * scale) or \
                   (j + 1 < kr and abs(d[j + 1] - d[j]) <= rel * scale)
            if not near:
                bad += 1
    return bad
