"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run where a source checkout of the reference (metal-flat) is available:

    python tests/golden/make_golden.py <path to the metal-flat checkout>

It compiles oracle/_ref/libref_golden.so from the reference's own
src/Distance.h and src/Log.cpp (recipe: oracle/Makefile) and records, for
seeded inputs:
  * Distance.h primitives: rowSqNorms, normalizeRows, sqL2, dot,
    l2ScoreFromDot, emptyValue                         (Distance.h:26-81)
  * cpuSearch top-k for L2 / InnerProduct / Cosine, including duplicate
    rows (tie rule), N < k and k = 1                   (FlatIndex.mm:259-290)
  * the CPU k-means assignment, including duplicated centroids
                                                       (CoarseQuantizer.mm:122-130)
The fixtures are small .npz files; tests read them on any machine (the
reference tree is not needed at test time).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
ORACLE = os.path.join(ROOT, "oracle")


def load_ref(ref_dir):
    subprocess.run(["make", "-s", "-C", ORACLE, f"REF={ref_dir}"], check=True)
    path = os.path.join(ORACLE, "_ref", "libref_golden.so")
    if not os.path.exists(path):
        sys.exit("reference tree not available: cannot build libref_golden.so")
    L = ctypes.CDLL(path)
    f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
    i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
    ci, cf = ctypes.c_int, ctypes.c_float
    L.ref_row_sq_norms.argtypes = [f32p, ci, ci, f32p]
    L.ref_normalize_rows.argtypes = [f32p, ci, ci]
    L.ref_sq_l2.argtypes = [f32p, f32p, ci]
    L.ref_sq_l2.restype = cf
    L.ref_dot.argtypes = [f32p, f32p, ci]
    L.ref_dot.restype = cf
    L.ref_l2_score_from_dot.argtypes = [cf, cf, cf]
    L.ref_l2_score_from_dot.restype = cf
    L.ref_empty_value.argtypes = [ci]
    L.ref_empty_value.restype = cf
    L.ref_cpu_search.argtypes = [f32p, ci, ci, ci, f32p, ci, ci, i32p, f32p]
    L.ref_kmeans_assign.argtypes = [f32p, ci, f32p, ci, ci, i32p]
    return L


def c32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def distance_primitives(L, rng, n, dim):
    v = c32(rng.standard_normal((n, dim)) * rng.uniform(0.1, 10.0, size=(n, 1)))
    v[0] = 0.0                      # zero row: normalizeRows leaves it as is
    norms = np.empty(n, np.float32)
    L.ref_row_sq_norms(v, n, dim, norms)
    vn = v.copy()
    L.ref_normalize_rows(vn, n, dim)
    a, b = v[: n // 2], v[n // 2: n // 2 * 2]
    sql2 = np.array([L.ref_sq_l2(c32(a[i]), c32(b[i]), dim) for i in range(len(a))], np.float32)
    dot = np.array([L.ref_dot(c32(a[i]), c32(b[i]), dim) for i in range(len(a))], np.float32)
    triples = c32(rng.standard_normal((64, 3)) * 10)
    l2s = np.array([L.ref_l2_score_from_dot(*map(float, t)) for t in triples], np.float32)
    return dict(v=v, norms=norms, normalized=vn, sql2=sql2, dot=dot,
                triples=triples, l2_score_from_dot=l2s)


def cpu_search(L, db, q, k, metric):
    """Reference cpuSearch on the vectors the index would hold (Cosine
    normalises db on add and queries at search: FlatIndex.mm:241-242, 311-315)."""
    db, q = c32(db).copy(), c32(q).copy()
    if metric == 2:
        L.ref_normalize_rows(db, db.shape[0], db.shape[1])
        L.ref_normalize_rows(q, q.shape[0], q.shape[1])
    m, dim = q.shape
    ids = np.empty((m, k), np.int32)
    dist = np.empty((m, k), np.float32)
    L.ref_cpu_search(db, db.shape[0], dim, metric, q, m, k, ids, dist)
    return ids, dist


def main():
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path to the metal-flat checkout>")
    L = load_ref(os.path.abspath(sys.argv[1]))
    rng = np.random.default_rng(20261201)
    out = {}
    for n, dim in ((37, 19), (64, 128), (9, 1)):
        prim = distance_primitives(L, rng, n, dim)
        for key, val in prim.items():
            out[f"d{dim}_{key}"] = val
    out["empty_value"] = np.array([L.ref_empty_value(m) for m in (0, 1, 2)], np.float32)
    np.savez_compressed(os.path.join(HERE, "distance_h.npz"), **out)

    cases = {}
    # (name, n, dim, m, k, metric, kind)
    specs = [
        ("l2_basic", 300, 24, 13, 10, 0, "normal"),
        ("ip_basic", 300, 24, 13, 10, 1, "normal"),
        ("cos_basic", 300, 24, 13, 10, 2, "normal"),
        ("l2_d128", 600, 128, 8, 64, 0, "normal"),
        ("l2_dups", 120, 16, 7, 12, 0, "dups"),
        ("ip_dups", 120, 16, 7, 12, 1, "dups"),
        ("l2_n_lt_k", 5, 8, 4, 10, 0, "normal"),
        ("cos_n_lt_k", 3, 8, 2, 6, 2, "normal"),
        ("l2_k1", 500, 33, 20, 1, 0, "uniform"),
        ("ip_d3", 257, 3, 11, 17, 1, "uniform"),
    ]
    for name, n, dim, m, k, metric, kind in specs:
        if kind == "uniform":
            db = rng.random((n, dim), dtype=np.float32)
            q = rng.random((m, dim), dtype=np.float32)
        else:
            db = c32(rng.standard_normal((n, dim)))
            q = c32(rng.standard_normal((m, dim)))
        if kind == "dups":
            base = db[:10].copy()
            db = c32(base[rng.integers(0, 10, size=n)])   # only 10 distinct rows
            q[0] = db[5]                                   # exact hit, many ties
        ids, dist = cpu_search(L, db, q, k, metric)
        cases.update({f"{name}_db": db, f"{name}_q": q, f"{name}_ids": ids,
                      f"{name}_dist": dist,
                      f"{name}_meta": np.array([n, dim, m, k, metric], np.int64)})
    np.savez_compressed(os.path.join(HERE, "cpusearch.npz"), **cases)

    km = {}
    for name, n, dim, nc in (("km_a", 600, 16, 37), ("km_b", 300, 128, 64), ("km_c", 200, 5, 9)):
        cents = c32(rng.standard_normal((nc, dim)))
        cents[nc // 2] = cents[1]                         # duplicated centroid -> tie
        lab = rng.integers(0, nc, size=n)
        pts = c32(cents[lab] + 0.3 * rng.standard_normal((n, dim)))
        pts[:5] = cents[1]                                # exact tie at distance 0
        assign = np.empty(n, np.int32)
        L.ref_kmeans_assign(pts, n, cents, nc, dim, assign)
        km.update({f"{name}_pts": pts, f"{name}_cents": cents, f"{name}_assign": assign})
    np.savez_compressed(os.path.join(HERE, "kmeans_assign.npz"), **km)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
