"""The CPU oracle pinned against golden vectors produced by the reference's own
src/Distance.h (compiled in place, see tests/golden/make_golden.py)."""
import numpy as np
import pytest

import oracle as O


def _golden(golden_dir, name):
    return np.load(f"{golden_dir}/{name}")


@pytest.mark.parametrize("dim", [19, 128, 1])
def test_distance_primitives_bit_exact(golden_dir, dim):
    g = _golden(golden_dir, "distance_h.npz")
    v = g[f"d{dim}_v"]
    assert np.array_equal(O.row_sq_norms(v), g[f"d{dim}_norms"])
    assert np.array_equal(O.normalize_rows(v), g[f"d{dim}_normalized"])
    n = v.shape[0]
    a, b = v[: n // 2], v[n // 2: n // 2 * 2]
    sq = np.array([O.lib().mfo_sq_l2_f32(np.ascontiguousarray(a[i]), np.ascontiguousarray(b[i]), dim)
                   for i in range(len(a))], np.float32)
    dt = np.array([O.lib().mfo_dot_f32(np.ascontiguousarray(a[i]), np.ascontiguousarray(b[i]), dim)
                   for i in range(len(a))], np.float32)
    assert np.array_equal(sq, g[f"d{dim}_sql2"])
    assert np.array_equal(dt, g[f"d{dim}_dot"])


def _cases(golden_dir):
    c = _golden(golden_dir, "cpusearch.npz")
    names = sorted({k.rsplit("_", 1)[0] for k in c.files})
    return c, names


def test_cpusearch_restatement_matches_reference(golden_dir):
    c, names = _cases(golden_dir)
    for nm in names:
        n, dim, m, k, metric = (int(x) for x in c[nm + "_meta"])
        ids, dist = O.flat_search_cpusearch(c[nm + "_db"], c[nm + "_q"], k, metric)
        assert np.array_equal(ids, c[nm + "_ids"]), nm
        assert np.array_equal(dist, c[nm + "_dist"]), nm


def test_fp64_oracle_agrees_with_reference_cpusearch(golden_dir):
    """Same ids as the reference's fp32 cpuSearch except inside near-ties, and
    distances within 1e-5 relative."""
    c, names = _cases(golden_dir)
    for nm in names:
        n, dim, m, k, metric = (int(x) for x in c[nm + "_meta"])
        ids, dist = O.flat_search_f64(c[nm + "_db"], c[nm + "_q"], k, metric)
        ref_i, ref_d = c[nm + "_ids"], c[nm + "_dist"]
        assert O.exact_ids_match(ids, dist, ref_i, ref_d, rel=1e-6) == 0, nm
        fin = np.isfinite(ref_d)
        assert np.array_equal(fin, np.isfinite(dist)), nm
        assert np.allclose(dist[fin], ref_d[fin], rtol=1e-5, atol=1e-5), nm


def test_empty_and_tie_conventions():
    db = np.zeros((0, 4), np.float32)
    q = np.ones((3, 4), np.float32)
    for metric, empty in ((O.L2, np.inf), (O.IP, -np.inf), (O.COSINE, -np.inf)):
        ids, dist = O.flat_search_f64(db, q, 5, metric)
        assert (ids == -1).all() and (dist == empty).all()
    db = np.array([[1, 0], [0, 1], [1, 0], [1, 0]], np.float32)
    ids, _ = O.flat_search_f64(db, np.array([[1, 0]], np.float32), 3, O.L2)
    assert ids.tolist() == [[0, 2, 3]]          # equal distances -> lowest id first


def test_kmeans_assign_matches_reference(golden_dir):
    g = _golden(golden_dir, "kmeans_assign.npz")
    for nm in ("km_a", "km_b", "km_c"):
        got = O.kmeans_assign_f32(g[nm + "_pts"], g[nm + "_cents"])
        assert np.array_equal(got, g[nm + "_assign"]), nm


def test_merge_shards_equals_single_shard():
    rng = np.random.default_rng(5)
    db = rng.standard_normal((997, 12)).astype(np.float32)
    db[500] = db[3]                            # cross-shard tie
    q = rng.standard_normal((9, 12)).astype(np.float32)
    q[0] = db[3]
    for metric in (O.L2, O.IP):
        ref_i, ref_d = O.flat_search_f64(db, q, 17, metric)
        bounds = [0, 300, 650, 997]
        pi, pd = [], []
        for a, b in zip(bounds[:-1], bounds[1:]):
            i, d = O.flat_search_f64(db[a:b], q, 17, metric)
            pi.append(np.where(i >= 0, i + a, -1))
            pd.append(d)
        mi, md = O.merge_shards(np.stack(pi), np.stack(pd), metric)
        assert np.array_equal(mi, ref_i)
        assert np.array_equal(md, ref_d)


def test_kmeans_oracle_self_consistent():
    """The training restatement: the seed permutation is a permutation, the
    CSR groups every point under its final cell, and the centroids are the
    double means of the training subset's cells."""
    p = O.kmeans_seed_permutation(1000)
    assert np.array_equal(np.sort(p), np.arange(1000))
    rng = np.random.default_rng(3)
    x = rng.standard_normal((4000, 6)).astype(np.float32)
    c, a, s, r = O.kmeans_train(x, 12, 4, 256)
    assert s[0] == 0 and s[-1] == 4000 and np.all(np.diff(s) >= 0)
    for cell in range(12):
        ids = r[s[cell]:s[cell + 1]]
        assert np.all(a[ids] == cell) and np.all(np.diff(ids) > 0)
    assert np.array_equal(a, O.kmeans_assign_f32(x, c))
