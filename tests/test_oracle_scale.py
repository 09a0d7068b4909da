"""The screened oracle used at the benchmarked sizes (oracle/scale.py) gives
exactly the plain oracle's answers: fp64 top-k ids and distances
(oracle.flat_search_f64) and sequential-fp32 k-means assignments
(oracle.kmeans_assign_f32), including duplicate rows, exact ties, k larger
than one block and the streaming of the database in uneven blocks."""
import numpy as np
import pytest

import oracle as O
import scale as S


def stream(db, q, k, metric, blocks):
    se = S.StreamingExact(q, k, metric)
    cuts = np.r_[0, np.sort(blocks), db.shape[0]]
    for a, z in zip(cuts[:-1], cuts[1:]):
        se.add(db[a:z], int(a))
    return se


@pytest.mark.parametrize("metric", [O.L2, O.IP, O.COSINE])
@pytest.mark.parametrize("k", [1, 10, 100])
def test_streaming_matches_fp64_oracle(metric, k):
    rng = np.random.default_rng(7 + k + 3 * metric)
    db = rng.standard_normal((6000, 48), dtype=np.float32)
    db[100:140] = db[50]                      # duplicated rows: exact ties
    db[4000:4003] = db[7]
    q = rng.standard_normal((37, 48), dtype=np.float32)
    q[3] = db[50]
    se = stream(db, q, k, metric, [900, 2500, 2501, 5900])
    got_i, got_d = se.result()
    ref_i, ref_d = O.flat_search_f64(db, q, k, metric)
    np.testing.assert_array_equal(got_i, ref_i)
    np.testing.assert_array_equal(got_d, ref_d)


def test_streaming_uniform_like_config3():
    rng = np.random.default_rng(11)
    db = rng.random((20000, 128), dtype=np.float32)
    q = rng.random((16, 128), dtype=np.float32)
    se = stream(db, q, 10, O.L2, [8192, 16384])
    got_i, got_d = se.result()
    ref_i, ref_d = O.flat_search_f64(db, q, 10, O.L2)
    np.testing.assert_array_equal(got_i, ref_i)
    np.testing.assert_array_equal(got_d, ref_d)
    # the screen keeps few rows beyond the answer
    assert se.rescored < 40 * 16 * 10


def test_streaming_rank_merge_and_short_db():
    rng = np.random.default_rng(3)
    db = rng.standard_normal((700, 16), dtype=np.float32)
    q = rng.standard_normal((9, 16), dtype=np.float32)
    parts = []
    for a, z in ((0, 300), (300, 700)):
        se = S.StreamingExact(q, 50, O.L2)
        se.add(db[a:z], a)
        parts.append(se.pools())
    got_i, got_d = se.result(S.merge_pools(parts))
    ref_i, ref_d = O.flat_search_f64(db, q, 50, O.L2)
    np.testing.assert_array_equal(got_i, ref_i)
    np.testing.assert_array_equal(got_d, ref_d)
    # fewer rows than k: padding like the plain oracle
    se = S.StreamingExact(q, 20, O.IP)
    se.add(db[:5], 0)
    gi, gd = se.result()
    ri, rd = O.flat_search_f64(db[:5], q, 20, O.IP)
    np.testing.assert_array_equal(gi, ri)
    np.testing.assert_array_equal(gd, rd)


def test_kmeans_screened_matches_sequential_oracle():
    rng = np.random.default_rng(5)
    centres = rng.standard_normal((300, 64), dtype=np.float32)
    cents = centres + np.float32(0.05) * rng.standard_normal(centres.shape, dtype=np.float32)
    cents[17] = cents[3]                       # tied centroids: lowest index wins
    cents[200] = cents[3]
    comp = rng.integers(0, 300, size=9000)
    pts = centres[comp] + np.float32(0.3) * rng.standard_normal((9000, 64), dtype=np.float32)
    pts[:50] = cents[3]
    pts[50:60] = 0.5 * (cents[8] + cents[9])  # near-equidistant points
    got = S.kmeans_assign_screened(pts, cents, block=1000)
    ref = O.kmeans_assign_f32(pts, cents)
    np.testing.assert_array_equal(got, ref)
