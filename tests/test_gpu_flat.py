"""GPU parity of the exact flat path, through the C ABI.

Criterion: ids identical to the fp64 brute-force oracle
(reference Distance.h semantics, ties to the lowest id) except inside near-ties
closer than 1e-6 relative; distances within 1e-5 relative."""
import os

import zlib

import numpy as np
import pytest

import mflat_b200 as M
import oracle as O

pytestmark = pytest.mark.gpu

METRIC = {"l2": O.L2, "ip": O.IP, "cosine": O.COSINE}
REL_TIE = 1e-6
REL_DIST = 1e-5


def search(db, q, k, metric, timing=None, **kw):
    idx = M.FlatIndex(db.shape[1], metric, **kw)
    assert idx.ready
    if db.shape[0]:
        idx.add(db)
    idx.set_timing(True)
    out = idx.search(q, k)
    if timing is not None:
        timing.append(idx.last_timing())
    return out


def assert_exact(ids, dist, db, q, k, metric):
    ref_i, ref_d = O.flat_search_f64(db, q, k + 1, METRIC[metric])
    assert ids.shape == (q.shape[0], k)
    assert O.exact_ids_match(ids, dist, ref_i, ref_d, rel=REL_TIE) == 0
    rd = ref_d[:, :k]
    fin = np.isfinite(rd)
    assert np.array_equal(fin, np.isfinite(dist))
    assert np.array_equal(ids[~fin], np.full((~fin).sum(), -1))
    err = np.abs(dist[fin].astype(np.float64) - rd[fin]) / np.maximum(np.abs(rd[fin]), 1e-20)
    assert err.max(initial=0.0) <= REL_DIST


SHAPES = [  # n, dim, m, k
    (1, 8, 3, 1), (5, 8, 4, 10), (255, 17, 7, 10), (256, 32, 128, 10), (257, 33, 129, 5),
    (1000, 100, 300, 16), (3000, 128, 64, 21), (4099, 3, 33, 7), (2000, 1, 5, 4),
    (1500, 129, 20, 10), (800, 200, 11, 8),
    (20000, 768, 300, 10), (4000, 960, 130, 21),   # query tile streamed with the rows
]


@pytest.mark.parametrize("metric", ["l2", "ip", "cosine"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "n%d_d%d_m%d_k%d" % s)
def test_random_shapes(metric, shape):
    n, dim, m, k = shape
    rng = np.random.default_rng(zlib.crc32(repr((metric,) + shape).encode()))
    db = rng.standard_normal((n, dim)).astype(np.float32)
    q = rng.standard_normal((m, dim)).astype(np.float32)
    tm = []
    ids, dist = search(db, q, k, metric, timing=tm)
    assert_exact(ids, dist, db, q, k, metric)
    if 32 <= dim <= 256 and n >= 256:
        # well-separated data: the error-bound proof holds for every query,
        # so the tensor-core screen alone produced the candidates (at d ~ 1000
        # the distances of N(0,1) rows concentrate and a few queries' k-th and
        # KP-th scores come within the bound: they take the exact scan)
        assert tm[0].fallback_queries == 0


def test_golden_cases(golden_dir):
    """The reference's own cpuSearch results (golden) and the fp64 oracle."""
    c = np.load(os.path.join(golden_dir, "cpusearch.npz"))
    names = sorted({f.rsplit("_", 1)[0] for f in c.files})
    mname = {0: "l2", 1: "ip", 2: "cosine"}
    for nm in names:
        n, dim, m, k, metric = (int(x) for x in c[nm + "_meta"])
        db, q = c[nm + "_db"], c[nm + "_q"]
        ids, dist = search(db, q, k, mname[metric])
        assert_exact(ids, dist, db, q, k, mname[metric])
        assert O.exact_ids_match(ids, dist, c[nm + "_ids"], c[nm + "_dist"], rel=1e-5) == 0, nm


@pytest.mark.parametrize("metric", ["l2", "ip"])
def test_duplicates_and_exact_ties(metric):
    """Many identical rows: ties must come back lowest-id first (the proof
    fails for these queries and the exact full scan answers them)."""
    rng = np.random.default_rng(11)
    base = rng.standard_normal((6, 24)).astype(np.float32)
    db = base[rng.integers(0, 6, size=700)]
    q = np.concatenate([base[:3], rng.standard_normal((5, 24)).astype(np.float32)])
    tm = []
    ids, dist = search(db, q, 12, metric, timing=tm)
    assert tm[0].fallback_queries > 0            # the exact full scan was exercised
    ref_i, ref_d = O.flat_search_f64(db, q, 12, METRIC[metric])
    assert np.array_equal(ids, ref_i)
    assert np.array_equal(dist, ref_d)


def test_all_rows_identical():
    db = np.ones((5000, 16), np.float32)
    ids, dist = search(db, np.zeros((3, 16), np.float32), 10, "l2")
    assert (ids == np.arange(10)).all()
    assert (dist == 16.0).all()


@pytest.mark.parametrize("metric,empty", [("l2", np.inf), ("ip", -np.inf), ("cosine", -np.inf)])
def test_empty_database(metric, empty):
    idx = M.FlatIndex(8, metric)
    ids, dist = idx.search(np.ones((3, 8), np.float32), 4)
    assert ids.shape == (3, 4) and (ids == -1).all() and (dist == empty).all()


def test_incremental_add_and_reset():
    rng = np.random.default_rng(2)
    parts = [rng.standard_normal((n, 40)).astype(np.float32) for n in (100, 1, 333, 4096)]
    q = rng.standard_normal((50, 40)).astype(np.float32)
    idx = M.FlatIndex(40, "l2")
    for p in parts:
        idx.add(p)
    db = np.concatenate(parts)
    assert idx.size == db.shape[0]
    ids, dist = idx.search(q, 10)
    assert_exact(ids, dist, db, q, 10, "l2")
    idx.reset()
    assert idx.size == 0
    ids, _ = idx.search(q, 3)
    assert (ids == -1).all()
    idx.add(parts[2])
    ids, dist = idx.search(q, 10)
    assert_exact(ids, dist, parts[2], q, 10, "l2")


def test_n_smaller_than_k_pads():
    rng = np.random.default_rng(4)
    db = rng.standard_normal((3, 8)).astype(np.float32)
    q = rng.standard_normal((2, 8)).astype(np.float32)
    ids, dist = search(db, q, 10, "l2")
    assert (ids[:, 3:] == -1).all() and np.isinf(dist[:, 3:]).all()
    assert_exact(ids, dist, db, q, 10, "l2")


@pytest.mark.parametrize("dim", [128, 384])
def test_simt_screen_agrees_with_tensor_core_screen(dim):
    """d = 128 keeps the query tile resident, d = 384 streams it."""
    rng = np.random.default_rng(8 + dim)
    db = rng.random((20000, dim), dtype=np.float32)
    q = rng.random((300, dim), dtype=np.float32)
    ta, tb = [], []
    a = search(db, q, 10, "l2", timing=ta)
    os.environ["MFLAT_SCREEN"] = "simt"
    try:
        b = search(db, q, 10, "l2", timing=tb)
    finally:
        del os.environ["MFLAT_SCREEN"]
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    assert ta[0].fallback_queries == 0 and tb[0].fallback_queries == 0
    assert_exact(a[0], a[1], db, q, 10, "l2")


def test_config1_full():
    """N=100k x 128, Q=1000, N(0,1) seed 0, k=10, all queries."""
    rng = np.random.default_rng(0)
    db = rng.standard_normal((100_000, 128), dtype=np.float32)
    q = rng.standard_normal((1000, 128), dtype=np.float32)
    idx = M.FlatIndex(128, "l2")
    idx.add(db)
    idx.set_timing(True)
    ids, dist = idx.search(q, 10)
    t = idx.last_timing()
    assert t.screen_launches == 1 and t.launches >= 3
    assert t.fallback_queries == 0 and t.screen_ms > 0
    assert_exact(ids, dist, db, q, 10, "l2")


def test_device_pointer_api():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(9)
    db = rng.standard_normal((5000, 64)).astype(np.float32)
    q = rng.standard_normal((77, 64)).astype(np.float32)
    idx = M.FlatIndex(64, "ip")
    d_db = torch.from_numpy(db).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    idx.add_device(d_db.data_ptr(), db.shape[0], stream)
    d_q = torch.from_numpy(q).cuda()
    d_ids = torch.empty((77, 10), dtype=torch.int32, device="cuda")
    d_dist = torch.empty((77, 10), dtype=torch.float32, device="cuda")
    used = idx.search_device(d_q.data_ptr(), 77, 10, d_ids.data_ptr(), d_dist.data_ptr(), stream)
    assert used == 10
    torch.cuda.synchronize()
    assert_exact(d_ids.cpu().numpy(), d_dist.cpu().numpy(), db, q, 10, "ip")


LARGE = [  # n, dim, m, k   (n <= 32768: every row buffered; larger: floor pre-pass;
           #                 n >= 2M at these k: two-stage floor, sparse lists then a buffer pass)
    (3000, 40, 30, 22), (3000, 128, 17, 300), (150_000, 128, 40, 64),
    (150_000, 64, 33, 1024), (200_003, 17, 20, 100), (60_000, 160, 9, 50),
    (2_000_000, 64, 12, 100), (2_100_001, 20, 9, 22),
]


@pytest.mark.parametrize("metric", ["l2", "ip", "cosine"])
@pytest.mark.parametrize("shape", LARGE, ids=lambda s: "n%d_d%d_m%d_k%d" % s)
def test_large_k_exact(metric, shape):
    n, dim, m, k = shape
    rng = np.random.default_rng(zlib.crc32(repr(("large", metric) + shape).encode()))
    db = rng.standard_normal((n, dim)).astype(np.float32)
    q = rng.standard_normal((m, dim)).astype(np.float32)
    ids, dist = search(db, q, k, metric)
    assert_exact(ids, dist, db, q, k, metric)


def test_large_k_two_stage_floor_k1024():
    """17M rows at k = 1024: the floor comes from lists over 1/256 of the tiles,
    sharpened by a buffer pass over 1/16 of them, before the full pass."""
    rng = np.random.default_rng(zlib.crc32(b"two-stage-1024"))
    db = rng.standard_normal((17_000_000, 8), dtype=np.float32)
    q = rng.standard_normal((6, 8), dtype=np.float32)
    ids, dist = search(db, q, 1024, "l2")
    assert_exact(ids, dist, db, q, 1024, "l2")


def test_large_k_two_stage_denser_stage_a():
    """5M rows at k = 1024: too few tiles for lists over 1/256 of them, so
    stage A samples every 128th tile before the 1/16 buffer pass."""
    rng = np.random.default_rng(zlib.crc32(b"two-stage-stride-64"))
    db = rng.standard_normal((5_000_000, 8), dtype=np.float32)
    q = rng.standard_normal((5, 8), dtype=np.float32)
    ids, dist = search(db, q, 1024, "l2")
    assert_exact(ids, dist, db, q, 1024, "l2")


def test_large_k_clamp_and_uniform():
    """k above 1024 is clamped (one-time warning); uniform data, 1M rows."""
    rng = np.random.default_rng(21)
    db = rng.random((1_000_000, 128), dtype=np.float32)
    q = rng.random((12, 128), dtype=np.float32)
    ids, dist = search(db, q, 5000, "l2")
    assert ids.shape == (12, 1024)
    assert_exact(ids, dist, db, q, 1024, "l2")


def test_large_k_statistical_floor_redo():
    """The rows nearest to the query sit in tile 0, which every floor sample
    contains: the statistical floor from the sample is then far above the
    200th-best row, the check after the full pass catches it and the batch is
    redone with the valid floor -- the result stays exact."""
    rng = np.random.default_rng(zlib.crc32(b"stat-floor-redo"))
    n, dim, k = 2_000_000, 16, 100
    db = rng.standard_normal((n, dim)).astype(np.float32) + 4.0
    centre = np.zeros(dim, np.float32)
    db[:200] = centre + 0.01 * rng.standard_normal((200, dim)).astype(np.float32)
    q = np.stack([centre + 0.001, rng.standard_normal(dim).astype(np.float32) + 4.0])
    tm = []
    ids, dist = search(db, q, k, "l2", timing=tm)
    assert_exact(ids, dist, db, q, k, "l2")
    assert tm[0].screen_launches == 2          # the redo ran
    assert set(ids[0].tolist()) <= set(range(200))


def test_large_k_stage_b_guess_redo():
    """70 rows near the query sit in tile 0, which every sample contains: the
    stage-A guess for the stage-B floor lands among them, stage B keeps fewer
    than 2k rows, and stage B is redone above the valid stage-A floor."""
    rng = np.random.default_rng(zlib.crc32(b"stage-b-guess"))
    n, dim, k = 2_000_000, 16, 100
    db = rng.standard_normal((n, dim)).astype(np.float32)
    centre = np.full(dim, 0.5, np.float32)
    db[:70] = centre + 0.01 * rng.standard_normal((70, dim)).astype(np.float32)
    q = np.stack([centre, rng.standard_normal(dim).astype(np.float32)])
    ids, dist = search(db, q, k, "l2")
    assert_exact(ids, dist, db, q, k, "l2")
    assert set(range(70)) <= set(ids[0].tolist())
