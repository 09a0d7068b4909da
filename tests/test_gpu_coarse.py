"""CoarseQuantizer (k-means train, CSR scaffold, cell probing) on the device,
through the C ABI, against the CPU restatement of the reference's training
(oracle/mflat_oracle_kmeans.cpp): centroids bit-exact, CSR identical."""
import zlib

import numpy as np
import pytest

import mflat_b200 as M
import oracle as O

pytestmark = pytest.mark.gpu


def check_train(data, nlist, iters):
    cq = M.CoarseQuantizer(data.shape[1])
    cq.train(data, nlist, iters)
    c_ref, a_ref, s_ref, r_ref = O.kmeans_train(data, nlist, iters, 256)
    assert cq.nlist == c_ref.shape[0] and cq.size == data.shape[0]
    c = cq.centroids()
    assert np.array_equal(c.view(np.uint32), c_ref.view(np.uint32))
    s, r = cq.csr()
    assert np.array_equal(s, s_ref)
    assert np.array_equal(r, r_ref)
    return cq, c_ref


@pytest.mark.parametrize("shape", [(20000, 16, 50, 6), (3000, 100, 40, 5), (9000, 128, 30, 3)],
                         ids=lambda s: "n%d_d%d_nl%d_it%d" % s)
def test_train_matches_oracle(shape):
    n, dim, nlist, iters = shape
    rng = np.random.default_rng(zlib.crc32(repr(("coarse",) + shape).encode()))
    centres = rng.standard_normal((max(4, nlist // 3), dim)).astype(np.float32)
    data = (centres[rng.integers(0, centres.shape[0], n)] +
            0.3 * rng.standard_normal((n, dim))).astype(np.float32)
    check_train(data, nlist, iters)


def test_train_with_empty_cells_reseeds():
    """Ten distinct points repeated: many seeds coincide, cells go empty and are
    reseeded from the host's mt19937 stream in cell order."""
    rng = np.random.default_rng(7)
    base = rng.standard_normal((10, 12)).astype(np.float32)
    data = base[rng.integers(0, 10, 2500)]
    check_train(data, 32, 4)


def test_nlist_clamped_and_probe():
    rng = np.random.default_rng(11)
    data = rng.standard_normal((700, 24)).astype(np.float32)
    cq, cents = check_train(data, 1000, 2)            # nlist clamped to n
    assert cq.nlist == 700
    q = rng.standard_normal((33, 24)).astype(np.float32)
    got = cq.probe(q, 9)
    ref_i, ref_d = O.flat_search_f64(cents, q, 10, O.L2)
    dist = ((q[:, None, :].astype(np.float64) - cents[got].astype(np.float64)) ** 2).sum(-1)
    assert O.exact_ids_match(got, dist.astype(np.float32), ref_i, ref_d, rel=1e-6) == 0


def test_probe_clustered_cells():
    rng = np.random.default_rng(5)
    data = rng.standard_normal((30000, 32)).astype(np.float32)
    cq, cents = check_train(data, 128, 5)
    q = data[:100] + 0.01
    got = cq.probe(q, 4)
    ref_i, ref_d = O.flat_search_f64(cents, q, 5, O.L2)
    dist = ((q[:, None, :].astype(np.float64) - cents[got].astype(np.float64)) ** 2).sum(-1)
    assert O.exact_ids_match(got, dist.astype(np.float32), ref_i, ref_d, rel=1e-6) == 0


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:                                  # noqa: BLE001
        return 0


@pytest.mark.skipif(_gpus() < 2, reason="needs at least two GPUs")
def test_sharded_training_matches_oracle():
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    world = min(_gpus(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MFLAT_NCCL_TIMEOUT_S="120")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", "29541",
           os.path.join(root, "tests", "coarse_shard_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0


def test_single_rank_shard_setting_is_plain_training():
    """set_shard(0, 1, ...) is the unsharded path."""
    rng = np.random.default_rng(12)
    data = rng.standard_normal((4000, 20)).astype(np.float32)
    cq = M.CoarseQuantizer(20)
    cq.set_shard(0, 1, None, np.array([0, 4000], np.int64))
    cq.train(data, 16, 3)
    c_ref, _, s_ref, r_ref = O.kmeans_train(data, 16, 3, 256)
    assert np.array_equal(cq.centroids().view(np.uint32), c_ref.view(np.uint32))
    s, r = cq.csr()
    assert np.array_equal(s, s_ref) and np.array_equal(r, r_ref)
