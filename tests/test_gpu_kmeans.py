"""GPU k-means assignment step: bit-exact against the fp32 oracle
(sequential sqL2, strict '<', lowest centroid wins ties), through the C ABI."""
import os

import numpy as np
import pytest

import mflat_b200 as M
import oracle as O

pytestmark = pytest.mark.gpu


def test_golden_assignments(golden_dir):
    g = np.load(os.path.join(golden_dir, "kmeans_assign.npz"))
    for nm in ("km_a", "km_b", "km_c"):
        got = M.kmeans_assign(g[nm + "_pts"], g[nm + "_cents"])
        assert np.array_equal(got, g[nm + "_assign"]), nm


@pytest.mark.parametrize("n,dim,nc", [(5000, 128, 1024), (3000, 16, 300), (2000, 100, 77),
                                      (1000, 129, 50), (777, 2, 9), (40000, 64, 4096)])
def test_mixture_bit_exact(n, dim, nc):
    rng = np.random.default_rng(n + dim + nc)
    centres = rng.standard_normal((nc, dim)).astype(np.float32)
    lab = rng.integers(0, nc, size=n)
    pts = (centres[lab] + 0.3 * rng.standard_normal((n, dim))).astype(np.float32)
    cents = (centres + 0.05 * rng.standard_normal((nc, dim))).astype(np.float32)
    cents[nc // 3] = cents[nc // 2]          # an exact duplicate centroid
    pts[:7] = cents[nc // 2]                 # points sitting on it: tie at 0
    got = M.kmeans_assign(pts, cents)
    ref = O.kmeans_assign_f32(pts, cents)
    assert np.array_equal(got, ref)
    assert (got[:7] == min(nc // 3, nc // 2)).all()


def test_uniform_near_ties():
    """Uniform data has many near-equal distances; the re-check must follow
    the fp32 sequential order exactly."""
    rng = np.random.default_rng(3)
    pts = rng.random((20000, 32), dtype=np.float32)
    cents = rng.random((512, 32), dtype=np.float32)
    assert np.array_equal(M.kmeans_assign(pts, cents), O.kmeans_assign_f32(pts, cents))
