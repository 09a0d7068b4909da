"""Persistence of a flat index (save -> load) through the C ABI: the loaded
index holds the same rows and returns bit-identical results, for every
storage precision and metric (Cosine rows are stored normalised and must not
be normalised again on load)."""
import os
import shutil
import subprocess
import zlib

import numpy as np
import pytest

import mflat_b200 as M

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("storage", ["fp32", "fp16", "bf16"])
@pytest.mark.parametrize("metric", ["l2", "ip", "cosine"])
def test_save_load_roundtrip(tmp_path, storage, metric):
    rng = np.random.default_rng(zlib.crc32(repr(("persist", storage, metric)).encode()))
    dim = 37
    a = rng.standard_normal((3000, dim)).astype(np.float32)
    b = rng.standard_normal((1500, dim)).astype(np.float32) * 3
    q = rng.standard_normal((70, dim)).astype(np.float32)
    idx = M.FlatIndex(dim, metric, storage)
    idx.add(a)
    idx.add(b)
    path = str(tmp_path / f"flat_{storage}_{metric}.mffl")
    idx.save(path)
    with open(path, "rb") as f:
        assert f.read(4) == b"MFFL"
    hdr = np.fromfile(path, np.int32, count=8)
    assert list(hdr[1:]) == [1, dim, M.METRICS[metric], M.STORAGES[storage], 4500, 0, 0]
    elem = 4 if storage == "fp32" else 2
    assert (tmp_path / f"flat_{storage}_{metric}.mffl").stat().st_size == 32 + 4500 * dim * elem
    back = M.FlatIndex.load(path)
    assert back.size == 4500 and back.dim == dim
    assert back.storage == M.STORAGES[storage]
    for k in (10, 100):
        i0, d0 = idx.search(q, k)
        i1, d1 = back.search(q, k)
        assert np.array_equal(i0, i1)
        assert np.array_equal(d0.view(np.uint32), d1.view(np.uint32))
    # a saved-and-reloaded index can be saved again byte for byte
    path2 = str(tmp_path / "again.mffl")
    back.save(path2)
    assert open(path, "rb").read() == open(path2, "rb").read()


def test_load_into_index_and_empty(tmp_path):
    idx = M.FlatIndex(8, "l2")
    path = str(tmp_path / "empty.mffl")
    idx.save(path)
    back = M.FlatIndex.load(path)
    assert back.size == 0
    ids, dist = back.search(np.zeros((2, 8), np.float32), 3)
    assert (ids == -1).all() and np.isinf(dist).all()


def test_truncated_file_leaves_index_unchanged(tmp_path):
    """FlatIndex::load (C++ API) on an index that holds rows: a file shorter
    than its header announces is refused before anything is replaced."""
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    src = M.FlatIndex(37, "l2")
    src.add(np.random.default_rng(2).standard_normal((900, 37)).astype(np.float32))
    full = str(tmp_path / "full.mffl")
    src.save(full)
    cut = str(tmp_path / "cut.mffl")
    with open(full, "rb") as f, open(cut, "wb") as g:
        g.write(f.read()[: 32 + 600 * 37 * 4 + 5])
    pkg = os.path.join(ROOT, "metal-flat_b200")
    exe = str(tmp_path / "cxx_load_probe")
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Werror", "-I", os.path.join(pkg, "include"),
                    os.path.join(ROOT, "tests", "cxx_load_probe.cpp"), "-L", os.path.join(pkg, "lib"),
                    "-lmetalflat_c", "-Wl,-rpath," + os.path.join(pkg, "lib"), "-o", exe], check=True)
    out = subprocess.run([exe, full, cut], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout + out.stderr
    assert out.stdout.split() == ["ok", "900"]
