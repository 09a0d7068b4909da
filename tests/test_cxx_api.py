"""The C++ API (metal-flat_b200/include/metalflat) as a C++ caller links it, on CPU.

A small C++ program is compiled against the public headers and linked against
libmetalflat_c.so; without a CUDA device it checks that the classes resolve,
that DeviceError crosses the library boundary, the index-file header reader,
and the k-means seed permutation against the oracle's restatement.
"""
import os
import shutil
import struct
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "metal-flat_b200")
LIBDIR = os.path.join(PKG, "lib")
sys.path.insert(0, os.path.join(ROOT, "oracle"))


@pytest.fixture(scope="module")
def probe(tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    if not os.path.exists(os.path.join(LIBDIR, "libmetalflat_c.so")):
        pytest.skip("library not built")
    exe = str(tmp_path_factory.mktemp("cxx") / "cxx_api_probe")
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Werror",
                    "-I", os.path.join(PKG, "include"), os.path.join(ROOT, "tests", "cxx_api_probe.cpp"),
                    "-L", LIBDIR, "-lmetalflat_c", "-Wl,-rpath," + LIBDIR, "-o", exe], check=True)

    def run(index_file):
        env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
        out = subprocess.run([exe, index_file], capture_output=True, text=True, check=True,
                             env=env).stdout
        return {ln.split()[0]: ln.split()[1:] for ln in out.splitlines() if ln.strip()}
    return run


def header(magic=b"MFFL", version=1, dim=96, metric=1, storage=2, n=12345):
    return magic + struct.pack("<7i", version, dim, metric, storage, n, 0, 0)


def test_cxx_api_links_and_fails_loudly_without_device(probe, tmp_path):
    f = tmp_path / "db.mffl"
    f.write_bytes(header())
    r = probe(str(f))
    assert r["loglevel"] == ["3"]
    assert r["index"] == ["0", "8", "0", "1"]           # not ready, dim 8, empty, inner product
    assert r["search"] == ["DeviceError"] and r["searchInto"] == ["DeviceError"]
    assert r["empty"] == ["0"]                           # m = 0: nothing to do, no device needed
    assert r["info"] == ["1", "96", "1", "2", "12345"]
    assert r["coarse_dim0"] == ["invalid_argument"]
    assert r["coarse"] == ["8", "0", "0"]
    assert r["coarse_shard"] == ["invalid_argument"]
    assert r["coarse_train"] == ["DeviceError"]


@pytest.mark.parametrize("blob", [
    header(magic=b"LFFM"), header(magic=b"\0\0\0\0"), header(version=2), header(dim=0), header(metric=3),
    header(storage=5), header(n=-1), b"MF",
])
def test_header_reader_rejects_bad_files(probe, tmp_path, blob):
    f = tmp_path / "bad.mffl"
    f.write_bytes(blob)
    assert probe(str(f))["info"][0] == "0"


def test_header_reader_missing_file(probe, tmp_path):
    assert probe(str(tmp_path / "missing.mffl"))["info"][0] == "0"


def test_seed_permutation_matches_oracle(probe, tmp_path):
    import oracle as O
    perm = np.array(probe(str(tmp_path / "none"))["perm"], dtype=np.int64)
    assert sorted(perm.tolist()) == list(range(37))
    assert np.array_equal(perm, np.asarray(O.kmeans_seed_permutation(37, 12345), dtype=np.int64))
