"""C-ABI conformance that needs no GPU: the library loads, exports every entry
point include/mflat.h declares, and keeps the reference's argument checks,
constants, status strings and logging semantics (c/mflat.cpp, src/Log.cpp)."""
import ctypes
import os
import re

import numpy as np
import pytest

import mflat_b200 as M

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "mflat.h")


def header_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"MFLAT_API\b[^;{]*?\b(mflat_\w+)\s*\(", text, flags=re.S)))


def has_gpu():
    try:
        L = ctypes.CDLL(M.CUDA_LIB_PATH)
        return L.mflat_cu_device_count() > 0
    except OSError:
        return False


def test_exports_every_declared_symbol(built_lib):
    syms = header_symbols()
    assert len(syms) >= 25
    for s in syms:
        assert hasattr(built_lib, s), s
    assert sorted(M.EXPORTS) == syms


def test_constants_and_strings(built_lib):
    assert M.version() == "0.1.0"
    assert M.max_k() == 1024
    L = built_lib
    for code, text in M.STATUS.items():
        assert L.mflat_status_str(code).decode() == text
    assert L.mflat_status_str(99).decode() == "unknown"


def test_argument_checks_without_device(built_lib):
    L = built_lib
    st = ctypes.c_int(-1)
    assert L.mflat_flat_create(0, 0, ctypes.byref(st)) is None and st.value == 2
    assert L.mflat_flat_create(-3, 0, ctypes.byref(st)) is None and st.value == 2
    # NULL handle / pointer checks come before any device work (c/mflat.cpp:110-129)
    f = np.zeros(4, np.float32)
    fp = f.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    assert L.mflat_flat_add(None, fp, 1) == 1
    assert L.mflat_flat_search(None, fp, 1, 1, None, None, None) == 1
    assert L.mflat_flat_reset(None) == 1
    assert L.mflat_flat_ready(None) == 0
    assert L.mflat_flat_size(None) == 0
    assert L.mflat_flat_dim(None) == 0
    h = L.mflat_flat_create(4, 0, ctypes.byref(st))
    assert h and st.value == 0
    try:
        assert L.mflat_flat_dim(h) == 4
        assert L.mflat_flat_add(h, None, 1) == 1
        assert L.mflat_flat_add(h, fp, -1) == 2
        assert L.mflat_flat_search(h, None, 1, 1, None, None, None) == 1
        assert L.mflat_flat_search(h, fp, -1, 1, None, None, None) == 2
        assert L.mflat_flat_search(h, fp, 1, 0, None, None, None) == 2
        used = ctypes.c_int(-1)
        # m == 0 is valid and produces nothing
        assert L.mflat_flat_search(h, fp, 0, 5, None, None, ctypes.byref(used)) == 0
        assert used.value == 0
        # the allocation-free entry takes a null query pointer when m == 0,
        # like the device layer, and still rejects it for m > 0
        used.value = -1
        assert L.mflat_flat_search_noalloc(h, None, 0, 5, None, None, ctypes.byref(used), None) == 0
        assert used.value == 0
        assert L.mflat_flat_search_noalloc(h, None, 1, 5, None, None, None, None) == 1
        assert L.mflat_flat_search_noalloc(None, None, 0, 5, None, None, None, None) == 1
        assert L.mflat_flat_set_shard(h, 2, 2, None, 0) == 2
    finally:
        L.mflat_flat_free(h)
    L.mflat_flat_free(None)


@pytest.mark.skipif(has_gpu(), reason="checks the no-device behaviour")
def test_no_cpu_fallback_without_device(built_lib):
    """Without a CUDA device the index is not ready and search reports a
    device error instead of silently computing on the CPU."""
    L = built_lib
    L.mflat_set_log_level(3)
    try:
        idx = M.FlatIndex(8)
        assert not idx.ready
        with pytest.raises(M.MflatError) as e:
            idx.search(np.zeros((2, 8), np.float32), 3)
        assert e.value.status == 6
        with pytest.raises(M.MflatError):
            idx.add(np.zeros((2, 8), np.float32))
    finally:
        L.mflat_set_log_level(0)


def test_log_level_and_handler_roundtrip(built_lib):
    L = built_lib
    seen = []

    @M.LOG_HANDLER
    def handler(level, msg, user):
        seen.append((level, msg.decode(), user))

    try:
        for lvl in (0, 1, 2, 3):
            L.mflat_set_log_level(lvl)
            assert L.mflat_log_level() == lvl
        L.mflat_set_log_level(0)
        L.mflat_set_log_handler(handler, ctypes.c_void_p(1234))
        if not has_gpu():
            M.FlatIndex(8)                      # logs "CUDA device unavailable"
            assert seen and seen[-1][0] == 2 and "CUDA" in seen[-1][1]
            assert seen[-1][2] == 1234
            assert not seen[-1][1].startswith("[metalflat]") and not seen[-1][1].endswith("\n")
            n = len(seen)
            L.mflat_set_log_level(3)            # Off drops everything
            M.FlatIndex(8)
            assert len(seen) == n
    finally:
        L.mflat_set_log_handler(M.LOG_HANDLER(0), None)
        L.mflat_set_log_level(0)


def test_kmeans_argument_checks(built_lib):
    L = built_lib
    f = np.zeros(8, np.float32)
    fp = f.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    o = np.zeros(2, np.int32)
    op = o.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))
    assert L.mflat_kmeans_assign(None, 2, fp, 1, 4, op, -1) == 1
    assert L.mflat_kmeans_assign(fp, -1, fp, 1, 4, op, -1) == 2
    assert L.mflat_kmeans_assign(fp, 2, fp, 0, 4, op, -1) == 2
    assert L.mflat_kmeans_assign(fp, 0, fp, 1, 4, op, -1) == 0   # nothing to assign


def test_persistence_argument_checks_without_device(built_lib, tmp_path):
    """save / load reject NULLs and unreadable or malformed files before any
    device work (the file header is checked first)."""
    L = built_lib
    st = ctypes.c_int(-1)
    assert L.mflat_flat_save(None, b"/tmp/x.mffl") == 1
    assert L.mflat_flat_load(None, -1, ctypes.byref(st)) is None and st.value == 1
    missing = str(tmp_path / "missing.mffl").encode()
    assert L.mflat_flat_load(missing, -1, ctypes.byref(st)) is None and st.value == 7
    bad = tmp_path / "bad.mffl"
    bad.write_bytes(b"not an index file at all, 32+ bytes long.......")
    assert L.mflat_flat_load(str(bad).encode(), -1, ctypes.byref(st)) is None and st.value == 7
    # right magic, unsupported version
    ver = tmp_path / "ver.mffl"
    ver.write_bytes(b"MFFL" + np.array([9, 4, 0, 0, 0, 0, 0], np.int32).tobytes())
    assert L.mflat_flat_load(str(ver).encode(), -1, ctypes.byref(st)) is None and st.value == 7
    # a valid header without a device: the handle cannot be made ready
    ok = tmp_path / "ok.mffl"
    ok.write_bytes(b"MFFL" + np.array([1, 4, 0, 0, 0, 0, 0], np.int32).tobytes())
    h = L.mflat_flat_load(str(ok).encode(), -1, ctypes.byref(st))
    if has_gpu():
        assert h and st.value == 0
        L.mflat_flat_free(h)
    else:
        assert h is None and st.value == 6


def test_coarse_argument_checks_without_device(built_lib):
    L = built_lib
    st = ctypes.c_int(-1)
    assert L.mflat_coarse_create(0, -1, ctypes.byref(st)) is None and st.value == 2
    h = L.mflat_coarse_create(8, -1, ctypes.byref(st))
    assert h and st.value == 0
    f = np.zeros(16, np.float32)
    fp = f.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    ip = np.zeros(16, np.int32).ctypes.data_as(ctypes.POINTER(ctypes.c_int32))
    assert L.mflat_coarse_train(None, fp, 2, 1, 1) == 1
    assert L.mflat_coarse_train(h, None, 2, 1, 1) == 1
    assert L.mflat_coarse_train(h, fp, 0, 1, 1) == 2
    assert L.mflat_coarse_train(h, fp, 2, 0, 1) == 2
    assert L.mflat_coarse_nlist(h) == 0 and L.mflat_coarse_size(h) == 0 and L.mflat_coarse_dim(h) == 8
    assert L.mflat_coarse_centroids(h, fp) == 4          # not trained yet
    assert L.mflat_coarse_csr(h, ip, ip) == 4
    assert L.mflat_coarse_probe(h, fp, 1, 1, ip) == 4
    assert L.mflat_coarse_probe(h, fp, 1, 0, ip) == 2
    L.mflat_coarse_free(h)
