"""Python binding over the C ABI of include/mflat.h (libmetalflat_c.so).

A thin ctypes layer, the kind of FFI binding the reference's C ABI is meant
for ("Python / Swift / other bindings", reference CMakeLists.txt:38).  It
calls the in-tree library only; when that library is missing or cannot load
it raises, there is no fallback implementation.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_DIR = os.path.join(PKG, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libmetalflat_c.so")
CUDA_LIB_PATH = os.path.join(LIB_DIR, "libmflat_cuda.so")

METRICS = {"l2": 0, "ip": 1, "inner_product": 1, "cosine": 2}
STORAGES = {"fp32": 0, "fp16": 1, "bf16": 2}
STATUS = {0: "ok", 1: "null argument", 2: "bad argument", 3: "allocation failed",
          4: "index not built", 5: "internal error", 6: "device error", 7: "index file error"}

EXPORTS = [
    "mflat_version", "mflat_status_str", "mflat_max_k",
    "mflat_set_log_handler", "mflat_set_log_level", "mflat_log_level",
    "mflat_flat_create", "mflat_flat_free", "mflat_flat_ready", "mflat_flat_size",
    "mflat_flat_dim", "mflat_flat_add", "mflat_flat_reset", "mflat_flat_search",
    "mflat_flat_create_ex", "mflat_flat_storage", "mflat_flat_device",
    "mflat_flat_add_device", "mflat_flat_search_device", "mflat_flat_set_timing",
    "mflat_flat_last_timing", "mflat_flat_timing_sum", "mflat_kmeans_assign", "mflat_kmeans_assign_device",
    "mflat_comm_unique_id", "mflat_flat_set_shard", "mflat_flat_search_noalloc",
    "mflat_flat_save", "mflat_flat_load",
    "mflat_coarse_create", "mflat_coarse_free", "mflat_coarse_train", "mflat_coarse_nlist",
    "mflat_coarse_size", "mflat_coarse_dim", "mflat_coarse_centroids", "mflat_coarse_csr",
    "mflat_coarse_probe", "mflat_coarse_set_shard",
]


class MflatError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        super().__init__(f"{what}: {STATUS.get(status, status)} ({status})")
        self.status = status


class Timing(ctypes.Structure):
    _fields_ = [("total_ms", ctypes.c_float), ("screen_ms", ctypes.c_float),
                ("select_ms", ctypes.c_float), ("screen_launches", ctypes.c_int),
                ("launches", ctypes.c_int), ("fallback_queries", ctypes.c_int)]


LOG_HANDLER = ctypes.CFUNCTYPE(None, ctypes.c_int, ctypes.c_char_p, ctypes.c_void_p)

_lib = None


def lib() -> ctypes.CDLL:
    """Load libmetalflat_c.so (raises OSError when it is not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise OSError(f"{LIB_PATH} is not built; run __graft_entry__.build() or make -C metal-flat_b200")
    L = ctypes.CDLL(LIB_PATH)
    vp, ci, cf = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    i32p = ctypes.POINTER(ctypes.c_int32)
    f32p = ctypes.POINTER(ctypes.c_float)
    sig = {
        "mflat_version": ([], ctypes.c_char_p),
        "mflat_status_str": ([ci], ctypes.c_char_p),
        "mflat_max_k": ([], ci),
        "mflat_set_log_handler": ([LOG_HANDLER, vp], None),
        "mflat_set_log_level": ([ci], None),
        "mflat_log_level": ([], ci),
        "mflat_flat_create": ([ci, ci, ctypes.POINTER(ci)], vp),
        "mflat_flat_create_ex": ([ci, ci, ci, ci, ctypes.POINTER(ci)], vp),
        "mflat_flat_free": ([vp], None),
        "mflat_flat_ready": ([vp], ci),
        "mflat_flat_size": ([vp], ci),
        "mflat_flat_dim": ([vp], ci),
        "mflat_flat_storage": ([vp], ci),
        "mflat_flat_device": ([vp], ci),
        "mflat_flat_add": ([vp, f32p, ci], ci),
        "mflat_flat_add_device": ([vp, vp, ci, vp], ci),
        "mflat_flat_reset": ([vp], ci),
        "mflat_flat_search": ([vp, f32p, ci, ci, i32p, f32p, ctypes.POINTER(ci)], ci),
        "mflat_flat_search_device": ([vp, vp, ci, ci, vp, vp, ctypes.POINTER(ci), vp], ci),
        "mflat_flat_search_noalloc": ([vp, vp, ci, ci, vp, vp, ctypes.POINTER(ci), vp], ci),
        "mflat_flat_set_timing": ([vp, ci], ci),
        "mflat_flat_last_timing": ([vp, ctypes.POINTER(Timing)], ci),
        "mflat_flat_timing_sum": ([vp, ctypes.POINTER(Timing), ctypes.POINTER(ci)], ci),
        "mflat_kmeans_assign": ([f32p, ci, f32p, ci, ci, i32p, ci], ci),
        "mflat_kmeans_assign_device": ([vp, ci, vp, ci, ci, vp, ci, vp], ci),
        "mflat_comm_unique_id": ([ctypes.c_char_p], ci),
        "mflat_flat_set_shard": ([vp, ci, ci, ctypes.c_char_p, ctypes.c_int64], ci),
        "mflat_flat_save": ([vp, ctypes.c_char_p], ci),
        "mflat_flat_load": ([ctypes.c_char_p, ci, ctypes.POINTER(ci)], vp),
        "mflat_coarse_create": ([ci, ci, ctypes.POINTER(ci)], vp),
        "mflat_coarse_free": ([vp], None),
        "mflat_coarse_train": ([vp, f32p, ci, ci, ci], ci),
        "mflat_coarse_nlist": ([vp], ci),
        "mflat_coarse_size": ([vp], ci),
        "mflat_coarse_dim": ([vp], ci),
        "mflat_coarse_centroids": ([vp, f32p], ci),
        "mflat_coarse_csr": ([vp, i32p, i32p], ci),
        "mflat_coarse_probe": ([vp, f32p, ci, ci, i32p], ci),
        "mflat_coarse_set_shard": ([vp, ci, ci, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64)], ci),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a, t):
    return a.ctypes.data_as(ctypes.POINTER(t))


def _check(st: int, what: str) -> None:
    if st != 0:
        raise MflatError(st, what)


def version() -> str:
    return lib().mflat_version().decode()


def max_k() -> int:
    return lib().mflat_max_k()


def comm_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    _check(lib().mflat_comm_unique_id(buf), "comm_unique_id")
    return buf.raw


def _out_array(a, n: int, dt, name: str) -> np.ndarray:
    """A caller-owned result buffer: writeable, C-contiguous, dtype dt, >= n entries."""
    if (not isinstance(a, np.ndarray) or a.dtype != dt or not a.flags.c_contiguous
            or not a.flags.writeable):
        raise ValueError(f"out {name}: a writeable C-contiguous {np.dtype(dt).name} array is required")
    if a.size < n:
        raise ValueError(f"out {name}: {a.size} entries, the call needs {n}")
    return a.reshape(-1)


def kmeans_assign(points, centroids, device: int = -1, out=None) -> np.ndarray:
    """Nearest centroid of each point (bit-exact fp32 sqL2, lowest index on
    ties).  out: optional caller-owned int32 buffer of >= n entries."""
    p, c = _f32(points), _f32(centroids)
    out = (np.empty(p.shape[0], np.int32) if out is None
           else _out_array(out, p.shape[0], np.int32, "assign")[: p.shape[0]])
    _check(lib().mflat_kmeans_assign(_ptr(p, ctypes.c_float), p.shape[0], _ptr(c, ctypes.c_float),
                                     c.shape[0], p.shape[1], _ptr(out, ctypes.c_int32), device),
           "kmeans_assign")
    return out


class FlatIndex:
    """Exact flat index on one GPU (the reference's FlatIndex through the C ABI)."""

    def __init__(self, dim: int, metric: str | int = "l2", storage: str | int = "fp32",
                 device: int = -1):
        L = lib()
        m = METRICS[metric] if isinstance(metric, str) else int(metric)
        s = STORAGES[storage] if isinstance(storage, str) else int(storage)
        st = ctypes.c_int(0)
        self._h = L.mflat_flat_create_ex(int(dim), m, s, int(device), ctypes.byref(st))
        if not self._h:
            raise MflatError(st.value, "create")
        self._lib = L
        self.metric = m

    @classmethod
    def load(cls, path: str, device: int = -1) -> "FlatIndex":
        """A new index holding the rows of a file written by save()."""
        L = lib()
        st = ctypes.c_int(0)
        h = L.mflat_flat_load(os.fsencode(path), int(device), ctypes.byref(st))
        if not h:
            raise MflatError(st.value, f"load {path}")
        self = cls.__new__(cls)
        self._h, self._lib = h, L
        self.metric = None
        return self

    def save(self, path: str) -> None:
        _check(self._lib.mflat_flat_save(self._h, os.fsencode(path)), f"save {path}")

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.mflat_flat_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    @property
    def ready(self) -> bool:
        return bool(self._lib.mflat_flat_ready(self._h))

    @property
    def size(self) -> int:
        return self._lib.mflat_flat_size(self._h)

    @property
    def dim(self) -> int:
        return self._lib.mflat_flat_dim(self._h)

    @property
    def device(self) -> int:
        return self._lib.mflat_flat_device(self._h)

    @property
    def storage(self) -> int:
        return self._lib.mflat_flat_storage(self._h)

    def add(self, vectors) -> None:
        v = _f32(vectors)
        n = v.shape[0] if v.ndim == 2 else 0
        _check(self._lib.mflat_flat_add(self._h, _ptr(v, ctypes.c_float), n), "add")

    def add_device(self, ptr: int, n: int, stream: int = 0) -> None:
        _check(self._lib.mflat_flat_add_device(self._h, ctypes.c_void_p(ptr), n,
                                               ctypes.c_void_p(stream)), "add_device")

    def reset(self) -> None:
        _check(self._lib.mflat_flat_reset(self._h), "reset")

    def search(self, queries, k: int, out=None):
        """Top-k rows of each query: (ids, dist), each m x k_used (nearest first).

        out: optional (ids, dist) pair of caller-owned, writeable, C-contiguous
        int32 / float32 arrays with room for m * k entries (the C ABI's output
        contract).  The results are written there and views of them returned,
        so a caller can reuse (for example page-locked) buffers across calls.
        """
        q = _f32(queries)
        m = q.shape[0]
        cap = max(1, m * max(1, k))
        if out is None:
            ids = np.empty(cap, np.int32)
            dist = np.empty(cap, np.float32)
        else:
            ids = _out_array(out[0], cap, np.int32, "ids")
            dist = _out_array(out[1], cap, np.float32, "dist")
        used = ctypes.c_int(0)
        _check(self._lib.mflat_flat_search(self._h, _ptr(q, ctypes.c_float), m, k,
                                           _ptr(ids, ctypes.c_int32), _ptr(dist, ctypes.c_float),
                                           ctypes.byref(used)), "search")
        ku = used.value
        return ids[: m * ku].reshape(m, ku), dist[: m * ku].reshape(m, ku)

    def search_device(self, q_ptr: int, m: int, k: int, ids_ptr: int, dist_ptr: int,
                      stream: int = 0) -> int:
        used = ctypes.c_int(0)
        _check(self._lib.mflat_flat_search_device(self._h, ctypes.c_void_p(q_ptr), m, k,
                                                  ctypes.c_void_p(ids_ptr),
                                                  ctypes.c_void_p(dist_ptr), ctypes.byref(used),
                                                  ctypes.c_void_p(stream)), "search_device")
        return used.value

    def search_noalloc(self, q_ptr: int, m: int, k: int, ids_ptr: int, dist_ptr: int,
                       stream: int = 0) -> int:
        """Device-pointer search that allocates no device memory (m <= 128,
        dim <= 128, k <= 21); see mflat_flat_search_noalloc in include/mflat.h."""
        used = ctypes.c_int(0)
        _check(self._lib.mflat_flat_search_noalloc(self._h, ctypes.c_void_p(q_ptr), m, k,
                                                   ctypes.c_void_p(ids_ptr),
                                                   ctypes.c_void_p(dist_ptr), ctypes.byref(used),
                                                   ctypes.c_void_p(stream)), "search_noalloc")
        return used.value

    def set_timing(self, on: bool = True) -> None:
        _check(self._lib.mflat_flat_set_timing(self._h, 1 if on else 0), "set_timing")

    def last_timing(self) -> Timing:
        t = Timing()
        _check(self._lib.mflat_flat_last_timing(self._h, ctypes.byref(t)), "last_timing")
        return t

    def timing_sum(self) -> tuple[Timing, int]:
        """(field-wise sums, number of searches) since set_timing(True)."""
        t = Timing()
        n = ctypes.c_int(0)
        _check(self._lib.mflat_flat_timing_sum(self._h, ctypes.byref(t), ctypes.byref(n)),
               "timing_sum")
        return t, n.value

    def set_shard(self, rank: int, world: int, comm_id: bytes | None, id_base: int) -> None:
        _check(self._lib.mflat_flat_set_shard(self._h, rank, world, comm_id, int(id_base)),
               "set_shard")


class CoarseQuantizer:
    """IVF coarse layer (k-means train, CSR scaffold, cell probing) through the C ABI."""

    def __init__(self, dim: int, device: int = -1):
        L = lib()
        st = ctypes.c_int(0)
        self._h = L.mflat_coarse_create(int(dim), int(device), ctypes.byref(st))
        if not self._h:
            raise MflatError(st.value, "coarse create")
        self._lib = L

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.mflat_coarse_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    @property
    def nlist(self) -> int:
        return self._lib.mflat_coarse_nlist(self._h)

    @property
    def size(self) -> int:
        return self._lib.mflat_coarse_size(self._h)

    @property
    def dim(self) -> int:
        return self._lib.mflat_coarse_dim(self._h)

    def set_shard(self, rank: int, world: int, comm_id: bytes | None, row_offsets) -> None:
        """This handle holds global rows [row_offsets[rank], row_offsets[rank + 1])."""
        off = np.ascontiguousarray(row_offsets, dtype=np.int64)
        _check(self._lib.mflat_coarse_set_shard(self._h, int(rank), int(world), comm_id,
                                                _ptr(off, ctypes.c_int64)), "coarse set_shard")

    def train(self, data, nlist: int, iters: int = 12) -> None:
        d = _f32(data)
        n = d.shape[0] if d.ndim == 2 else 0
        _check(self._lib.mflat_coarse_train(self._h, _ptr(d, ctypes.c_float), n, int(nlist),
                                            int(iters)), "coarse train")

    def centroids(self) -> np.ndarray:
        out = np.empty((self.nlist, self.dim), np.float32)
        _check(self._lib.mflat_coarse_centroids(self._h, _ptr(out, ctypes.c_float)), "coarse centroids")
        return out

    def csr(self):
        cs = np.empty(self.nlist + 1, np.int32)
        ro = np.empty(self.size, np.int32)
        _check(self._lib.mflat_coarse_csr(self._h, _ptr(cs, ctypes.c_int32), _ptr(ro, ctypes.c_int32)),
               "coarse csr")
        return cs, ro

    def probe(self, queries, nprobe: int) -> np.ndarray:
        q = _f32(queries)
        out = np.empty((q.shape[0], nprobe), np.int32)
        _check(self._lib.mflat_coarse_probe(self._h, _ptr(q, ctypes.c_float), q.shape[0], int(nprobe),
                                            _ptr(out, ctypes.c_int32)), "coarse probe")
        return out
