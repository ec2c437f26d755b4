"""Python binding of the B200 exact k-NN engine (ctypes over the C ABI in
include/cuvs_b200.h).

Mirrors the reference's search interface for this path:
``cuvs::neighbors::cagra::build`` / ``search`` with a graph-less index
(include/cuvs/neighbors/cagra.hpp:94-106 of ysys143/cuvs-silicon) and the
``brute_force`` build/search pair the engine adds.  Argument errors raise
``ValueError`` (the reference throws ``std::invalid_argument``,
src/cagra.cpp:26-32,100-111); device and communication errors raise
``RuntimeError`` (src/metal_context.mm:146-147,245-246).

Inputs may be numpy arrays (host memory) or CUDA tensors exposing
``data_ptr()`` (device memory); results come back in the same kind of memory
the caller provides, or as new numpy arrays.

The compiled engine (lib/libcuvs_b200.so) is required; there is no CPU
fallback: importing this module on a machine without the library raises.
"""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libcuvs_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "cuvs_b200.h")

KNN_OK = 0
KNN_EINVAL = 1
KNN_ECUDA = 2
KNN_ENCCL = 3
KNN_ETIMEOUT = 4
KNN_ENOMEM = 5
KNN_EUNSUPPORTED = 6
DTYPE_F32 = 0
DTYPE_F16 = 1
METRIC_L2_EXPANDED = 0
METRIC_INNER_PRODUCT = 1
FILE_FVECS = 0
FILE_BIN_F32 = 1
NO_INDEX = 0xFFFFFFFF
MAX_K = 256


class KnnPlan(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in (
        "query_block", "query_tiles", "row_tiles", "splits", "units", "grid",
        "stages", "smem_bytes", "partial_bytes", "pair", "unit_queries",
        "compact_heap")]


_lib = None


def lib() -> ctypes.CDLL:
    """Loads lib/libcuvs_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build the CUDA engine first "
                           "(python -c 'import __graft_entry__ as g; g.build()')")
    L = ctypes.CDLL(LIB_PATH)
    P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    sig = {
        "knn_last_error": (ctypes.c_char_p, []),
        "knn_status_string": (ctypes.c_char_p, [I]),
        "knn_index_create": (I, [I, ctypes.POINTER(P)]),
        "knn_index_destroy": (I, [P]),
        "knn_index_set_stream": (I, [P, P]),
        "knn_index_build": (I, [P, P, I, I64, I64, I]),
        "knn_index_build_shard": (I, [P, P, I, I64, I64, I, I64, I64]),
        "knn_index_rows": (I64, [P]),
        "knn_index_dim": (I64, [P]),
        "knn_index_copy_rows": (I, [P, P, I]),
        "knn_index_search": (I, [P, P, I64, I64, P, P]),
        "knn_index_search_i64": (I, [P, P, I64, I64, P, P]),
        "knn_index_search_async": (I, [P, P, I64, I64, P, P]),
        "knn_index_sync": (I, [P]),
        "knn_plan_search": (I, [I64, I64, I64, I64, I, ctypes.POINTER(KnnPlan)]),
        "knn_shard_range": (I, [I64, I, I, ctypes.POINTER(I64), ctypes.POINTER(I64)]),
        "knn_comm_unique_id": (I, [P]),
        "knn_index_attach_comm": (I, [P, P, I, I]),
        "knn_index_set_profiling": (I, [P, I]),
        "knn_index_set_graphs": (I, [P, I]),
        "knn_index_set_peer_exchange": (I, [P, I]),
        "knn_index_set_peer_timeout": (I, [P, I64]),
        "knn_index_device": (I, [P]),
        "knn_index_device_rows": (I, [P, ctypes.POINTER(P), ctypes.POINTER(I64)]),
        "knn_index_device_norms": (I, [P, ctypes.POINTER(P)]),
        "knn_index_build_prepared": (I, [P, P, P, I64, I64, I, I64, I64]),
        "knn_index_search_lists": (I, [P, P, I64, I64, P, P]),
        "knn_merge_lists": (I, [I, P, P, P, I, I64, I64, I, P, I, P]),
        "knn_index_kernel_stats": (I, [P, ctypes.POINTER(ctypes.c_double),
                                       ctypes.POINTER(ctypes.c_double),
                                       ctypes.POINTER(I64), ctypes.POINTER(I64)]),
        "knn_index_reset_kernel_stats": (I, [P]),
        "knn_index_set_rerank": (I, [P, I]),
        "knn_index_build_file": (I, [P, ctypes.c_char_p, I, I, I, I]),
        "knn_rerank_bound": (ctypes.c_double, [I, ctypes.c_double, ctypes.c_double,
                                               ctypes.c_double, I64]),
        "knn_index_rerank_stats": (I, [P, ctypes.POINTER(I64), ctypes.POINTER(I64)]),
        "knn_index_search_noalloc": (I, [P, P, I64, I64, P, P]),
        "knn_selftest_bounded_wait": (I, [I, I64]),
        "knn_dispatch_count": (ctypes.c_uint64, []),
        "knn_reset_dispatch_count": (None, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def header_functions() -> list[str]:
    """Names of every function include/cuvs_b200.h declares."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(knn_[a-z0-9_]+)\s*\(", text)))


def _check(status: int) -> None:
    if status == KNN_OK:
        return
    msg = lib().knn_last_error().decode(errors="replace")
    name = lib().knn_status_string(status).decode()
    if status == KNN_EINVAL:
        raise ValueError(f"{name}: {msg}")
    raise RuntimeError(f"{name}: {msg}")


def plan_search(n_rows: int, dim: int, n_queries: int, k: int, num_sms: int = 148) -> dict:
    p = KnnPlan()
    _check(lib().knn_plan_search(n_rows, dim, n_queries, k, num_sms, ctypes.byref(p)))
    return {n: getattr(p, n) for n, _ in KnnPlan._fields_}


def shard_range(n_rows: int, n_ranks: int, rank: int) -> tuple[int, int]:
    b, e = ctypes.c_int64(), ctypes.c_int64()
    _check(lib().knn_shard_range(n_rows, n_ranks, rank, ctypes.byref(b), ctypes.byref(e)))
    return b.value, e.value


def comm_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    _check(lib().knn_comm_unique_id(buf))
    return buf.raw


def dispatch_count() -> int:
    return int(lib().knn_dispatch_count())


def reset_dispatch_count() -> None:
    lib().knn_reset_dispatch_count()


def _ptr(x):
    """(pointer, keepalive) for a numpy array or a tensor with data_ptr()."""
    if hasattr(x, "data_ptr"):
        if not x.is_contiguous():
            raise ValueError("tensors must be contiguous")
        return ctypes.c_void_p(x.data_ptr()), x
    a = np.ascontiguousarray(x)
    return ctypes.c_void_p(a.ctypes.data), a


def _shape(x):
    return tuple(int(s) for s in x.shape)


def _dtype_code(x) -> int:
    name = str(x.dtype)
    if name.endswith("float32"):
        return DTYPE_F32
    if name.endswith("float16"):
        return DTYPE_F16
    raise ValueError(f"dataset dtype {name} is not float32 or float16")


class Index:
    """Exact brute-force index on one B200 (or one row shard of a dataset).

    The index owns the fp16 rows and fp32 row norms in HBM (filled at build
    time); the reference computed them lazily at the first search and cached
    them by raw pointer (src/metal_context.mm:155-175).
    """

    def __init__(self, device: int = 0):
        h = ctypes.c_void_p()
        _check(lib().knn_index_create(device, ctypes.byref(h)))
        self._h = h
        self.device = device

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().knn_index_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def rows(self) -> int:
        return int(lib().knn_index_rows(self._h))

    @property
    def dim(self) -> int:
        return int(lib().knn_index_dim(self._h))

    def copy_rows(self, dtype=np.float32) -> np.ndarray:
        """The stored (fp16-rounded) rows, as a host array."""
        out = np.empty((self.rows, self.dim), dtype=dtype)
        code = DTYPE_F32 if out.dtype == np.float32 else DTYPE_F16
        _check(lib().knn_index_copy_rows(self._h, ctypes.c_void_p(out.ctypes.data), code))
        return out

    def set_stream(self, stream_handle: int | None) -> None:
        _check(lib().knn_index_set_stream(self._h, ctypes.c_void_p(stream_handle or 0)))

    def build(self, dataset, metric: int = METRIC_L2_EXPANDED, row_offset: int = 0,
              total_rows: int | None = None) -> "Index":
        if len(_shape(dataset)) != 2:
            raise ValueError("dataset must be 2-D")
        n, d = _shape(dataset)
        ptr, keep = _ptr(dataset)
        code = _dtype_code(keep)
        if row_offset == 0 and total_rows is None:
            _check(lib().knn_index_build(self._h, ptr, code, n, d, metric))
        else:
            total = n + row_offset if total_rows is None else total_rows
            _check(lib().knn_index_build_shard(self._h, ptr, code, n, d, metric,
                                               row_offset, total))
        return self

    def build_file(self, path: str, fmt: int = FILE_FVECS, metric: int = METRIC_L2_EXPANDED,
                   n_ranks: int = 1, rank: int = 0) -> None:
        """Streams a dataset file (FILE_FVECS or FILE_BIN_F32) into the index;
        with n_ranks > 1 only this rank's row shard is read."""
        _check(lib().knn_index_build_file(self._h, os.fsencode(path), fmt, metric,
                                          n_ranks, rank))

    def attach_comm(self, unique_id: bytes, n_ranks: int, rank: int) -> None:
        buf = ctypes.create_string_buffer(bytes(unique_id), 128)
        _check(lib().knn_index_attach_comm(self._h, buf, n_ranks, rank))

    def search(self, queries, k: int, neighbors=None, distances=None, int64: bool = False):
        """Exact k-NN; returns (neighbors, distances) of shape (n_queries, k)."""
        shp = _shape(queries)
        if len(shp) != 2:
            raise ValueError("queries must be 2-D")
        nq = shp[0]
        if neighbors is None:
            neighbors = np.empty((nq, k), dtype=np.int64 if int64 else np.uint32)
        if distances is None:
            distances = np.empty((nq, k), dtype=np.float32)
        if _shape(neighbors) != (nq, k) or _shape(distances) != (nq, k):
            # reference: src/cagra.cpp:107-111
            raise ValueError("output shape mismatch")
        if shp[1] != self.dim and self.rows > 0:
            # reference: src/cagra.cpp:104-106
            raise ValueError("query dimension mismatch")
        if not hasattr(queries, "data_ptr"):
            queries = np.ascontiguousarray(queries, dtype=np.float32)
        qp, qk = _ptr(queries)
        ip, ik = _ptr(neighbors)
        dp, dk = _ptr(distances)
        fn = lib().knn_index_search_i64 if int64 else lib().knn_index_search
        _check(fn(self._h, qp, nq, k, ip, dp))
        return neighbors, distances

    def search_async(self, queries, k: int, neighbors, distances) -> None:
        qp, _ = _ptr(queries)
        ip, _ = _ptr(neighbors)
        dp, _ = _ptr(distances)
        _check(lib().knn_index_search_async(self._h, qp, _shape(queries)[0], k, ip, dp))

    def sync(self) -> None:
        _check(lib().knn_index_sync(self._h))

    def set_rerank(self, on: bool) -> None:
        """Exact fp32 re-ranking (call before build; see knn_index_set_rerank)."""
        _check(lib().knn_index_set_rerank(self._h, 1 if on else 0))

    def rerank_stats(self) -> dict:
        """{'uncertified': queries of the last search not proven exact,
        'widened': queries searched again with more candidates}."""
        u, w = ctypes.c_int64(), ctypes.c_int64()
        _check(lib().knn_index_rerank_stats(self._h, ctypes.byref(u), ctypes.byref(w)))
        return {"uncertified": u.value, "widened": w.value}

    def set_peer_exchange(self, on: bool) -> None:
        _check(lib().knn_index_set_peer_exchange(self._h, 1 if on else 0))

    def set_peer_timeout(self, seconds: float) -> None:
        """Bound of the peer-exchange wait (every rank must issue each search
        within it of the others; see knn_index_set_peer_timeout)."""
        _check(lib().knn_index_set_peer_timeout(self._h, int(round(seconds * 1e6))))

    def set_graphs(self, on: bool) -> None:
        _check(lib().knn_index_set_graphs(self._h, 1 if on else 0))

    def set_profiling(self, on: bool) -> None:
        _check(lib().knn_index_set_profiling(self._h, 1 if on else 0))

    def kernel_stats(self) -> dict:
        a, b = ctypes.c_double(), ctypes.c_double()
        c, d = ctypes.c_int64(), ctypes.c_int64()
        _check(lib().knn_index_kernel_stats(self._h, ctypes.byref(a), ctypes.byref(b),
                                            ctypes.byref(c), ctypes.byref(d)))
        return {"scan_ms": a.value, "merge_ms": b.value, "scan_launches": c.value,
                "kernel_launches": d.value}

    def reset_kernel_stats(self) -> None:
        _check(lib().knn_index_reset_kernel_stats(self._h))


# ------------------------------------------------------------ dataset files
# numpy readers and writers of the formats knn_index_build_file streams and
# the C++ loaders (include/cuvs_silicon/sift_loader.hpp) read.

def write_fvecs(path: str, rows) -> None:
    rows = np.ascontiguousarray(rows, dtype=np.float32)
    rec = np.empty((rows.shape[0], rows.shape[1] + 1), dtype=np.float32)
    rec[:, 0] = np.array([rows.shape[1]], dtype=np.int32).view(np.float32)[0]
    rec[:, 1:] = rows
    rec.tofile(path)


def read_fvecs(path: str) -> np.ndarray:
    raw = np.fromfile(path, dtype=np.int32)
    if raw.size == 0:
        return np.empty((0, 0), np.float32)
    dim = int(raw[0])
    if dim <= 0 or raw.size % (dim + 1):
        raise ValueError(f"{path}: not an fvecs file")
    rec = raw.reshape(-1, dim + 1)
    if np.any(rec[:, 0] != dim):
        raise ValueError(f"{path}: rows of different widths")
    return rec[:, 1:].view(np.float32).copy()


def write_bin(path: str, matrix) -> None:
    m = np.ascontiguousarray(matrix)
    if m.dtype not in (np.float32, np.int32):
        raise ValueError("bin matrices hold float32 or int32")
    with open(path, "wb") as f:
        np.array(m.shape, dtype=np.int32).tofile(f)
        m.tofile(f)


def read_bin(path: str, dtype=np.float32) -> np.ndarray:
    raw = np.fromfile(path, dtype=np.int32)
    rows, cols = int(raw[0]), int(raw[1])
    if rows < 0 or cols < 0 or raw.size != 2 + rows * cols:
        raise ValueError(f"{path}: shape {rows} x {cols} does not match the file")
    return raw[2:].view(dtype).reshape(rows, cols).copy()


def rerank_bound(metric: int, r: float, query_norm: float, row_norm: float, dim: int) -> float:
    """The exact re-rank certificate's bound (knn_rerank_bound)."""
    return float(lib().knn_rerank_bound(metric, r, query_norm, row_norm, dim))
