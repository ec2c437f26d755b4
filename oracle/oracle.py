"""CPU oracle for the exact L2 k-NN path.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs
import this module, and only as the checker or the timed CPU baseline.  The
product library (``cuvs-silicon_b200``) never imports it and has no CPU
fallback.

Contents
--------
* Seeded input generators for the benchmark configurations: i.i.d. N(0, 1)
  rows, and the unit-norm Gaussian mixture (centres N(0, I), per-point noise
  sigma = 0.3, rows L2-normalised).  Rows are generated in 65,536-row chunks,
  chunk ``i`` from ``SeedSequence(seed, spawn_key=(i,))`` with PCG64, so any
  row range is reproducible on its own (used for row shards).
* ``round_fp16``: the device storage format.  numpy's float32 -> float16
  cast rounds to nearest even, the same rounding as the reference's
  ``(__fp16)`` casts at src/metal_context.mm:164-167,195-198 and the CUDA
  engine's ``__float2half_rn``.
* ``ref_knn``: the reference's own exact search (src/cagra.cpp:211-252)
  compiled unmodified into ``oracle/_ref/libref_cagra.so``.
* ``port_knn``: the C restatement in ``oracle/knn_oracle.c`` (bit-identical to
  ``ref_knn``; pinned against it and against the golden fixtures by tests).
* ``blas_knn``: the reference's expanded-form pattern
  ``|q|^2 - 2 q.x + |x|^2`` with ``cblas_sgemm`` (src/cagra.cpp:139-177),
  generalised from argmin to top-k.  numpy's float32 matmul calls the
  ``sgemm`` of numpy's bundled OpenBLAS in place of Apple Accelerate.
* ``check_parity``: the acceptance rule for the fp16 engine against the
  oracle, adjudicated with float64 distances on the fp16-rounded vectors.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
NO_INDEX = 0xFFFFFFFF
CHUNK_ROWS = 65536

# Seeds of the benchmark generators (configs 2-5 share the centres).
SEED_IID_BASE = 1
SEED_IID_QUERIES = 2
SEED_CENTRES = 11
SEED_BASE = 12
SEED_QUERIES = 13


# --------------------------------------------------------------------------
# generators
# --------------------------------------------------------------------------
def _chunk_rng(seed: int, chunk: int) -> np.random.Generator:
    return np.random.Generator(
        np.random.PCG64(np.random.SeedSequence(seed, spawn_key=(chunk,))))


def _chunks(begin: int, end: int):
    c0 = begin // CHUNK_ROWS
    c1 = (end - 1) // CHUNK_ROWS if end > begin else c0 - 1
    for c in range(c0, c1 + 1):
        lo = max(begin, c * CHUNK_ROWS)
        hi = min(end, (c + 1) * CHUNK_ROWS)
        yield c, lo, hi


def _run_chunks(begin, end, dim, fill, threads):
    out = np.empty((end - begin, dim), dtype=np.float32)

    def job(args):
        c, lo, hi = args
        block = fill(c)  # full chunk (rows of chunk c)
        out[lo - begin:hi - begin] = block[lo - c * CHUNK_ROWS:hi - c * CHUNK_ROWS]

    jobs = list(_chunks(begin, end))
    if threads > 1 and len(jobs) > 1:
        with ThreadPoolExecutor(threads) as ex:
            list(ex.map(job, jobs))
    else:
        for j in jobs:
            job(j)
    return out


def _chunk_len(c: int, total: int) -> int:
    return min(CHUNK_ROWS, total - c * CHUNK_ROWS)


def gen_iid(n: int, dim: int, seed: int, begin: int = 0, end: int | None = None,
            threads: int = 8) -> np.ndarray:
    """Rows [begin, end) of an n x dim matrix of i.i.d. N(0, 1) fp32."""
    end = n if end is None else end

    def fill(c):
        return _chunk_rng(seed, c).standard_normal(
            (_chunk_len(c, n), dim), dtype=np.float32)

    return _run_chunks(begin, end, dim, fill, threads)


def gen_centres(n_centres: int, dim: int, seed: int = SEED_CENTRES) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence(seed)))
    return rng.standard_normal((n_centres, dim), dtype=np.float32)


def gen_mixture(n: int, dim: int, n_centres: int, seed: int,
                begin: int = 0, end: int | None = None, sigma: float = 0.3,
                centres: np.ndarray | None = None, threads: int = 8) -> np.ndarray:
    """Rows [begin, end) of the unit-norm Gaussian mixture (fp32)."""
    end = n if end is None else end
    if centres is None:
        centres = gen_centres(n_centres, dim)

    def fill(c):
        rng = _chunk_rng(seed, c)
        rows = _chunk_len(c, n)
        u = rng.integers(0, n_centres, size=rows)
        x = rng.standard_normal((rows, dim), dtype=np.float32)
        x *= np.float32(sigma)
        x += centres[u]
        x /= np.linalg.norm(x, axis=1, keepdims=True).astype(np.float32)
        return x

    return _run_chunks(begin, end, dim, fill, threads)


def round_fp16(x: np.ndarray) -> np.ndarray:
    """fp32 -> fp16 (round to nearest even) -> fp32."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


# --------------------------------------------------------------------------
# native checkers
# --------------------------------------------------------------------------
_LIBS: dict[str, ctypes.CDLL] = {}


def build_native(quiet: bool = True) -> None:
    """Build oracle/_build/liboracle.so and, when the reference tree is
    present, oracle/_ref/libref_cagra.so."""
    kw = dict(stdout=subprocess.DEVNULL, stderr=subprocess.STDOUT) if quiet else {}
    subprocess.run(["make", "-C", HERE, "all"], check=True, **kw)


def _load(name: str, path: str) -> ctypes.CDLL:
    if name not in _LIBS:
        if not os.path.exists(path):
            build_native()
        _LIBS[name] = ctypes.CDLL(path)
    return _LIBS[name]


def port_lib() -> ctypes.CDLL:
    lib = _load("port", os.path.join(HERE, "_build", "liboracle.so"))
    lib.oracle_l2_knn.restype = ctypes.c_int
    lib.oracle_l2_knn.argtypes = [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int]
    lib.oracle_ip_knn.restype = ctypes.c_int
    lib.oracle_ip_knn.argtypes = lib.oracle_l2_knn.argtypes
    lib.oracle_merge_lists.restype = ctypes.c_int
    lib.oracle_merge_lists.argtypes = [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.oracle_squared_l2_128.restype = ctypes.c_float
    lib.oracle_squared_l2_128.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    return lib


def ref_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libref_cagra.so"))


def ref_lib() -> ctypes.CDLL:
    lib = _load("ref", os.path.join(HERE, "_ref", "libref_cagra.so"))
    lib.ref_cagra_knn.restype = ctypes.c_int
    lib.ref_cagra_knn.argtypes = [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int]
    lib.ref_cagra_build_inner_product.restype = ctypes.c_int
    lib.ref_cagra_build_inner_product.argtypes = [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64]
    lib.ref_cagra_save_index.restype = ctypes.c_int
    lib.ref_cagra_save_index.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_char_p]
    lib.ref_cagra_load_search.restype = ctypes.c_int
    lib.ref_cagra_load_search.argtypes = [
        ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64)]
    lib.ref_squared_l2_distance_128.restype = ctypes.c_float
    lib.ref_squared_l2_distance_128.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    lib.ref_last_error.restype = ctypes.c_char_p
    return lib


def _c(a: np.ndarray, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


def port_knn(base, queries, k, threads: int = 1, metric: int = 0):
    """C restatement (oracle/knn_oracle.c).  Returns (idx uint32, dist f32).

    metric 0: squared L2, ascending.  metric 1: inner product, descending
    (no reference counterpart: parity unpinned, see knn_oracle.c)."""
    base = _c(base, np.float32)
    queries = _c(queries, np.float32)
    n, dim = base.shape
    nq = queries.shape[0]
    idx = np.empty((nq, k), dtype=np.uint32)
    dist = np.empty((nq, k), dtype=np.float32)
    fn = port_lib().oracle_ip_knn if metric == 1 else port_lib().oracle_l2_knn
    rc = fn(base.ctypes.data, n, dim, queries.ctypes.data,
            nq, k, idx.ctypes.data, dist.ctypes.data, threads)
    if rc != 0:
        raise ValueError("oracle knn failed")
    return idx, dist


def ref_knn(base, queries, k, threads: int = 1):
    """The reference's own cagra::build + cagra::search (CPU exact path).

    With ``threads > 1`` the queries are split across threads, each calling the
    reference's public search on its slice (the reference search is
    re-entrant: it only reads the index).  Returns (idx uint32, dist f32).
    """
    base = _c(base, np.float32)
    queries = _c(queries, np.float32)
    n, dim = base.shape
    nq = queries.shape[0]
    idx = np.empty((nq, k), dtype=np.uint32)
    dist = np.empty((nq, k), dtype=np.float32)
    lib = ref_lib()

    def run(lo, hi):
        if hi <= lo:
            return 0
        return lib.ref_cagra_knn(base.ctypes.data, n, dim,
                                 queries[lo:hi].ctypes.data, hi - lo, k,
                                 idx[lo:hi].ctypes.data, dist[lo:hi].ctypes.data, 1)

    threads = max(1, min(threads, nq))
    if threads == 1:
        rcs = [run(0, nq)]
    else:
        # each slice is contiguous in the row-major outputs
        bounds = [(nq * t // threads, nq * (t + 1) // threads) for t in range(threads)]
        with ThreadPoolExecutor(threads) as ex:
            rcs = list(ex.map(lambda b: run(*b), bounds))
    if any(rcs):
        raise ValueError("reference search failed: "
                         + lib.ref_last_error().decode(errors="replace"))
    return idx, dist


def ref_save_index(base, path: str) -> None:
    """The reference's cagra::build + cagra::save_index (src/cagra.cpp:268-328)."""
    base = _c(base, np.float32)
    lib = ref_lib()
    if lib.ref_cagra_save_index(base.ctypes.data, base.shape[0], base.shape[1],
                                path.encode()) != 0:
        raise ValueError("reference save_index failed: "
                         + lib.ref_last_error().decode(errors="replace"))


def ref_load_search(path: str, queries, k):
    """The reference's cagra::load_index (src/cagra.cpp:330-366) and its exact
    search on the loaded index.  Returns (idx, dist, (rows, dim))."""
    queries = _c(queries, np.float32)
    nq = queries.shape[0]
    idx = np.empty((nq, k), dtype=np.uint32)
    dist = np.empty((nq, k), dtype=np.float32)
    rows, dim = ctypes.c_int64(), ctypes.c_int64()
    lib = ref_lib()
    if lib.ref_cagra_load_search(path.encode(), queries.ctypes.data, nq, k, idx.ctypes.data,
                                 dist.ctypes.data, ctypes.byref(rows), ctypes.byref(dim)) != 0:
        raise ValueError("reference load_index/search failed: "
                         + lib.ref_last_error().decode(errors="replace"))
    return idx, dist, (rows.value, dim.value)


def merge_lists(list_d, list_i, index_offset=None):
    """Oracle merge of per-part top-k lists shaped (nq, n_parts, k)."""
    list_d = _c(list_d, np.float32)
    list_i = _c(list_i, np.uint32)
    nq, n_parts, k = list_d.shape
    off = None if index_offset is None else _c(index_offset, np.int64)
    out_i = np.empty((nq, k), dtype=np.uint32)
    out_d = np.empty((nq, k), dtype=np.float32)
    rc = port_lib().oracle_merge_lists(
        list_d.ctypes.data, list_i.ctypes.data, nq, n_parts, k,
        None if off is None else off.ctypes.data, out_i.ctypes.data, out_d.ctypes.data)
    if rc != 0:
        raise ValueError("oracle_merge_lists failed")
    return out_i, out_d


def blas_knn(base, queries, k, chunk_rows: int = 65536):
    """Expanded-form search |q|^2 - 2 q.x + |x|^2 through OpenBLAS sgemm
    (numpy float32 matmul), chunked over the base rows, top-k by
    (distance, index).  Restates the cblas_sgemm pattern of
    src/cagra.cpp:139-177 (argmin there) generalised to top-k."""
    base = _c(base, np.float32)
    queries = _c(queries, np.float32)
    n = base.shape[0]
    nq = queries.shape[0]
    qn = np.einsum("ij,ij->i", queries, queries)
    best_d = np.full((nq, 0), np.inf, dtype=np.float32)
    best_i = np.zeros((nq, 0), dtype=np.int64)
    for lo in range(0, n, chunk_rows):
        x = base[lo:lo + chunk_rows]
        xn = np.einsum("ij,ij->i", x, x)
        d = queries @ x.T  # sgemm
        d *= -2.0
        d += qn[:, None]
        d += xn[None, :]
        kk = min(k, d.shape[1])
        part = np.argpartition(d, kk - 1, axis=1)[:, :kk] if kk < d.shape[1] else \
            np.tile(np.arange(d.shape[1]), (nq, 1))
        cd = np.take_along_axis(d, part, axis=1)
        ci = part + lo
        all_d = np.concatenate([best_d, cd], axis=1)
        all_i = np.concatenate([best_i, ci], axis=1)
        order = np.lexsort((all_i, all_d), axis=1)[:, :k]
        best_d = np.take_along_axis(all_d, order, axis=1)
        best_i = np.take_along_axis(all_i, order, axis=1)
    out_i = np.full((nq, k), NO_INDEX, dtype=np.uint32)
    out_d = np.full((nq, k), np.inf, dtype=np.float32)
    m = best_d.shape[1]
    out_i[:, :m] = best_i.astype(np.uint32)
    out_d[:, :m] = best_d
    return out_i, out_d


def blas_threads() -> str:
    try:
        cfg = np.show_config(mode="dicts")
        blas = cfg.get("Build Dependencies", {}).get("blas", {})
        return f"{blas.get('name', '?')} {blas.get('version', '?')}"
    except Exception:  # pragma: no cover - informational only
        return "unknown"


# --------------------------------------------------------------------------
# parity
# --------------------------------------------------------------------------
@dataclass
class Parity:
    ok: bool
    n_index_mismatch: int
    n_tol_violation: int
    recall: float
    max_rel_dist_err: float
    sorted_ok: bool
    padding_ok: bool
    detail: str = ""


def exact_dist64(base16: np.ndarray, queries16: np.ndarray, idx: np.ndarray) -> np.ndarray:
    """float64 squared L2 between each query and the rows it lists (fp16-
    rounded inputs).  Invalid indices give +inf."""
    nq, k = idx.shape
    out = np.full((nq, k), np.inf, dtype=np.float64)
    valid = idx != NO_INDEX
    for q in range(nq):
        rows = idx[q][valid[q]].astype(np.int64)
        if rows.size:
            diff = base16[rows].astype(np.float64) - queries16[q].astype(np.float64)
            out[q, valid[q]] = np.einsum("ij,ij->i", diff, diff)
    return out


def check_parity(base16, queries16, got_i, got_d, ora_i, ora_d,
                 rel_tol: float = 1e-3, eps: float = 1e-6) -> Parity:
    with np.errstate(invalid="ignore"):  # inf - inf of padding slots (masked)
        return _check_parity(base16, queries16, got_i, got_d, ora_i, ora_d, rel_tol, eps)


def _check_parity(base16, queries16, got_i, got_d, ora_i, ora_d,
                  rel_tol: float, eps: float) -> Parity:
    """Acceptance rule of the fp16 engine against the oracle.

    * rank by rank, the index equals the oracle's, or the float64 distances of
      the two indices differ by at most rel_tol * max(D_oracle, eps);
    * recall@k = 1 where a returned row counts as a hit if its float64
      distance is <= the oracle's k-th distance * (1 + rel_tol) + eps
      (tie-aware at the boundary), and no index is repeated;
    * returned distances are within rel_tol (abs eps near 0) of float64;
    * output sorted ascending; slots beyond n padded with UINT32_MAX / +inf.
    """
    got_i = np.asarray(got_i, dtype=np.uint32)
    ora_i = np.asarray(ora_i, dtype=np.uint32)
    got_d = np.asarray(got_d, dtype=np.float32)
    nq, k = ora_i.shape
    D_o = exact_dist64(base16, queries16, ora_i)
    D_g = exact_dist64(base16, queries16, got_i)
    pad_o = ora_i == NO_INDEX
    pad_g = got_i == NO_INDEX
    padding_ok = bool(np.array_equal(pad_o, pad_g)) and bool(
        np.all(np.isinf(got_d[pad_g]))) if pad_g.any() or pad_o.any() else bool(
        np.array_equal(pad_o, pad_g))
    mism = (got_i != ora_i) & ~pad_o
    both = ~pad_o & ~pad_g
    scale = np.maximum(np.where(np.isfinite(D_o), D_o, 0.0), eps)
    tol_bad = mism & both & (np.abs(D_g - D_o) > rel_tol * scale)
    tol_bad |= mism & (pad_o != pad_g)
    # recall (tie-aware)
    hits = 0
    total = 0
    for q in range(nq):
        valid = ~pad_o[q]
        m = int(valid.sum())
        if m == 0:
            continue
        kth = D_o[q][valid].max()
        g = got_i[q][~pad_g[q]]
        gd = D_g[q][~pad_g[q]]
        uniq = len(set(g.tolist())) == len(g)
        h = int(np.sum(gd <= kth * (1 + rel_tol) + eps)) if uniq else 0
        hits += min(h, m)
        total += m
    recall = hits / total if total else 1.0
    # distance accuracy
    fin = both & np.isfinite(D_g)
    derr = np.abs(got_d.astype(np.float64) - D_g)
    dscale = np.maximum(D_g, eps)
    rel = np.where(fin, derr / np.maximum(dscale, 1e-30), 0.0)
    dist_ok = bool(np.all((derr[fin] <= rel_tol * D_g[fin]) | (derr[fin] <= 1e-4)))
    max_rel = float(rel[fin].max()) if fin.any() else 0.0
    # sortedness
    sorted_ok = True
    for q in range(nq):
        v = got_d[q][~pad_g[q]]
        if np.any(np.diff(v) < 0):
            sorted_ok = False
            break
    ok = (not tol_bad.any()) and recall == 1.0 and dist_ok and sorted_ok and padding_ok
    detail = (f"idx_mismatch={int(mism.sum())} tol_violation={int(tol_bad.sum())} "
              f"recall={recall:.6f} max_rel_dist_err={max_rel:.3e} dist_ok={dist_ok} "
              f"sorted={sorted_ok} padding={padding_ok}")
    return Parity(ok, int(mism.sum()), int(tol_bad.sum()), recall, max_rel,
                  sorted_ok, padding_ok, detail)


def check_parity_ip(base16, queries16, got_i, got_d, ora_i, ora_d,
                    rel_tol: float = 1e-3) -> Parity:
    with np.errstate(invalid="ignore"):  # inf - inf of padding slots (masked)
        return _check_parity_ip(base16, queries16, got_i, got_d, ora_i, ora_d, rel_tol)


def _check_parity_ip(base16, queries16, got_i, got_d, ora_i, ora_d,
                     rel_tol: float) -> Parity:
    """Acceptance rule for the inner-product metric (scores, largest first).

    Scores are float64 dot products of the fp16-rounded vectors.  The error
    scale of a score is s_q = |q| * max_x |x| (Cauchy-Schwarz bound of any
    score of q), and:
    * rank by rank, the index equals the oracle's, or the two scores differ
      by at most rel_tol * s_q;
    * recall@k = 1 where a returned row counts as a hit if its score is
      >= the oracle's k-th score - rel_tol * s_q, and no index repeats;
    * returned scores are within rel_tol * s_q of float64;
    * output sorted descending; slots beyond n padded with UINT32_MAX / -inf.
    """
    got_i = np.asarray(got_i, dtype=np.uint32)
    ora_i = np.asarray(ora_i, dtype=np.uint32)
    got_d = np.asarray(got_d, dtype=np.float32)
    nq, k = ora_i.shape
    b64 = base16.astype(np.float64)
    q64 = queries16.astype(np.float64)
    xmax = float(np.sqrt((b64 * b64).sum(1)).max()) if len(b64) else 0.0
    s_q = np.maximum(np.sqrt((q64 * q64).sum(1)) * xmax, 1e-30)

    def scores(idx):
        out = np.full(idx.shape, -np.inf)
        for q in range(nq):
            v = idx[q] != NO_INDEX
            if v.any():
                out[q, v] = b64[idx[q][v].astype(np.int64)] @ q64[q]
        return out

    S_o, S_g = scores(ora_i), scores(got_i)
    pad_o, pad_g = ora_i == NO_INDEX, got_i == NO_INDEX
    padding_ok = bool(np.array_equal(pad_o, pad_g)) and bool(
        np.all(np.isneginf(got_d[pad_g])))
    mism = (got_i != ora_i) & ~pad_o
    both = ~pad_o & ~pad_g
    tol = rel_tol * s_q[:, None]
    tol_bad = (mism & both & (np.abs(S_g - S_o) > tol)) | (mism & (pad_o != pad_g))
    hits = total = 0
    for q in range(nq):
        m = int((~pad_o[q]).sum())
        if m == 0:
            continue
        kth = S_o[q][~pad_o[q]].min()
        g = got_i[q][~pad_g[q]]
        uniq = len(set(g.tolist())) == len(g)
        h = int(np.sum(S_g[q][~pad_g[q]] >= kth - tol[q, 0])) if uniq else 0
        hits += min(h, m)
        total += m
    recall = hits / total if total else 1.0
    derr = np.where(both, np.abs(got_d.astype(np.float64) - np.where(both, S_g, 0.0)), 0.0)
    dist_ok = bool(np.all(derr <= tol))
    max_rel = float((derr / tol).max() * rel_tol) if both.any() else 0.0
    sorted_ok = all(not np.any(np.diff(got_d[q][~pad_g[q]]) > 0) for q in range(nq))
    ok = (not tol_bad.any()) and recall == 1.0 and dist_ok and sorted_ok and padding_ok
    detail = (f"idx_mismatch={int(mism.sum())} tol_violation={int(tol_bad.sum())} "
              f"recall={recall:.6f} max_score_err/s_q={max_rel:.3e} dist_ok={dist_ok} "
              f"sorted={sorted_ok} padding={padding_ok}")
    return Parity(ok, int(mism.sum()), int(tol_bad.sum()), recall, max_rel,
                  sorted_ok, padding_ok, detail)


if __name__ == "__main__":  # pragma: no cover
    build_native(quiet=False)
    print("oracle libraries built", file=sys.stderr)
