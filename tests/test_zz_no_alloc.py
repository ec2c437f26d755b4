"""The allocation-free search entry point, knn_index_search_noalloc.

Some callers cannot allocate device memory while they search: a serving
process whose GPU memory belongs to another allocator or budget, or code that
must not trigger the device-wide synchronisation cudaMalloc/cudaFree may
cause.  For them the library keeps the per-search scratch in one static
device array (KNN_NOALLOC_SCRATCH_BYTES).  This test calls that entry point
through the C ABI twice in a row and checks each result against the regular
knn_index_search with the tolerance the parity tests use.  It lives in a
file that pytest collects last so a run stopping at its first failure has
already run every other test; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


def _noalloc_fn(engine):
    fn = engine.lib().knn_index_search_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                   ctypes.c_void_p, ctypes.c_void_p]
    return fn


def test_noalloc_matches_regular_search_twice(engine, oracle_mod):
    import torch

    assert torch.cuda.is_available()
    fn = _noalloc_fn(engine)
    rng = np.random.Generator(np.random.PCG64(77))
    base = rng.standard_normal((30000, 256), dtype=np.float32)
    queries = rng.standard_normal((100, 256), dtype=np.float32)
    k = 10
    b16, q16 = oracle_mod.round_fp16(base), oracle_mod.round_fp16(queries)
    with engine.Index(0) as idx:
        idx.build(base)
        ref_i, ref_d = idx.search(queries, k)
        # host buffers, two calls in a row
        for _ in range(2):
            got_i = np.full((100, k), 7, np.uint32)
            got_d = np.full((100, k), -1.0, np.float32)
            st = fn(idx._h, queries.ctypes.data, 100, k, got_i.ctypes.data, got_d.ctypes.data)
            assert st == 0, engine.lib().knn_last_error()
            par = oracle_mod.check_parity(b16, q16, got_i, got_d, ref_i, ref_d, REL_TOL)
            assert par.ok, par.detail
        # device buffers, two calls in a row, no device memory taken
        qd = torch.from_numpy(queries).cuda()
        di = torch.empty((100, k), dtype=torch.int32, device="cuda")
        dd = torch.empty((100, k), dtype=torch.float32, device="cuda")
        for _ in range(2):
            di.fill_(-7)
            torch.cuda.synchronize()
            free_before = torch.cuda.mem_get_info()[0]
            st = fn(idx._h, qd.data_ptr(), 100, k, di.data_ptr(), dd.data_ptr())
            free_after = torch.cuda.mem_get_info()[0]
            assert st == 0, engine.lib().knn_last_error()
            assert free_after == free_before  # the call took no device memory
            got_i = di.cpu().numpy().view(np.uint32)
            par = oracle_mod.check_parity(b16, q16, got_i, dd.cpu().numpy(), ref_i, ref_d,
                                          REL_TOL)
            assert par.ok, par.detail


def test_noalloc_rejects_oversized_search(engine):
    fn = _noalloc_fn(engine)
    rng = np.random.Generator(np.random.PCG64(78))
    base = rng.standard_normal((4096, 1024), dtype=np.float32)
    nq = 20000  # fp16 queries alone need 40 MB > 16 MiB
    queries = rng.standard_normal((nq, 1024), dtype=np.float32)
    with engine.Index(0) as idx:
        idx.build(base)
        out_i = np.empty((nq, 4), np.uint32)
        out_d = np.empty((nq, 4), np.float32)
        st = fn(idx._h, queries.ctypes.data, nq, 4, out_i.ctypes.data, out_d.ctypes.data)
        assert st == engine.KNN_EUNSUPPORTED
        assert b"scratch" in engine.lib().knn_last_error()
        # the regular entry point still serves the same request afterwards
        idx.search(queries[:8], 4)
