"""Runs searches through the bounds-checked debug engine
(cuvs-silicon_b200/lib/libcuvs_b200_debug.so, built with KNN_DEBUG_BOUNDS=1).

Every index the debug kernels compute is checked before the access it
guards; a failed check records an error code that the search reports as
KNN_ECUDA (RuntimeError here), so a search that returns at all stayed in
bounds.  The shapes cover what the kernels index differently: dimensions
below, at and above the 64-wide slice and not multiples of 8, datasets
smaller than one granule, ragged last tiles, k above the row count
(padding), the register top-k (k <= 16), the heap (k > 16) with the pilot
pass (k >= 17), several query tiles, CTA pairs (more than 128 queries with
k >= 62), the inner product, exact re-ranking,
the search without allocation, host and device buffers and graph replay.
Results are checked against the oracle too.  Exit code 0 = pass.
Run in its own process: the binding loads one engine library per process.
"""
import ctypes
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "cuvs-silicon_b200"))


def main():
    import torch

    import cuvs_b200 as E
    import oracle as O

    E.LIB_PATH = os.path.join(ROOT, "cuvs-silicon_b200", "lib", "libcuvs_b200_debug.so")
    assert os.path.exists(E.LIB_PATH), E.LIB_PATH
    E.lib()
    rng = np.random.Generator(np.random.PCG64(77))
    cases = [  # n, dim, nq, k, metric
        (5, 3, 2, 8, 0), (31, 64, 3, 10, 0), (257, 65, 7, 16, 0), (1000, 72, 33, 17, 0),
        (4097, 128, 130, 32, 0), (20011, 100, 37, 100, 0), (3000, 200, 300, 10, 0),
        (600, 96, 5, 256, 0), (9000, 64, 64, 10, 1), (777, 130, 9, 50, 1),
        (20011, 72, 257, 64, 0), (3001, 200, 600, 100, 1),  # CTA pairs
        (1000, 128, 100, 64, 0), (700, 64, 300, 100, 0),  # compact heaps
    ]
    for n, dim, nq, k, metric in cases:
        base = rng.standard_normal((n, dim), dtype=np.float32)
        queries = rng.standard_normal((nq, dim), dtype=np.float32)
        b16, q16 = O.round_fp16(base), O.round_fp16(queries)
        with E.Index(0) as idx:
            idx.build(base, metric=metric)
            gi, gd = idx.search(queries, k)
            oi, od = O.port_knn(b16, q16, k, threads=8, metric=metric)
            chk = O.check_parity_ip if metric == 1 else O.check_parity
            par = chk(b16, q16, gi, gd, oi, od, 1e-3)
            assert par.ok, (n, dim, nq, k, metric, par.detail)
            # device buffers, repeated: direct, captured, replayed
            qd = torch.from_numpy(queries).cuda()
            ni = torch.empty((nq, k), dtype=torch.int32, device="cuda")
            nd = torch.empty((nq, k), dtype=torch.float32, device="cuda")
            for _ in range(3):
                idx.search_async(qd, k, ni, nd)
                idx.sync()
                assert np.array_equal(ni.cpu().numpy().view(np.uint32), gi), (n, dim, nq, k)
            # the search without allocation (its own scratch carving)
            ai = np.empty((nq, k), np.uint32)
            ad = np.empty((nq, k), np.float32)
            st = E.lib().knn_index_search_noalloc(
                idx._h, queries.ctypes.data_as(ctypes.c_void_p), nq, k,
                ai.ctypes.data_as(ctypes.c_void_p), ad.ctypes.data_as(ctypes.c_void_p))
            assert st == E.KNN_OK, E.lib().knn_last_error()
            assert np.array_equal(ai, gi) and np.array_equal(ad, gd), (n, dim, nq, k)
        print(f"ok n={n} dim={dim} nq={nq} k={k} metric={metric}", flush=True)
    # exact fp32 re-ranking
    base = rng.standard_normal((5000, 80), dtype=np.float32)
    queries = rng.standard_normal((21, 80), dtype=np.float32)
    with E.Index(0) as idx:
        idx.set_rerank(True)
        idx.build(base)
        gi, gd = idx.search(queries, 12)
    oi, od = O.port_knn(base, queries, 12, threads=8)
    assert np.array_equal(gi, oi) and np.array_equal(gd, od), "re-rank"
    print("ok re-rank", flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
