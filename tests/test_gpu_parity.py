"""GPU parity tests: the CUDA engine, called through its C ABI (via the
ctypes binding), against the oracle on identical seeded inputs.

Acceptance rule (oracle.check_parity): rank by rank the index equals the
oracle's, or the two float64 distances differ by at most rel 1e-3; recall@k
is 1.0 (tie-aware); returned distances within rel 1e-3 (abs 1e-4 near 0);
sorted ascending; k > n padded with UINT32_MAX / +inf.  The oracle runs on
the fp16-ROUNDED vectors, the engine's storage format.
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def _search(engine, base, queries, k, **kw):
    with engine.Index(0) as idx:
        idx.build(base)
        return idx.search(queries, k, **kw)


def _check(oracle_mod, base, queries, k, threads=8):
    b16 = oracle_mod.round_fp16(base)
    q16 = oracle_mod.round_fp16(queries)
    oi, od = oracle_mod.port_knn(b16, q16, k, threads=threads)
    return b16, q16, oi, od


def test_faiss_smoke_golden(engine, oracle_mod, torch_cuda):
    """The reference adapter's asserted values
    (tests/faiss_v1_8_cagra_runtime_smoke.cpp:299-383), exactly."""
    g = json.load(open(os.path.join(GOLDEN, "faiss_smoke.json")))
    db = np.array(g["database"], np.float32)
    with engine.Index(0) as idx:
        idx.build(db)
        for case in g["cases"]:
            q = np.array(case["queries"], np.float32)
            i, d = idx.search(q, case["k"])
            assert i.astype(np.int64).tolist() == case["neighbors"], case["name"]
            exp = [[np.inf if x == "inf" else x for x in row] for row in case["distances"]]
            assert d.tolist() == exp, case["name"]
        # FAISS-style int64 labels: UINT32_MAX -> -1 (adapter :201-206)
        i64, d = idx.search(np.array(g["cases"][0]["queries"], np.float32), 5, int64=True)
        assert i64[0, 4] == -1 and i64[1, 4] == -1 and np.isinf(d[0, 4])


def test_dispatch_spy(engine, oracle_mod, torch_cuda):
    """tests/test_metal_search.cpp:16-58: search must launch device kernels;
    here also the values must match the reference."""
    g = np.load(os.path.join(GOLDEN, "dispatch_spy.npz"))
    with engine.Index(0) as idx:
        idx.build(g["base"])
        engine.reset_dispatch_count()
        i, d = idx.search(g["queries"], 4)
        assert engine.dispatch_count() > 0
    assert np.array_equal(i, g["neighbors"])
    assert np.array_equal(d, g["distances"])


def test_batching_l2_known_answer(engine, oracle_mod, torch_cuda):
    """tests/test_benchmark_batching.py:220-239 of the reference: query e0
    against e0, 2 e0 and e1 at D = 128 gives [0, 1, 2] exactly."""
    dim = 128
    query = np.zeros((1, dim), np.float32)
    query[0, 0] = 1.0
    cands = np.zeros((3, dim), np.float32)
    cands[0, 0] = 1.0
    cands[1, 0] = 2.0
    cands[2, 1] = 1.0
    i, d = _search(engine, cands, query, 3)
    assert i.tolist() == [[0, 1, 2]] and d.tolist() == [[0.0, 1.0, 2.0]]


def test_ties_duplicates_padding(engine, oracle_mod, torch_cuda):
    g = np.load(os.path.join(GOLDEN, "ties.npz"))
    i, d = _search(engine, g["base"], g["queries"], 45)
    # integer data: the expanded form is exact, so the order is bit-exact
    assert np.array_equal(i, g["neighbors"])
    assert np.array_equal(d, g["distances"])


def test_c1_golden(engine, oracle_mod, torch_cuda):
    """Config 1 (N=10,000, D=128, Q=100, K=10, iid) vs the reference's own
    output on the fp16-rounded inputs."""
    g = np.load(os.path.join(GOLDEN, "c1_fp16.npz"))
    base = oracle_mod.gen_iid(10000, 128, oracle_mod.SEED_IID_BASE)
    queries = oracle_mod.gen_iid(100, 128, oracle_mod.SEED_IID_QUERIES)
    i, d = _search(engine, base, queries, 10)
    b16, q16 = oracle_mod.round_fp16(base), oracle_mod.round_fp16(queries)
    par = oracle_mod.check_parity(b16, q16, i, d, g["neighbors"], g["distances"], REL_TOL)
    assert par.ok, par.detail
    # recall vs the reference's fp32 ground truth (informational bound)
    g32 = np.load(os.path.join(GOLDEN, "c1_fp32.npz"))
    hits = sum(len(set(a) & set(b)) for a, b in zip(i.tolist(), g32["neighbors"].tolist()))
    assert hits / i.size >= 0.97


SHAPES = [
    # (n, dim, nq, k)
    (1, 1, 1, 1),
    (7, 5, 3, 9),
    (64, 8, 4, 4),
    (255, 64, 17, 10),
    (256, 64, 1, 16),
    (257, 100, 33, 17),
    (1000, 128, 100, 10),
    (1000, 1000, 4, 64),
    (5000, 1024, 129, 10),
    (3000, 72, 300, 32),
    (4099, 256, 16, 256),
    (2500, 128, 100, 256),
    (1500, 64, 40, 200),
    (700, 64, 300, 100),
    # CTA pairs (more than 128 queries, k >= 62): a last pair tile with one
    # query, a dataset of three 64-row granules, several pair tiles
    (20011, 72, 257, 64),
    (130, 33, 129, 62),
    (3001, 200, 600, 128),
    # compact 6-byte heap entries (k > 16 where they buy a stage): single
    # CTAs at k = 64, and CTA pairs whose units span 62,163 rows (row
    # offsets near the 16-bit limit)
    (1000, 128, 100, 64),
    (50000, 64, 100, 64),
    (2300000, 16, 260, 100),
    # CTA pairs at small k (query padding no worse than single CTAs'):
    # register top-k, several pair tiles, and the pilot pass at k = 32
    (20011, 64, 1000, 16),
    (1000, 128, 200, 32),
    # 32-query blocks spread over the four TMEM lane quadrants (k > 16):
    # a ragged single block, and two blocks the second of which holds 5
    (3001, 128, 29, 100),
    (2000, 64, 37, 256),
]


@pytest.mark.parametrize("n,dim,nq,k", SHAPES)
def test_random_shapes(engine, oracle_mod, torch_cuda, n, dim, nq, k):
    rng = np.random.Generator(np.random.PCG64(n * 7919 + dim * 31 + nq * 7 + k))
    base = rng.standard_normal((n, dim), dtype=np.float32)
    queries = rng.standard_normal((nq, dim), dtype=np.float32)
    i, d = _search(engine, base, queries, k)
    b16, q16, oi, od = _check(oracle_mod, base, queries, k)
    par = oracle_mod.check_parity(b16, q16, i, d, oi, od, REL_TOL)
    assert par.ok, par.detail


def test_identical_rows_tie_by_index(engine, oracle_mod, torch_cuda):
    """Every row at the same distance: the first-tile threshold seed equals
    that distance, and the result must be rows 0..k-1 in index order."""
    base = np.tile(np.arange(64, dtype=np.float32) / 64, (3000, 1))
    queries = np.zeros((3, 64), np.float32)
    i, d = _search(engine, base, queries, 10)
    assert i.tolist() == [list(range(10))] * 3
    assert np.all(d == d[0, 0])


def test_c2_mixture(engine, oracle_mod, torch_cuda):
    """Config 2: N=100,000, D=1024, Q=100, K=10, unit-norm mixture."""
    centres = oracle_mod.gen_centres(1000, 1024)
    base = oracle_mod.gen_mixture(100_000, 1024, 1000, oracle_mod.SEED_BASE, centres=centres)
    queries = oracle_mod.gen_mixture(100, 1024, 1000, oracle_mod.SEED_QUERIES, centres=centres)
    i, d = _search(engine, base, queries, 10)
    b16, q16, oi, od = _check(oracle_mod, base, queries, 10)
    par = oracle_mod.check_parity(b16, q16, i, d, oi, od, REL_TOL, eps=1e-6)
    assert par.ok, par.detail


def test_device_pointers_and_async(engine, oracle_mod, torch_cuda):
    torch = torch_cuda
    rng = np.random.Generator(np.random.PCG64(5))
    base = rng.standard_normal((3000, 256), dtype=np.float32)
    queries = rng.standard_normal((50, 256), dtype=np.float32)
    b16, q16, oi, od = _check(oracle_mod, base, queries, 10)
    with engine.Index(0) as idx:
        idx.build(torch.from_numpy(base).cuda())          # device fp32 rows
        qd = torch.from_numpy(queries).cuda()
        ni = torch.empty((50, 10), dtype=torch.int32, device="cuda")
        nd = torch.empty((50, 10), dtype=torch.float32, device="cuda")
        idx.search(qd, 10, neighbors=ni, distances=nd)
        i = ni.cpu().numpy().view(np.uint32)
        par = oracle_mod.check_parity(b16, q16, i, nd.cpu().numpy(), oi, od, REL_TOL)
        assert par.ok, par.detail
        ni.zero_()
        idx.search_async(qd, 10, ni, nd)
        idx.sync()
        assert np.array_equal(ni.cpu().numpy().view(np.uint32), i)
        # fp16 device rows build to the same index
        idx.build(torch.from_numpy(b16).half().cuda())
        i2, d2 = idx.search(queries, 10)
        assert np.array_equal(i2, i)


def test_graph_replay_follows_buffer_contents(engine, oracle_mod, torch_cuda):
    """Repeated device-resident searches are replayed from a CUDA graph; a
    replay must read the current contents of the (same) query buffer and
    match the graph-free path bit for bit."""
    torch = torch_cuda
    rng = np.random.Generator(np.random.PCG64(12))
    base = rng.standard_normal((6000, 128), dtype=np.float32)
    qa = rng.standard_normal((40, 128), dtype=np.float32)
    qb = rng.standard_normal((40, 128), dtype=np.float32)
    with engine.Index(0) as idx:
        idx.build(base)
        qd = torch.from_numpy(qa).cuda()
        ni = torch.empty((40, 10), dtype=torch.int32, device="cuda")
        nd = torch.empty((40, 10), dtype=torch.float32, device="cuda")
        outs = []
        for src in (qa, qa, qa, qb, qb, qa):
            qd.copy_(torch.from_numpy(src))
            idx.search_async(qd, 10, ni, nd)
            idx.sync()
            outs.append((ni.cpu().numpy().copy(), nd.cpu().numpy().copy()))
        idx.set_graphs(False)
        ref = {}
        for name, src in (("a", qa), ("b", qb)):
            qd.copy_(torch.from_numpy(src))
            idx.search_async(qd, 10, ni, nd)
            idx.sync()
            ref[name] = (ni.cpu().numpy().copy(), nd.cpu().numpy().copy())
    for (i, d), name in zip(outs, "aaabba"):
        assert np.array_equal(i, ref[name][0]) and np.array_equal(d, ref[name][1])


def test_pinned_host_buffers_in_place(engine, oracle_mod, torch_cuda):
    """Page-locked host queries and outputs are used in place by the kernels
    (no staging copies) and replayed from a CUDA graph; results equal the
    pageable-buffer path byte for byte and follow the buffers' contents."""
    torch = torch_cuda
    rng = np.random.Generator(np.random.PCG64(31))
    base = rng.standard_normal((9000, 200), dtype=np.float32)
    qa = rng.standard_normal((30, 200), dtype=np.float32)
    qb = rng.standard_normal((30, 200), dtype=np.float32)
    with engine.Index(0) as idx:
        idx.build(base)
        ref = {name: idx.search(q, 12) for name, q in (("a", qa), ("b", qb))}
        qp = torch.empty((30, 200), dtype=torch.float32).pin_memory()
        ip = torch.empty((30, 12), dtype=torch.int32).pin_memory()
        dp = torch.empty((30, 12), dtype=torch.float32).pin_memory()
        for name, src in (("a", qa), ("a", qa), ("b", qb), ("a", qa), ("b", qb)):
            qp.copy_(torch.from_numpy(src))
            idx.search(qp, 12, neighbors=ip, distances=dp)
            assert np.array_equal(ip.numpy().view(np.uint32), ref[name][0]), name
            assert np.array_equal(dp.numpy(), ref[name][1]), name
        # pinned queries with pageable outputs, and the reverse
        qp.copy_(torch.from_numpy(qb))
        i, d = idx.search(qp, 12)
        assert np.array_equal(i, ref["b"][0]) and np.array_equal(d, ref["b"][1])
        idx.search(qa, 12, neighbors=ip, distances=dp)
        assert np.array_equal(ip.numpy().view(np.uint32), ref["a"][0])
    b16, q16, oi, od = _check(oracle_mod, base, qa, 12)
    par = oracle_mod.check_parity(b16, q16, ref["a"][0], ref["a"][1], oi, od, REL_TOL)
    assert par.ok, par.detail


def test_repeat_is_bit_identical(engine, oracle_mod, torch_cuda):
    """Deterministic: two searches give the same bytes (run-twice check)."""
    rng = np.random.Generator(np.random.PCG64(9))
    base = rng.standard_normal((20000, 512), dtype=np.float32)
    queries = rng.standard_normal((64, 512), dtype=np.float32)
    with engine.Index(0) as idx:
        idx.build(base)
        a = idx.search(queries, 20)
        b = idx.search(queries, 20)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def test_shard_decomposition(engine, oracle_mod, torch_cuda):
    """Row shards built with global offsets, merged on the host by the
    oracle's merge, equal the single-index result."""
    rng = np.random.Generator(np.random.PCG64(11))
    n = 10001
    base = rng.standard_normal((n, 96), dtype=np.float32)
    queries = rng.standard_normal((20, 96), dtype=np.float32)
    k = 12
    full_i, full_d = _search(engine, base, queries, k)
    lists_d = np.empty((20, 3, k), np.float32)
    lists_i = np.empty((20, 3, k), np.uint32)
    for r in range(3):
        lo, hi = engine.shard_range(n, 3, r)
        with engine.Index(0) as idx:
            idx.build(base[lo:hi], row_offset=lo, total_rows=n)
            i, d = idx.search(queries, k)
        assert i[i != engine.NO_INDEX].min() >= lo
        lists_d[:, r], lists_i[:, r] = d, i
    mi, md = oracle_mod.merge_lists(lists_d, lists_i)
    assert np.array_equal(mi, full_i) and np.array_equal(md, full_d)


def test_argument_errors(engine, torch_cuda):
    with engine.Index(0) as idx:
        with pytest.raises(ValueError, match="non-empty"):
            idx.build(np.zeros((0, 4), np.float32))
        with pytest.raises(ValueError, match="L2Expanded"):
            idx.build(np.ones((4, 4), np.float32), metric=7)
        with pytest.raises(ValueError, match="no dataset"):
            idx.search(np.ones((2, 4), np.float32), 2)
        idx.build(np.ones((4, 4), np.float32))
        with pytest.raises(ValueError, match="dimension"):
            idx.search(np.ones((2, 5), np.float32), 2)
        with pytest.raises(RuntimeError, match="UNSUPPORTED"):
            idx.search(np.ones((2, 4), np.float32), 257)
        i, d = idx.search(np.ones((0, 4), np.float32), 3)   # no-op
        assert i.shape == (0, 3)
        i, d = idx.search(np.ones((2, 4), np.float32), 0)   # k = 0: no-op
        assert i.shape == (2, 0)


def test_bounded_wait_reports_timeout(engine, torch_cuda):
    """A device wait on a barrier nothing arrives on gives up after its limit
    and the host reads KNN_ETIMEOUT; the context stays usable."""
    lib = engine.lib()
    st = lib.knn_selftest_bounded_wait(0, 20000)  # 20 ms limit
    assert st == engine.KNN_ETIMEOUT, lib.knn_last_error()
    # the device still works afterwards
    i, d = _search(engine, np.eye(4, dtype=np.float32), np.eye(4, dtype=np.float32)[:1], 1)
    assert i[0, 0] == 0
