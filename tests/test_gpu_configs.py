"""Parity at the full sizes of the benchmark configurations (one GPU's share).

* Headline (the configuration bench.py times): N = 1M, D = 1024, Q = 100,
  K = 10; all 100 queries checked, 4 of them against the sequential C
  restatement as well.
* Config 5 (latency / top-K stress): N = 1M, D = 1024 unit-norm mixture
  (10,000 centres), Q in {1, 16}, K in {10, 256}; every query is checked
  against the oracle.
* Config 4 (compute-bound), one GPU's row shard: N = 1.25M (10M over 8 GPUs),
  D = 1024, Q = 10,000, K = 100.  All 10,000 queries are searched; 32 sampled
  queries are checked against the oracle, and every query through the
  size-independent properties of the output (ascending (distance, index)
  order, distinct in-range indices, a query equal to a dataset row finds
  that row first, at distance 0 up to fp32 rounding).

The oracle here is the expanded-form BLAS port (oracle.blas_knn,
src/cagra.cpp:139-177 generalised to top-k) on the fp16-rounded rows:
the sequential C restatement would take minutes at these sizes.  Its
indices only seed the comparison; the acceptance rule (oracle.check_parity,
rel 1e-3) recomputes every distance in float64.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def _mixture(oracle_mod, n, nq, dim=1024, centres=10_000):
    c = oracle_mod.gen_centres(centres, dim)
    base = oracle_mod.gen_mixture(n, dim, centres, oracle_mod.SEED_BASE, centres=c, threads=16)
    queries = oracle_mod.gen_mixture(nq, dim, centres, oracle_mod.SEED_QUERIES, centres=c)
    return base, queries


@pytest.fixture(scope="module")
def headline_index(engine, oracle_mod, torch_cuda):
    """The headline dataset (N = 1M, D = 1024, BASELINE mixture, seeds
    11/12/13) built once for the tests at that size: (index, fp16-rounded
    rows, centres)."""
    c = oracle_mod.gen_centres(10_000, 1024)
    base = oracle_mod.gen_mixture(1_000_000, 1024, 10_000, oracle_mod.SEED_BASE, centres=c,
                                  threads=16)
    idx = engine.Index(0)
    idx.build(base)
    b16 = oracle_mod.round_fp16(base)
    del base
    yield idx, b16, c
    idx.close()


def _queries(oracle_mod, c, nq):
    return oracle_mod.gen_mixture(nq, 1024, 10_000, oracle_mod.SEED_QUERIES, centres=c)


def test_headline_all_queries(engine, oracle_mod, headline_index):
    """The configuration bench.py times: N = 1M, D = 1024, Q = 100, K = 10.
    All 100 queries against the BLAS-seeded oracle (every distance
    re-checked in float64), and 4 of them against the sequential C
    restatement of the reference's search on all rows, which needs no seed.
    Then the same through the device-buffer path, replayed from its graph."""
    import torch

    idx, b16, c = headline_index
    queries = _queries(oracle_mod, c, 100)
    q16 = oracle_mod.round_fp16(queries)
    i, d = idx.search(queries, 10)
    oi, od = oracle_mod.blas_knn(b16, q16, 10)
    par = oracle_mod.check_parity(b16, q16, i, d, oi, od, REL_TOL)
    assert par.ok, par.detail
    pick = np.array([0, 33, 66, 99])
    pi, pd = oracle_mod.port_knn(b16, q16[pick], 10, threads=4)
    par4 = oracle_mod.check_parity(b16, q16[pick], i[pick], d[pick], pi, pd, REL_TOL)
    assert par4.ok, par4.detail
    qd = torch.from_numpy(queries).cuda()
    ni = torch.empty((100, 10), dtype=torch.int32, device="cuda")
    nd = torch.empty((100, 10), dtype=torch.float32, device="cuda")
    for _ in range(4):  # direct, captured, replayed, replayed
        ni.zero_()
        idx.search_async(qd, 10, ni, nd)
        idx.sync()
        assert np.array_equal(ni.cpu().numpy().view(np.uint32), i)
        assert np.array_equal(nd.cpu().numpy(), d)


def test_config5_latency_sweep(engine, oracle_mod, headline_index):
    idx, b16, c = headline_index
    queries = _queries(oracle_mod, c, 16)
    q16 = oracle_mod.round_fp16(queries)
    oi256, od256 = oracle_mod.blas_knn(b16, q16, 256)
    for nq in (1, 16):
        for k in (10, 256):
            i, d = idx.search(queries[:nq], k)
            par = oracle_mod.check_parity(b16, q16[:nq], i, d, oi256[:nq, :k],
                                          od256[:nq, :k], REL_TOL)
            assert par.ok, f"Q={nq} K={k}: {par.detail}"


def test_config4_shard_compute_bound(engine, oracle_mod, torch_cuda):
    n, nq, k = 1_250_000, 10_000, 100
    base, queries = _mixture(oracle_mod, n, nq)
    # plant exact copies of dataset rows among the queries
    planted = np.arange(0, nq, 997)
    rows = (planted * 131) % n
    queries[planted] = base[rows]
    b16 = oracle_mod.round_fp16(base)
    with engine.Index(0) as idx:
        idx.build(base)
        del base
        i, d = idx.search(queries, k)
    # every query: sorted by (distance, index), distinct indices in range
    assert np.all(i < n)
    assert np.all(np.diff(d, axis=1) >= 0)
    ties = np.diff(d, axis=1) == 0
    assert np.all(np.diff(i.astype(np.int64), axis=1)[ties] > 0)
    srt = np.sort(i, axis=1)
    assert np.all(srt[:, 1:] != srt[:, :-1])
    # planted copies come back first, at distance 0 up to the fp32
    # rounding of |q|^2 + |x|^2 - 2 q.x for unit vectors
    for q, r in zip(planted, rows):
        assert d[q, 0] <= 1e-5 and r in i[q][d[q] <= 1e-5], (q, r, i[q, :3], d[q, :3])
    # sampled queries against the oracle
    rng = np.random.Generator(np.random.PCG64(44))
    sample = np.sort(rng.choice(nq, 32, replace=False))
    q16 = oracle_mod.round_fp16(queries[sample])
    oi, od = oracle_mod.blas_knn(b16, q16, k)
    par = oracle_mod.check_parity(b16, q16, i[sample], d[sample], oi, od, REL_TOL)
    assert par.ok, par.detail
