"""Parity at the full sizes of the benchmark configurations (one GPU's share).

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


def test_config5_latency_sweep(engine, oracle_mod, torch_cuda):
    base, queries = _mixture(oracle_mod, 1_000_000, 16)
    b16, q16 = oracle_mod.round_fp16(base), oracle_mod.round_fp16(queries)
    oi256, od256 = oracle_mod.blas_knn(b16, q16, 256)
    with engine.Index(0) as idx:
        idx.build(base)
        del base
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
