"""GPU parity tests of the InnerProduct metric through the C ABI.

The reference declares DistanceType::InnerProduct
(include/cuvs/distance/distance.hpp:5-8) and rejects it at build
(src/cagra.cpp:26-28), so no reference output exists for it: the oracle is
the restated cuVS definition (oracle/knn_oracle.c, oracle_ip_knn) and the
integer-valued cases below, whose scores are exact in fp16 and fp32, must
match it bit for bit.

Acceptance rule for real-valued data (oracle.check_parity_ip): with
s_q = |q| * max |x| over the fp16-rounded vectors, rank by rank the index
equals the oracle's or the float64 scores differ by at most 1e-3 * s_q;
recall@k = 1 (tie-aware); scores within 1e-3 * s_q; sorted descending;
k > n padded with UINT32_MAX / -inf.
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3
IP = 1


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def _search(engine, base, queries, k, **kw):
    with engine.Index(0) as idx:
        idx.build(base, metric=IP)
        return idx.search(queries, k, **kw)


def test_integer_known_answers(engine, oracle_mod, torch_cuda):
    """Integer vectors (the FAISS smoke database and a random integer set
    with many equal scores): exact in every precision, so indices, scores,
    tie order and padding must equal the oracle's bytes."""
    g = json.load(open(os.path.join(GOLDEN, "faiss_smoke.json")))
    db = np.array(g["database"], np.float32)
    q = np.array(g["cases"][0]["queries"], np.float32)
    i, d = _search(engine, db, q, db.shape[0] + 1)
    oi, od = oracle_mod.port_knn(db, q, db.shape[0] + 1, metric=IP)
    assert np.array_equal(i, oi) and np.array_equal(d, od)
    assert np.isneginf(d[:, -1]).all() and (i[:, -1] == engine.NO_INDEX).all()

    rng = np.random.Generator(np.random.PCG64(77))
    base = rng.integers(-4, 5, (3000, 40)).astype(np.float32)
    queries = rng.integers(-4, 5, (70, 40)).astype(np.float32)
    for k in (1, 10, 33, 256):
        i, d = _search(engine, base, queries, k)
        oi, od = oracle_mod.port_knn(base, queries, k, metric=IP)
        assert np.array_equal(i, oi), k
        assert np.array_equal(d, od), k


def test_negative_scores_order(engine, oracle_mod, torch_cuda):
    """Every score negative: the descending order runs through negative
    values (the scan orders by -score, all positive here) and a query
    orthogonal to everything scores +0 everywhere (ties by index)."""
    rng = np.random.Generator(np.random.PCG64(5))
    base = np.abs(rng.standard_normal((5000, 64), dtype=np.float32)) + 0.1
    queries = -np.abs(rng.standard_normal((9, 64), dtype=np.float32))
    queries[0] = 0.0
    i, d = _search(engine, base, queries, 20)
    b16, q16 = oracle_mod.round_fp16(base), oracle_mod.round_fp16(queries)
    oi, od = oracle_mod.port_knn(b16, q16, 20, metric=IP)
    par = oracle_mod.check_parity_ip(b16, q16, i, d, oi, od, REL_TOL)
    assert par.ok, par.detail
    assert i[0].tolist() == list(range(20)) and np.all(d[0] == 0.0)
    assert np.all(d[1:] < 0)


SHAPES = [
    (1, 1, 1, 1),
    (7, 5, 3, 9),
    (257, 100, 33, 17),
    (1000, 128, 100, 10),
    (5000, 1024, 129, 10),
    (4099, 256, 16, 256),
    (700, 64, 300, 100),
    (20011, 72, 257, 64),
    (1000, 128, 100, 64),
    (20011, 64, 1000, 16),
]


@pytest.mark.parametrize("n,dim,nq,k", SHAPES)
def test_random_shapes(engine, oracle_mod, torch_cuda, n, dim, nq, k):
    rng = np.random.Generator(np.random.PCG64(n * 7 + dim * 3 + nq + k))
    base = rng.standard_normal((n, dim), dtype=np.float32)
    queries = rng.standard_normal((nq, dim), dtype=np.float32)
    i, d = _search(engine, base, queries, k)
    b16, q16 = oracle_mod.round_fp16(base), oracle_mod.round_fp16(queries)
    oi, od = oracle_mod.port_knn(b16, q16, k, threads=8, metric=IP)
    par = oracle_mod.check_parity_ip(b16, q16, i, d, oi, od, REL_TOL)
    assert par.ok, par.detail


def test_mixture_unit_norm(engine, oracle_mod, torch_cuda):
    """C2-shaped unit-norm mixture: on unit vectors the inner-product order
    is the L2 order (|q - x|^2 = 2 - 2 q.x), checked against both."""
    centres = oracle_mod.gen_centres(1000, 1024)
    base = oracle_mod.gen_mixture(100_000, 1024, 1000, oracle_mod.SEED_BASE, centres=centres)
    queries = oracle_mod.gen_mixture(100, 1024, 1000, oracle_mod.SEED_QUERIES, centres=centres)
    i, d = _search(engine, base, queries, 10)
    b16, q16 = oracle_mod.round_fp16(base), oracle_mod.round_fp16(queries)
    oi, od = oracle_mod.port_knn(b16, q16, 10, threads=8, metric=IP)
    par = oracle_mod.check_parity_ip(b16, q16, i, d, oi, od, REL_TOL)
    assert par.ok, par.detail
    li, _ = _search_l2(engine, base, queries, 10)
    overlap = sum(len(set(a) & set(b)) for a, b in zip(i.tolist(), li.tolist()))
    assert overlap / i.size >= 0.99


def _search_l2(engine, base, queries, k):
    with engine.Index(0) as idx:
        idx.build(base)
        return idx.search(queries, k)


def test_int64_padding_and_async(engine, oracle_mod, torch_cuda):
    """int64 neighbours: missing = -1 with score -inf; device buffers and
    the asynchronous entry point give the same bytes."""
    torch = torch_cuda
    rng = np.random.Generator(np.random.PCG64(8))
    base = rng.integers(-3, 4, (5, 16)).astype(np.float32)
    queries = rng.integers(-3, 4, (4, 16)).astype(np.float32)
    with engine.Index(0) as idx:
        idx.build(torch.from_numpy(base).cuda(), metric=IP)
        i64, d = idx.search(queries, 7, int64=True)
        oi, od = oracle_mod.port_knn(base, queries, 7, metric=IP)
        assert np.array_equal(d, od)
        assert (i64[:, 5:] == -1).all() and np.array_equal(i64[:, :5], oi[:, :5].astype(np.int64))
        qd = torch.from_numpy(queries).cuda()
        ni = torch.empty((4, 7), dtype=torch.int32, device="cuda")
        nd = torch.empty((4, 7), dtype=torch.float32, device="cuda")
        idx.search_async(qd, 7, ni, nd)
        idx.sync()
        assert np.array_equal(ni.cpu().numpy().view(np.uint32), oi)
        assert np.array_equal(nd.cpu().numpy(), od)
