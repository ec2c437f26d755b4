"""Exact fp32 re-ranking (knn_index_set_rerank) against the reference's own
fp32 exact search.

With re-ranking, results are the reference's portable exact search
(src/cagra.cpp:211-252) on the UNROUNDED fp32 rows, byte for byte: the
golden config-1 output of the reference binary (tests/golden/c1_fp32.npz)
and the C restatement (bit-identical to that binary, tests/test_oracle.py)
on every other case.  Every query of these cases must be certified.  The
near-duplicate cases check the certificate itself: rows that are equal in
fp16 but not in fp32 cannot be ordered by the fp16 scan, so a query with
more of them than candidates must be reported as not certified.
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def _rerank_search(engine, base, queries, k, metric=0, **kw):
    with engine.Index(0) as idx:
        idx.set_rerank(True)
        idx.build(base, metric=metric)
        i, d = idx.search(queries, k, **kw)
        return i, d, idx.rerank_stats()


def test_c1_equals_reference_fp32(engine, oracle_mod, torch_cuda):
    g = np.load(os.path.join(GOLDEN, "c1_fp32.npz"))
    base = oracle_mod.gen_iid(10000, 128, oracle_mod.SEED_IID_BASE)
    queries = oracle_mod.gen_iid(100, 128, oracle_mod.SEED_IID_QUERIES)
    i, d, st = _rerank_search(engine, base, queries, 10)
    assert st == {"uncertified": 0, "widened": 0}
    assert np.array_equal(i, g["neighbors"])
    assert np.array_equal(d, g["distances"])


def test_c2_mixture_equals_fp32_oracle(engine, oracle_mod, torch_cuda):
    centres = oracle_mod.gen_centres(1000, 1024)
    base = oracle_mod.gen_mixture(100_000, 1024, 1000, oracle_mod.SEED_BASE, centres=centres)
    queries = oracle_mod.gen_mixture(100, 1024, 1000, oracle_mod.SEED_QUERIES, centres=centres)
    i, d, st = _rerank_search(engine, base, queries, 10)
    oi, od = oracle_mod.port_knn(base, queries, 10, threads=8)
    assert st["uncertified"] == 0
    assert np.array_equal(i, oi) and np.array_equal(d, od)


SHAPES = [
    # (n, dim, nq, k): odd dims take the scalar path of the fp32 sums
    (1, 1, 1, 1),
    (7, 5, 3, 9),
    (300, 33, 20, 17),
    (2000, 128, 64, 64),
    (5000, 1000, 40, 100),
    (3000, 96, 50, 128),
]


@pytest.mark.parametrize("n,dim,nq,k", SHAPES)
@pytest.mark.parametrize("metric", [0, 1])
def test_random_shapes_exact(engine, oracle_mod, torch_cuda, n, dim, nq, k, metric):
    rng = np.random.Generator(np.random.PCG64(n + 13 * dim + 7 * nq + k + 1000 * metric))
    base = rng.standard_normal((n, dim), dtype=np.float32)
    queries = rng.standard_normal((nq, dim), dtype=np.float32)
    i, d, st = _rerank_search(engine, base, queries, k, metric=metric)
    oi, od = oracle_mod.port_knn(base, queries, k, threads=8, metric=metric)
    assert st["uncertified"] == 0
    assert np.array_equal(i, oi) and np.array_equal(d, od)


def _near_duplicates(n_dup, n_far=3000, dim=64, seed=4):
    """n_dup rows equal after fp16 rounding (but distinct in fp32) close to
    the queries, plus n_far rows far away."""
    rng = np.random.Generator(np.random.PCG64(seed))
    # fp16-exact coordinates with 0.125 <= |v| < 0.5 (no zeros: a tiny
    # jitter of 0 would survive as an fp16 subnormal)
    v = (rng.integers(32, 128, dim) * rng.choice([-1, 1], dim) / 256.0).astype(np.float32)
    jitter = rng.uniform(-2.0 ** -14, 2.0 ** -14, (n_dup, dim)).astype(np.float32)
    dups = v + jitter * np.abs(v)  # relative 2^-14: below half an fp16 ulp of v
    far = rng.standard_normal((n_far, dim), dtype=np.float32) + 4.0
    base = np.concatenate([far[: n_far // 2], dups, far[n_far // 2:]]).astype(np.float32)
    queries = (v + rng.uniform(-0.01, 0.01, (3, dim))).astype(np.float32)
    return base, queries


def test_certificate_widening_recovers_exactness(engine, oracle_mod, torch_cuda):
    """200 fp16-equal rows: the first 32 candidates cannot be certified,
    the repeat with 256 candidates holds all 200 and is exact."""
    base, queries = _near_duplicates(200)
    b16 = oracle_mod.round_fp16(base)
    assert len(np.unique(b16[1500:1700], axis=0)) == 1  # equal in fp16
    i, d, st = _rerank_search(engine, base, queries, 10)
    oi, od = oracle_mod.port_knn(base, queries, 10)
    assert st["widened"] == 3 and st["uncertified"] == 0
    assert np.array_equal(i, oi) and np.array_equal(d, od)


def test_certificate_reports_uncertified(engine, oracle_mod, torch_cuda):
    """600 fp16-equal rows exceed every candidate count: every query is
    reported uncertified; the result is still sorted, distinct and exact
    fp32 distances of the rows it names."""
    base, queries = _near_duplicates(600)
    i, d, st = _rerank_search(engine, base, queries, 10)
    assert st["uncertified"] == 3 and st["widened"] == 3
    for q in range(3):
        assert len(set(i[q].tolist())) == 10
        assert np.all(np.diff(d[q]) >= 0)
        diff = queries[q][None, :] - base[i[q].astype(np.int64)]
        exact = np.array([np.float32(0)] * 10)
        for r in range(10):  # sequential fp32 sum, as the reference
            acc = np.float32(0)
            for x in diff[r]:
                acc = np.float32(acc + np.float32(x * x))
            exact[r] = acc
        assert np.array_equal(d[q], exact)


def test_async_stats_and_switching(engine, oracle_mod, torch_cuda):
    torch = torch_cuda
    rng = np.random.Generator(np.random.PCG64(21))
    base = rng.standard_normal((4000, 128), dtype=np.float32)
    queries = rng.standard_normal((30, 128), dtype=np.float32)
    oi, od = oracle_mod.port_knn(base, queries, 10)
    with engine.Index(0) as idx:
        idx.build(base)
        fp16_i, fp16_d = idx.search(queries, 10)
        with pytest.raises(ValueError):
            idx.set_rerank(True)  # built without the fp32 rows
        idx.build(base)  # re-ranking stays requested: this build keeps them
        qd = torch.from_numpy(queries).cuda()
        ni = torch.empty((30, 10), dtype=torch.int32, device="cuda")
        nd = torch.empty((30, 10), dtype=torch.float32, device="cuda")
        idx.search_async(qd, 10, ni, nd)
        idx.sync()
        assert idx.rerank_stats()["uncertified"] == 0
        assert np.array_equal(ni.cpu().numpy().view(np.uint32), oi)
        assert np.array_equal(nd.cpu().numpy(), od)
        # the fp32 rows come back exactly
        assert np.array_equal(idx.copy_rows(np.float32), base)
        idx.set_rerank(False)
        i, d = idx.search(queries, 10)
        assert np.array_equal(i, fp16_i) and np.array_equal(d, fp16_d)
    with engine.Index(0) as idx:
        idx.set_rerank(True)
        with pytest.raises(ValueError):  # the fp32 rows are needed
            idx.build(base.astype(np.float16))
