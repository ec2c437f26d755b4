"""Dataset file loaders (the caller side of the path).

CPU: the reference's own tests/test_sift_loader.cpp, compiled unmodified
against this repository's include/cuvs_silicon/sift_loader.hpp and library,
passes; so does loader_test (the .bin matrices of the Cohere-wiki benchmark,
tests/test_cohere_wiki_validation.cpp:40-52, and multi-block fvecs files);
the numpy readers round-trip.
GPU: knn_index_build_file streams fvecs / .bin files (whole or one rank's
shard) into an index that searches exactly like one built from the array.
"""
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT

CPP = os.path.join(ROOT, "tests", "cpp")
BIN = os.path.join(CPP, "_bin")


@pytest.fixture(scope="module")
def built(engine):
    subprocess.run(["make", "-C", CPP], check=True, capture_output=True)
    return BIN


def test_reference_sift_loader_test_passes(built):
    path = os.path.join(built, "ref_test_sift_loader")
    if not os.path.exists(path):
        pytest.skip("reference tree absent and no prebuilt binary")
    r = subprocess.run([path], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr


def test_bin_and_fvecs_loader_program(built, tmp_path):
    r = subprocess.run([os.path.join(built, "loader_test"), str(tmp_path)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr


def test_numpy_readers_round_trip(engine, tmp_path):
    rng = np.random.Generator(np.random.PCG64(1))
    a = rng.standard_normal((33, 17), dtype=np.float32)
    engine.write_fvecs(str(tmp_path / "a.fvecs"), a)
    assert np.array_equal(engine.read_fvecs(str(tmp_path / "a.fvecs")), a)
    engine.write_bin(str(tmp_path / "a.bin"), a)
    assert np.array_equal(engine.read_bin(str(tmp_path / "a.bin")), a)
    gt = rng.integers(0, 1000, (4, 9)).astype(np.int32)
    engine.write_bin(str(tmp_path / "g.bin"), gt)
    assert np.array_equal(engine.read_bin(str(tmp_path / "g.bin"), np.int32), gt)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["fvecs", "bin"])
def test_build_file_matches_array_build(engine, oracle_mod, tmp_path, fmt):
    rng = np.random.Generator(np.random.PCG64(3))
    # 70,000 rows of 300 floats: 84 MB, more than one 64 MiB read chunk
    base = rng.standard_normal((70000, 300), dtype=np.float32)
    queries = rng.standard_normal((25, 300), dtype=np.float32)
    path = str(tmp_path / f"base.{fmt}")
    code = engine.FILE_FVECS if fmt == "fvecs" else engine.FILE_BIN_F32
    (engine.write_fvecs if fmt == "fvecs" else engine.write_bin)(path, base)
    with engine.Index(0) as a, engine.Index(0) as b:
        a.build(base)
        b.build_file(path, code)
        assert b.rows == 70000 and b.dim == 300
        ia, da = a.search(queries, 10)
        ib, db = b.search(queries, 10)
    assert np.array_equal(ia, ib) and np.array_equal(da, db)
    # one rank's shard of a 3-way split reports global row indices
    lo, hi = engine.shard_range(70000, 3, 1)
    with engine.Index(0) as s, engine.Index(0) as t:
        s.build_file(path, code, n_ranks=3, rank=1)
        t.build(base[lo:hi], row_offset=lo, total_rows=70000)
        assert s.rows == hi - lo
        i1, d1 = s.search(queries, 10)
        i2, d2 = t.search(queries, 10)
    assert np.array_equal(i1, i2) and np.array_equal(d1, d2)
    assert i1.min() >= lo and i1.max() < hi


@pytest.mark.gpu
def test_build_file_rerank_and_errors(engine, oracle_mod, tmp_path):
    rng = np.random.Generator(np.random.PCG64(4))
    base = rng.standard_normal((5000, 64), dtype=np.float32)
    queries = rng.standard_normal((10, 64), dtype=np.float32)
    path = str(tmp_path / "b.fvecs")
    engine.write_fvecs(path, base)
    with engine.Index(0) as idx:
        idx.set_rerank(True)
        idx.build_file(path, engine.FILE_FVECS)
        i, d = idx.search(queries, 10)
        assert idx.rerank_stats()["uncertified"] == 0
    oi, od = oracle_mod.port_knn(base, queries, 10)
    assert np.array_equal(i, oi) and np.array_equal(d, od)
    # a record of another width, a ragged tail, a missing file
    raw = np.fromfile(path, dtype=np.int32)
    bad = raw.copy()
    bad[65 * 100] = 63
    bad.tofile(str(tmp_path / "bad.fvecs"))
    raw[:-3].tofile(str(tmp_path / "short.fvecs"))
    with engine.Index(0) as idx:
        with pytest.raises(ValueError, match="width"):
            idx.build_file(str(tmp_path / "bad.fvecs"), engine.FILE_FVECS)
        with pytest.raises(ValueError, match="whole number"):
            idx.build_file(str(tmp_path / "short.fvecs"), engine.FILE_FVECS)
        with pytest.raises(ValueError, match="cannot open"):
            idx.build_file(str(tmp_path / "none.fvecs"), engine.FILE_FVECS)
