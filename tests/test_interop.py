"""Container files exchanged with the reference's own save/load code.

The reference's "CGRA" v1 container (src/cagra.cpp:268-366) is compiled
unmodified into oracle/_ref/libref_cagra.so; tests/cpp/interop_test is this
library's side.  GPU tests:
  * a file the reference's cagra::save_index wrote loads here (cagra::
    load_index and brute_force::deserialize agree) and searches correctly;
  * a file brute_force::serialize wrote loads in the reference's
    cagra::load_index, whose own exact search over it equals the C
    restatement byte for byte (the file holds the engine's fp16 rows
    widened exactly to fp32).
CPU test: the reference's own save/load round trip, driven through the
oracle, is consistent (pins the shim).
"""
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT

BIN = os.path.join(ROOT, "tests", "cpp", "_bin", "interop_test")


def _data(oracle_mod, n=3000, dim=64, nq=11):
    rng = np.random.Generator(np.random.PCG64(515))
    return (rng.standard_normal((n, dim), dtype=np.float32),
            rng.standard_normal((nq, dim), dtype=np.float32))


def _need_ref(oracle_mod):
    if not oracle_mod.ref_available():
        pytest.skip("oracle/_ref (the reference's compiled sources) is absent")


def test_reference_round_trip_on_cpu(oracle_mod, tmp_path):
    _need_ref(oracle_mod)
    base, queries = _data(oracle_mod)
    path = str(tmp_path / "ref.bin")
    oracle_mod.ref_save_index(base, path)
    i, d, shape = oracle_mod.ref_load_search(path, queries, 10)
    assert shape == base.shape
    oi, od = oracle_mod.port_knn(base, queries, 10, threads=4)
    assert np.array_equal(i, oi) and np.array_equal(d, od)


@pytest.mark.gpu
def test_reference_file_loads_here(engine, oracle_mod, tmp_path):
    _need_ref(oracle_mod)
    base, queries = _data(oracle_mod)
    path = str(tmp_path / "ref.bin")
    oracle_mod.ref_save_index(base, path)
    qf = str(tmp_path / "q.f32")
    queries.tofile(qf)
    oi_path, od_path = str(tmp_path / "i.u32"), str(tmp_path / "d.f32")
    r = subprocess.run([BIN, "read", path, qf, str(len(queries)), "10", oi_path, od_path],
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    gi = np.fromfile(oi_path, np.uint32).reshape(len(queries), 10)
    gd = np.fromfile(od_path, np.float32).reshape(len(queries), 10)
    b16, q16 = oracle_mod.round_fp16(base), oracle_mod.round_fp16(queries)
    oi, od = oracle_mod.port_knn(b16, q16, 10, threads=4)
    par = oracle_mod.check_parity(b16, q16, gi, gd, oi, od, 1e-3)
    assert par.ok, par.detail


@pytest.mark.gpu
def test_file_written_here_loads_in_reference(engine, oracle_mod, tmp_path):
    _need_ref(oracle_mod)
    base, queries = _data(oracle_mod)
    bf = str(tmp_path / "base.f32")
    base.tofile(bf)
    path = str(tmp_path / "ours.bin")
    r = subprocess.run([BIN, "write", path, bf, str(base.shape[0]), str(base.shape[1])],
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    i, d, shape = oracle_mod.ref_load_search(path, queries, 10)
    assert shape == base.shape
    # the rows in the file are the engine's fp16 rows, widened exactly
    b16 = oracle_mod.round_fp16(base)
    oi, od = oracle_mod.port_knn(b16, queries, 10, threads=4)
    assert np.array_equal(i, oi) and np.array_equal(d, od)
