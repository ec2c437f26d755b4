"""Generates the golden fixtures in this directory from the REFERENCE ITSELF.

Run from the repository root with the reference tree present:

    python tests/golden/make_golden.py

Every output below comes from the reference's own exact search, compiled
unmodified from src/cagra.cpp of ysys143/cuvs-silicon into
oracle/_ref/libref_cagra.so (oracle/Makefile) and called through its public
cuvs::neighbors::cagra::build/search API (oracle/ref_shim.cpp).  The inputs
are either written out in the fixture (small cases) or regenerated from the
seeded generators in oracle/oracle.py (with a SHA-256 of the fp32 bytes
stored, so a drift of the generator is detected).

Fixtures
--------
faiss_smoke.json     the FAISS v1.8 adapter smoke case of the reference
                     (tests/faiss_v1_8_cagra_runtime_smoke.cpp:236-245 inputs),
                     with the values it asserts (:299-306, :326-333, :353-357,
                     :376-383) checked against the reference run here.
dispatch_spy.npz     tests/test_metal_search.cpp:16-49 fixture (N=64, D=8,
                     Q=4, K=4) and the reference's answer.
l2_known.json        tests/test_l2_distance.cpp:16-51 known answers, evaluated
                     by the reference's squared_l2_distance_128.
c1_fp16.npz          config 1 (N=10,000, D=128, Q=100, K=10, i.i.d. N(0,1),
                     seeds 1/2) on fp16-rounded inputs: the primary parity
                     target of the fp16 engine.
c1_fp32.npz          config 1 on the raw fp32 inputs (the reference's own
                     ground truth; informational recall target).
ties.npz             integer-valued data with many exact ties and duplicate
                     rows (tie order by index), K > N padding, D = 3.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a, dtype=np.float32).tobytes()).hexdigest()


def faiss_smoke():
    database = np.array([[0, 0], [10, 0], [0, 10], [2, 2]], dtype=np.float32)
    queries = np.array([[0, 0], [9, 1]], dtype=np.float32)
    cases = []
    for name, q, k in [("search_k2", queries, 2), ("ordering_k4", queries[:1], 4),
                       ("oversized_single_k5", queries[:1], 5),
                       ("oversized_batched_k5", queries, 5)]:
        i, d = O.ref_knn(database, q, k)
        cases.append({"name": name, "queries": q.tolist(), "k": k,
                      "neighbors": i.astype(np.int64).tolist(),
                      "distances": [[float(x) if np.isfinite(x) else "inf" for x in row]
                                    for row in d]})
    # the values the reference's smoke test asserts
    c = {c["name"]: c for c in cases}
    assert c["search_k2"]["neighbors"] == [[0, 3], [1, 3]]
    assert c["search_k2"]["distances"] == [[0.0, 8.0], [2.0, 50.0]]
    assert c["ordering_k4"]["neighbors"] == [[0, 3, 1, 2]]
    assert c["ordering_k4"]["distances"] == [[0.0, 8.0, 100.0, 100.0]]
    assert c["oversized_single_k5"]["neighbors"][0][4] == O.NO_INDEX
    assert c["oversized_batched_k5"]["neighbors"][1][4] == O.NO_INDEX
    with open(os.path.join(OUT, "faiss_smoke.json"), "w") as f:
        json.dump({"source": "tests/faiss_v1_8_cagra_runtime_smoke.cpp:236-396",
                   "database": database.tolist(), "cases": cases}, f, indent=1)


def dispatch_spy():
    n, q, d, k = 64, 4, 8, 4
    base = np.zeros((n, d), np.float32)
    for i in range(n):
        base[i, i % d] = float(i)
    queries = np.zeros((q, d), np.float32)
    for j in range(q):
        queries[j, j % d] = 1.0
    i, dist = O.ref_knn(base, queries, k)
    np.savez_compressed(os.path.join(OUT, "dispatch_spy.npz"), base=base, queries=queries,
                        neighbors=i, distances=dist)


def l2_known():
    lib = O.ref_lib()
    dim = 128
    zeros = np.zeros(dim, np.float32)
    ones = np.ones(dim, np.float32)
    asc = np.arange(dim, dtype=np.float32)
    shifted = asc + np.float32(0.5)
    a = ((np.arange(dim) % 7) - 3).astype(np.float32) * np.float32(0.25)
    b = ((np.arange(dim) % 5) - 2).astype(np.float32) * np.float32(-0.5)
    out = []
    for name, x, y in [("zeros_ones", zeros, ones), ("ascending_shifted", asc, shifted),
                       ("mixed", a, b)]:
        v = lib.ref_squared_l2_distance_128(x.ctypes.data, y.ctypes.data)
        out.append({"name": name, "lhs": x.tolist(), "rhs": y.tolist(), "expected": float(v)})
    assert out[0]["expected"] == 128.0 and abs(out[1]["expected"] - 32.0) < 1e-4
    with open(os.path.join(OUT, "l2_known.json"), "w") as f:
        json.dump({"source": "tests/test_l2_distance.cpp:16-51", "cases": out}, f)


def c1():
    base = O.gen_iid(10000, 128, O.SEED_IID_BASE)
    queries = O.gen_iid(100, 128, O.SEED_IID_QUERIES)
    for tag, b, q in [("fp16", O.round_fp16(base), O.round_fp16(queries)),
                      ("fp32", base, queries)]:
        i, d = O.ref_knn(b, q, 10, threads=8)
        np.savez_compressed(os.path.join(OUT, f"c1_{tag}.npz"), neighbors=i, distances=d,
                            base_sha=sha(b), queries_sha=sha(q),
                            gen=np.array(["iid n=10000 d=128 seed=1; q=100 seed=2"]))


def ties():
    rng = np.random.Generator(np.random.PCG64(7))
    base = rng.integers(-2, 3, size=(40, 3)).astype(np.float32)
    base[10] = base[3]  # duplicate rows
    base[25] = base[3]
    queries = rng.integers(-2, 3, size=(6, 3)).astype(np.float32)
    queries[0] = base[3]
    i, d = O.ref_knn(base, queries, 45)  # k > n
    np.savez_compressed(os.path.join(OUT, "ties.npz"), base=base, queries=queries,
                        neighbors=i, distances=d)


if __name__ == "__main__":
    if not O.ref_available():
        O.build_native(quiet=False)
    faiss_smoke()
    dispatch_spy()
    l2_known()
    c1()
    ties()
    print("golden fixtures written to", OUT)
