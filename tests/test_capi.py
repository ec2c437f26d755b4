"""CPU tests of the C-ABI library: it loads, exports every function the
header declares, and its host-only logic (status strings, argument
validation, planner, shard ranges) behaves.  No compute call needs a GPU."""
import ctypes

import pytest


def test_library_exports_every_header_symbol(engine):
    names = engine.header_functions()
    assert len(names) >= 20
    lib = engine.lib()
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_status_strings(engine):
    lib = engine.lib()
    assert lib.knn_status_string(0) == b"KNN_OK"
    assert lib.knn_status_string(engine.KNN_EINVAL) == b"KNN_EINVAL"
    assert lib.knn_status_string(engine.KNN_ETIMEOUT) == b"KNN_ETIMEOUT"
    assert lib.knn_status_string(99) == b"KNN_UNKNOWN"


def test_null_handles_are_einval(engine):
    lib = engine.lib()
    assert lib.knn_index_build(None, None, 0, 1, 1, 0) == engine.KNN_EINVAL
    assert lib.knn_index_search(None, None, 1, 1, None, None) == engine.KNN_EINVAL
    assert lib.knn_index_sync(None) == engine.KNN_EINVAL
    assert lib.knn_index_destroy(None) == engine.KNN_OK
    assert lib.knn_index_create(0, None) == engine.KNN_EINVAL
    assert b"null" in lib.knn_last_error()


def test_create_without_gpu_fails_cleanly(engine):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    st = engine.lib().knn_index_create(0, ctypes.byref(h))
    assert st == engine.KNN_ECUDA and not h.value
    with pytest.raises(RuntimeError, match="KNN_ECUDA"):
        engine.Index(0)


def test_planner_headline(engine):
    p = engine.plan_search(1_000_000, 1024, 100, 10)
    assert p["query_block"] == 128 and p["query_tiles"] == 1
    assert p["row_tiles"] == 3907 and p["splits"] == 148 and p["grid"] == 148
    assert p["stages"] >= 4
    assert p["smem_bytes"] <= 232448
    assert p["partial_bytes"] == 100 * 148 * 10 * 8


@pytest.mark.parametrize("nq,k", [(1, 10), (16, 256), (100, 256), (10000, 100),
                                  (1, 256), (33, 1), (100, 100), (129, 10), (300, 10),
                                  (1000, 10), (10000, 10), (600, 32), (200, 32)])
def test_planner_fits_shared_memory(engine, nq, k):
    p = engine.plan_search(1_000_000, 1024, nq, k)
    assert p["smem_bytes"] <= 232448
    assert p["stages"] >= 2
    assert p["query_block"] % 32 == 0 and 32 <= p["query_block"] <= 128
    assert p["query_tiles"] * p["unit_queries"] >= nq
    # CTA pairs for more than 128 queries where one CTA would keep fewer
    # than 3 stages (k >= 62) or pairs pad the queries by at most 5% more
    single_rows, pair_rows = -(-nq // 128) * 128, -(-nq // 256) * 256
    want = nq > 128 and (k >= 62 or 20 * pair_rows <= 21 * single_rows)
    assert p["pair"] == (1 if want else 0), p
    if p["pair"]:
        assert p["grid"] % 2 == 0 and p["unit_queries"] == 256 and p["query_block"] == 128
    assert p["units"] == p["query_tiles"] * p["splits"]
    assert 1 <= p["splits"] <= p["row_tiles"]
    assert p["grid"] == (2 * min(p["units"], 74) if p["pair"] else min(p["units"], 148))
    if p["compact_heap"]:
        gran = 64 if p["pair"] else 32
        n_gran = -(-1_000_000 // gran)
        assert k > 16 and -(-n_gran // p["splits"]) * gran <= 65535


def test_planner_compact_heaps(engine):
    # compact 6-byte heap entries where they buy a pipeline stage and every
    # unit spans at most 65,535 rows; full keys otherwise
    c4 = engine.plan_search(1_250_000, 1024, 10_000, 100)
    assert c4["pair"] == 1 and c4["compact_heap"] == 1 and c4["stages"] == 4
    big = engine.plan_search(10_000_000, 1024, 10_000, 100)
    assert big["pair"] == 1 and big["compact_heap"] == 0 and big["stages"] == 3
    single = engine.plan_search(1_000_000, 1024, 128, 64)
    assert single["pair"] == 0 and single["compact_heap"] == 1 and single["stages"] == 3
    # a single query tile keeps heaps only for the batch's rows (104 of 128
    # at Q = 100), which leaves room for a third stage at K = 100
    q100 = engine.plan_search(1_000_000, 1024, 100, 100)
    assert q100["pair"] == 0 and q100["stages"] == 3 and q100["smem_bytes"] <= 232448
    assert engine.plan_search(1_000_000, 1024, 100, 10)["compact_heap"] == 0
    c5 = engine.plan_search(1_000_000, 1024, 16, 256)  # heaps for 16 rows: 4 stages
    assert c5["compact_heap"] == 1 and c5["stages"] == 4


def test_planner_limits(engine):
    with pytest.raises(RuntimeError, match="UNSUPPORTED"):
        engine.plan_search(1000, 64, 10, 257)
    with pytest.raises(ValueError):
        engine.plan_search(0, 64, 10, 10)
    p = engine.plan_search(4, 2, 2, 2)  # the FAISS smoke shape
    assert p["row_tiles"] == 1 and p["splits"] == 1 and p["grid"] == 1


def test_shard_ranges_cover_rows(engine):
    for n in [1, 7, 1000, 1_000_000, 10_000_000]:
        for g in [1, 2, 3, 4, 8]:
            ranges = [engine.shard_range(n, g, r) for r in range(g)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            for (a, b), (c, d) in zip(ranges, ranges[1:]):
                assert b == c and a <= b
    assert engine.shard_range(1_000_000, 8, 3) == (375000, 500000)
    with pytest.raises(ValueError):
        engine.shard_range(10, 2, 2)


def test_dispatch_counter_resets(engine):
    engine.reset_dispatch_count()
    assert engine.dispatch_count() == 0


def test_comm_unique_id_is_128_bytes(engine):
    try:
        uid = engine.comm_unique_id()
    except RuntimeError as e:  # NCCL may refuse without any network interface
        pytest.skip(str(e))
    assert len(uid) == 128
