"""GPU tests of the list merge (merge_kernel) on its own, through the C ABI
(knn_merge_lists), against the oracle's merge of the same lists.

The lists are built to reach every ordering path of the merge: long full
lists (a threshold from the lists' j-th entries, then a radix select of the
k-th distance), many short lists (fewer than r lists hold j entries, so
there is no threshold and every valid entry is a candidate), ties at the
k-th distance (the fallback that sorts every candidate), small k, and the
inner product's negative internal distances.  Results must be identical
bit for bit: the merge only reorders its inputs.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

NO_INDEX = 0xFFFFFFFF


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def make_lists(rng, n_lists, nq, k, pattern, negative=False):
    """Lists [n_lists][nq][k]: sorted valid prefixes (distinct row indices
    per query), padded with (+inf, UINT32_MAX)."""
    d = np.full((n_lists, nq, k), np.inf, np.float32)
    i = np.full((n_lists, nq, k), NO_INDEX, np.uint32)
    for q in range(nq):
        rows = rng.permutation(n_lists * k * 4)[: n_lists * k].astype(np.uint32)
        for l in range(n_lists):
            if pattern == "full":
                n = k
            elif pattern == "short":
                n = int(rng.integers(0, 8))
            elif pattern == "shortish":
                n = int(rng.integers(0, 40))
            elif pattern == "mixed":  # mostly short lists, every third long
                n = int(rng.integers(40, k + 1)) if l % 3 == 0 else int(rng.integers(0, 4))
            else:  # ties: few distinct distances
                n = int(rng.integers(k // 2, k + 1))
            if pattern == "ties":
                v = rng.integers(0, 6, n).astype(np.float32) * 0.25 + 1.0
            else:
                v = rng.random(n, dtype=np.float32) * 4.0
            if negative:
                v = v - 2.0
            ids = rows[l * k: l * k + n]
            order = np.lexsort((ids, v))
            d[l, q, :n] = v[order]
            i[l, q, :n] = ids[order]
    return d, i


CASES = [
    # (n_lists, nq, k, pattern, inner product)
    (148, 4, 256, "full", False),
    (148, 4, 256, "short", False),
    (148, 3, 256, "ties", False),
    (64, 3, 100, "shortish", False),
    (148, 5, 10, "full", False),
    (148, 5, 10, "short", False),
    (8, 7, 10, "ties", False),
    (148, 2, 256, "short", True),
    (24, 3, 200, "ties", True),
    # too few lists hold j entries for a threshold: the first 8 entries of
    # every list bound the k-th instead (exact when the lists are short,
    # loose when some are long)
    (148, 3, 256, "mixed", False),
    (148, 3, 100, "mixed", True),
    (200, 2, 64, "mixed", False),
]


@pytest.mark.parametrize("n_lists,nq,k,pattern,ip", CASES)
def test_merge_lists_matches_oracle(engine, oracle_mod, torch_cuda, n_lists, nq, k, pattern, ip):
    torch = torch_cuda
    rng = np.random.Generator(np.random.PCG64(n_lists * 131 + nq * 17 + k + len(pattern)))
    d, i = make_lists(rng, n_lists, nq, k, pattern, negative=ip)
    dev = torch.device("cuda", 0)
    ld = torch.from_numpy(d).to(dev)
    li = torch.from_numpy(i.view(np.int32)).to(dev)
    out_i = torch.empty((nq, k), dtype=torch.int32, device=dev)
    out_d = torch.empty((nq, k), dtype=torch.float32, device=dev)
    metric = engine.METRIC_INNER_PRODUCT if ip else engine.METRIC_L2_EXPANDED
    st = engine.lib().knn_merge_lists(0, None, ctypes.c_void_p(ld.data_ptr()),
                                      ctypes.c_void_p(li.data_ptr()), n_lists, nq, k, metric,
                                      ctypes.c_void_p(out_i.data_ptr()), 0,
                                      ctypes.c_void_p(out_d.data_ptr()))
    torch.cuda.synchronize()
    assert st == 0, engine.lib().knn_last_error()
    gi = out_i.cpu().numpy().view(np.uint32)
    gd = out_d.cpu().numpy()
    # oracle: lists as (nq, n_lists, k)
    oi, od = oracle_mod.merge_lists(np.ascontiguousarray(d.transpose(1, 0, 2)),
                                    np.ascontiguousarray(i.transpose(1, 0, 2)))
    if ip:
        od = np.where(oi == NO_INDEX, -np.inf, -od).astype(np.float32)
    assert np.array_equal(gi, oi), (pattern, np.argwhere(gi != oi)[:5])
    assert np.array_equal(gd.view(np.uint32), od.view(np.uint32)), pattern
