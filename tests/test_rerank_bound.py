"""The exact re-rank certificate's rounding bound, checked on the CPU.

knn_rerank_bound is the function the re-rank kernel evaluates (it is built
for host and device).  For a query q and a row x it must bound the gap
between the scan's distance (fp16-rounded vectors, fp32 norms, fp32
accumulation of the exact fp16 products, one fused multiply-add) and the
reference's fp32 distance (sequential sum over d of (q[d] - x[d])^2 in fp32,
src/cagra.cpp:218-226).  The scan's arithmetic is emulated here with
several accumulation orders, on Gaussian vectors at scales that reach the
fp16 subnormal range and large magnitudes, on near-duplicate pairs (tiny
distances, where the relative error is largest) and for both metrics.
"""
import numpy as np
import pytest

F32 = np.float32


def _seq_sum(terms):
    """Sequential fp32 sum over the last axis (every addition rounded)."""
    acc = np.zeros(terms.shape[0], dtype=F32)
    for j in range(terms.shape[1]):
        acc = (acc + terms[:, j]).astype(F32)
    return acc


def _sums(terms):
    """fp32 sums of the same terms in several orders."""
    t = terms.astype(F32)
    out = [_seq_sum(t), t.sum(axis=1, dtype=F32)]
    if t.shape[1] >= 16 and t.shape[1] % 16 == 0:  # blocks of 16, then sequential
        out.append(_seq_sum(t.reshape(t.shape[0], -1, 16).sum(axis=2, dtype=F32)))
    return out


def _pairs(rng, n, dim, scale, kind):
    q = (rng.standard_normal((n, dim)) * scale).astype(F32)
    if kind == "gauss":
        x = (rng.standard_normal((n, dim)) * scale).astype(F32)
    else:  # near-duplicates: x = q plus noise well below the values
        x = (q + rng.standard_normal((n, dim)) * (scale * 1e-3)).astype(F32)
    return q, x


@pytest.mark.parametrize("dim", [4, 64, 1024])
@pytest.mark.parametrize("scale", [1e-3, 1.0, 100.0])
@pytest.mark.parametrize("kind", ["gauss", "near"])
def test_bound_covers_scan_vs_fp32(engine, dim, scale, kind):
    rng = np.random.Generator(np.random.PCG64(dim * 7 + int(scale * 1000) + len(kind)))
    q, x = _pairs(rng, 400, dim, scale, kind)
    q16 = q.astype(np.float16).astype(F32)
    x16 = x.astype(np.float16).astype(F32)
    qn = np.sqrt((q.astype(np.float64) ** 2).sum(1))
    xn = np.sqrt((x.astype(np.float64) ** 2).sum(1))

    # reference: sequential fp32 sum of the squared differences
    diff = (q - x).astype(F32)
    d32 = _seq_sum((diff * diff).astype(F32))
    s32 = _seq_sum((q * x).astype(F32))
    bl = np.array([engine.rerank_bound(0, float(d32[i]), qn[i], xn[i], dim)
                   for i in range(len(d32))])
    bi = np.array([engine.rerank_bound(1, 0.0, qn[i], xn[i], dim) for i in range(len(d32))])
    assert np.all(bl > 0) and np.all(bi > 0)

    prods = q16 * x16  # exact in fp32 (fp16 x fp16)
    for dot in _sums(prods):
        for nq in _sums(q16 * q16):
            for nx in _sums(x16 * x16):
                s = (nq + nx).astype(F32)
                d16 = (s.astype(np.float64) - 2.0 * dot.astype(np.float64)).astype(F32)
                d16 = np.maximum(d16, F32(0))
                gap = np.abs(d16.astype(np.float64) - d32.astype(np.float64))
                assert np.all(gap <= bl), (gap / bl).max()
        gap_ip = np.abs(dot.astype(np.float64) - s32.astype(np.float64))
        assert np.all(gap_ip <= bi), (gap_ip / bi).max()


def test_bound_arguments(engine):
    assert engine.rerank_bound(0, 1.0, 1.0, 1.0, 0) < 0
    assert engine.rerank_bound(0, 1.0, -1.0, 1.0, 8) < 0
    # grows with the distance, the norms and the dimension
    b = engine.rerank_bound(0, 0.1, 1.0, 1.0, 128)
    assert engine.rerank_bound(0, 1.0, 1.0, 1.0, 128) > b
    assert engine.rerank_bound(0, 0.1, 2.0, 2.0, 128) > b
    assert engine.rerank_bound(0, 0.1, 1.0, 1.0, 1024) > b
