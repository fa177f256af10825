"""The oracle's restatement of BoundedExactScan (the reference's CPU batch
route at n >= 16384: int8 prefilter with provable lower bounds, fp32 rescore,
budget x4 until proven) against the exact brute force: identical ids and
distances, including data that defeats the first rounds of the prefilter.
Cases follow Tests/MetalANNSTests/BoundedExactScanTests.swift (exactness over
metrics and k, duplicate clusters)."""
import numpy as np
import pytest

import oracle as O


def unit_rows(rng, n, d):
    v = rng.standard_normal((n, d), dtype=np.float32)
    return v / np.linalg.norm(v, axis=1, keepdims=True)


def same(got, want, k):
    gd, gi, gc = got
    wd, wi, wc = want
    kk = min(k, gd.shape[1])
    np.testing.assert_array_equal(gc, wc)
    np.testing.assert_array_equal(gi[:, :kk], wi[:, :kk])
    np.testing.assert_array_equal(gd[:, :kk], wd[:, :kk])


def test_planes_follow_int8_code_buffer_fill():
    rng = np.random.default_rng(1)
    v = rng.standard_normal((300, 40), dtype=np.float32)
    v[7] = 0.0
    codes, u, w, nsq, inv = O.int8_planes(v)
    c8, s8 = O.int8_fill(v)
    np.testing.assert_array_equal(codes, c8)
    np.testing.assert_array_equal(u, s8)
    np.testing.assert_array_equal(nsq, O.row_norms(v))
    absum = np.abs(codes.astype(np.int32)).sum(1).astype(np.float32)
    ebase = ((absum / np.float32(2) + np.float32(40) / np.float32(4))
             * np.float32(1.0 + 1e-6) + np.float32(16)).astype(np.float32)
    np.testing.assert_array_equal(w, (u * ebase).astype(np.float32))
    assert inv[7] == 0.0 and u[7] == 1.0


@pytest.mark.parametrize("metric", [O.COSINE, O.L2, O.IP])
@pytest.mark.parametrize("k", [1, 10, 100, 256])
def test_bounded_scan_equals_brute_force(metric, k):
    rng = np.random.default_rng(k + 10 * metric)
    v = unit_rows(rng, 20000, 48)
    q = rng.standard_normal((6, 48), dtype=np.float32)
    planes = O.int8_planes(v)
    same(O.bounded_exact_batch(v, planes, q, k, metric, threads=3),
         O.flat_search(v, q, k, metric), k)


@pytest.mark.parametrize("metric", [O.COSINE, O.L2, O.IP])
def test_dense_cluster_grows_the_budget_and_stays_exact(metric):
    """A few thousand rows within quantisation error of each other around the
    query: the first budgets cannot prove the cutoff, the scan widens until
    it can (or covers every row), and the answer stays the brute force."""
    rng = np.random.default_rng(5)
    v = unit_rows(rng, 20000, 32)
    q = rng.standard_normal((3, 32), dtype=np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    v[:3000] = q[0] + rng.standard_normal((3000, 32), dtype=np.float32) * 1e-3
    v[3000:3004] = v[10]  # exact duplicates: ties ordered by id
    planes = O.int8_planes(v)
    for k in (10, 64):
        same(O.bounded_exact_batch(v, planes, q, k, metric, threads=2),
             O.flat_search(v, q, k, metric), k)


def test_small_corpus_is_declined():
    rng = np.random.default_rng(2)
    v = unit_rows(rng, 16383, 16)
    q = rng.standard_normal((2, 16), dtype=np.float32)
    _, _, c = O.bounded_exact_batch(v, O.int8_planes(v), q, 10, O.L2, threads=1)
    np.testing.assert_array_equal(c, [-1, -1])


def test_reference_dots_give_the_same_answer():
    if O.ref_lib() is None:
        pytest.skip("the reference dots.c was not built here")
    rng = np.random.default_rng(3)
    v = unit_rows(rng, 17000, 40)
    q = rng.standard_normal((4, 40), dtype=np.float32)
    planes = O.int8_planes(v)
    a = O.bounded_exact_batch(v, planes, q, 10, O.COSINE, threads=2, use_reference_dots=True)
    b = O.bounded_exact_batch(v, planes, q, 10, O.COSINE, threads=2, use_reference_dots=False)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)
