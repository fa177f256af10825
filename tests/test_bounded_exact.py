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


# ---- the cases of Tests/MetalANNSTests/BoundedExactScanTests.swift, on the
# oracle's restatement (data from its seeded generator, restated as
# oracle.lcg32_vectors) ------------------------------------------------------

CORPUS = 16384 + 512  # BoundedExactScanTests.corpusSize
MET = (O.COSINE, O.L2, O.IP)


@pytest.mark.parametrize("dim", [384, 128, 333, 16])
@pytest.mark.parametrize("seed", [7, 99])
def test_reference_cases_across_metrics_dims_seeds(dim, seed):
    """exactAcrossMetricsDimsAndSeeds (:176-208)."""
    v = O.lcg32_vectors(CORPUS, dim, seed)
    q = O.lcg32_vectors(4, dim, seed + 123)
    planes = O.int8_planes(v)
    for metric in MET:
        for k in (1, 24, 97):
            same(O.bounded_exact_batch(v, planes, q, k, metric, threads=4),
                 O.flat_search(v, q, k, metric), k)


def test_reference_case_adversarial_rows():
    """adversarialDataStaysExact (:212-250): quarter zero rows, quarter
    copies of one row, the rest spread over magnitudes 1e-5 .. 1e5."""
    dim = 64
    nrand = sum(1 for row in range(CORPUS) if row % 4 >= 2)
    draws = O.lcg32_vectors(1 + nrand + 1, dim, 2024)
    v = np.empty((CORPUS, dim), np.float32)
    j = 1
    for row in range(CORPUS):
        m = row % 4
        if m == 0:
            v[row] = 0.0
        elif m == 1:
            v[row] = draws[0]
        else:
            mag = (np.float32(1e-5) if row % 8 == 0 else
                   (np.float32(1e5) if row % 8 == 4 else np.float32(1)))
            v[row] = draws[j] * mag
            j += 1
    q = draws[j:j + 1].copy()
    planes = O.int8_planes(v)
    for metric in MET:
        for k in (24, 256):
            same(O.bounded_exact_batch(v, planes, q, k, metric, threads=2),
                 O.flat_search(v, q, k, metric), k)


def test_reference_cases_zero_query_and_large_k():
    """zeroQueryStaysExact (:253-274) and largeKMultiRoundGrowthStaysExact
    (:277-303)."""
    v = O.lcg32_vectors(CORPUS, 96, 31)
    zq = np.zeros((1, 96), np.float32)
    planes = O.int8_planes(v)
    for metric in MET:
        same(O.bounded_exact_batch(v, planes, zq, 24, metric, threads=1),
             O.flat_search(v, zq, 24, metric), 24)
    v = O.lcg32_vectors(CORPUS, 384, 55)
    q = O.lcg32_vectors(1, 384, 77)
    planes = O.int8_planes(v)
    for metric in MET:
        for k in (97, 256):
            same(O.bounded_exact_batch(v, planes, q, k, metric, threads=1),
                 O.flat_search(v, q, k, metric), k)


def test_reference_case_tail_rows_are_covered():
    """sliceCoverageCoversEntireCorpus (:355-393): targets in the last rows
    of a 4 x 16384-row corpus, perturbed so they are the strict nearest."""
    dim, count = 64, 4 * 16384
    v = O.lcg32_vectors(count, dim, 404)
    targets = [count - 1, count - 7, count // 2 + 3]
    queries = [v[t].copy() for t in targets]
    noise = O.lcg32_vectors(2 * len(targets), dim, 405)
    for i, t in enumerate(targets):
        v[t] = v[t] + noise[i] * np.float32(1e-3)
    q = np.stack([queries[i] + noise[len(targets) + i] * np.float32(1e-3)
                  for i in range(len(targets))]).astype(np.float32)
    planes = O.int8_planes(v)
    got = O.bounded_exact_batch(v, planes, q, 5, O.L2, threads=3)
    want = O.flat_search(v, q, 5, O.L2)
    same(got, want, 5)
    np.testing.assert_array_equal(got[1][:, 0], targets)
