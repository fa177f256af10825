"""GPU int8 prefilter path (row f4): tcgen05 kind::i8 candidate pass over the
reference's Int8CodeBuffer codes, certified bound, exact fp32 re-score.

* codes and scales bit-equal to the oracle's restatement of
  Int8CodeBuffer.fill (Int8CodeCache.swift:64-99);
* results bit-equal (ids and distances) to the oracle's exact search on the
  cases of Tests/MetalANNSTests/BoundedExactScanTests.swift: metrics x dims
  {384, 128, 333, 16} x seeds {7, 99} x k {1, 24, 97} (:176-208), adversarial
  rows (:212-250), zero query (:253-274), k up to 256 (:277-303), mutation
  (:306-336)."""
import numpy as np
import pytest

import meltan_b200 as mb
import oracle as O

pytestmark = pytest.mark.gpu

MET = [(mb.Metric.cosine, O.COSINE), (mb.Metric.l2, O.L2), (mb.Metric.innerProduct, O.IP)]
CORPUS = 16384 + 512  # BoundedExactScanTests.corpusSize


@pytest.fixture(scope="module")
def i8ctx():
    c = mb.Context(0)
    c.set_tensor_core_batch(1)
    c.set_tensor_core_format(mb.TC_INT8)
    yield c
    c.close()


def same(got, want):
    np.testing.assert_array_equal(got[2], want[2])
    np.testing.assert_array_equal(got[1], want[1])
    np.testing.assert_array_equal(got[0], want[0])


def test_int8_codes_match_reference_quantisation(i8ctx):
    v = O.lcg32_vectors(3000, 333, 7)
    v[::97] = 0.0
    v[5::97] *= np.float32(1e5)
    buf = mb.VectorBuffer(i8ctx, v)
    codes, scales = buf.int8_codes()
    want_c, want_s = O.int8_fill(v)
    np.testing.assert_array_equal(scales, want_s)
    np.testing.assert_array_equal(codes, want_c)
    buf.close()


@pytest.mark.parametrize("dim", [384, 128, 333, 16])
@pytest.mark.parametrize("seed", [7, 99])
def test_int8_exact_across_metrics_dims_seeds(i8ctx, dim, seed):
    v = O.lcg32_vectors(CORPUS, dim, seed)
    q = O.lcg32_vectors(4, dim, seed + 123)
    buf = mb.VectorBuffer(i8ctx, v)
    for mg, mo in MET:
        for k in (1, 24, 97):
            same(mb.FlatGPUSearch.batch_search_arrays(i8ctx, q, buf, k, mg),
                 O.flat_search(v, q, k, mo))
    buf.close()


def test_int8_adversarial_rows(i8ctx):
    dim = 64
    # the test's draw order: base row, then one row per non-zero, non-duplicate
    # row in order, then the query
    nrand = sum(1 for row in range(CORPUS) if row % 4 >= 2)
    draws = O.lcg32_vectors(1 + nrand + 1, dim, 2024)
    base = draws[0]
    v = np.empty((CORPUS, dim), np.float32)
    j = 1
    for row in range(CORPUS):
        m = row % 4
        if m == 0:
            v[row] = 0.0
        elif m == 1:
            v[row] = base
        else:
            mag = np.float32(1e-5) if row % 8 == 0 else (np.float32(1e5) if row % 8 == 4 else np.float32(1))
            v[row] = draws[j] * mag
            j += 1
    q = draws[j:j + 1].copy()
    buf = mb.VectorBuffer(i8ctx, v)
    for mg, mo in MET:
        for k in (24, 256):
            same(mb.FlatGPUSearch.batch_search_arrays(i8ctx, q, buf, k, mg),
                 O.flat_search(v, q, k, mo))
    buf.close()


def test_int8_zero_query_and_large_k(i8ctx):
    v = O.lcg32_vectors(CORPUS, 96, 31)
    buf = mb.VectorBuffer(i8ctx, v)
    zq = np.zeros((1, 96), np.float32)
    for mg, mo in MET:
        same(mb.FlatGPUSearch.batch_search_arrays(i8ctx, zq, buf, 24, mg),
             O.flat_search(v, zq, 24, mo))
    buf.close()
    v = O.lcg32_vectors(CORPUS, 384, 55)
    q = O.lcg32_vectors(1, 384, 77)
    buf = mb.VectorBuffer(i8ctx, v)
    for mg, mo in MET:
        for k in (97, 256):
            same(mb.FlatGPUSearch.batch_search_arrays(i8ctx, q, buf, k, mg),
                 O.flat_search(v, q, k, mo))
    buf.close()


def test_int8_codes_invalidate_after_mutation(i8ctx):
    v = O.lcg32_vectors(CORPUS, 48, 5)
    q = O.lcg32_vectors(3, 48, 6)
    buf = mb.VectorBuffer(i8ctx, v)
    mb.FlatGPUSearch.batch_search_arrays(i8ctx, q, buf, 10, mb.Metric.l2)
    v2 = v.copy()
    v2[100:103] = q
    buf.batch_insert(q, 100)
    for mg, mo in MET:
        same(mb.FlatGPUSearch.batch_search_arrays(i8ctx, q, buf, 10, mg),
             O.flat_search(v2, q, 10, mo))
    codes, _ = buf.int8_codes()
    np.testing.assert_array_equal(codes, O.int8_fill(v2)[0])
    buf.close()


@pytest.mark.parametrize("nq", [1, 7, 64, 200])
def test_int8_batches_unit_rows(i8ctx, nq):
    rng = np.random.default_rng(nq)
    v = rng.standard_normal((50000, 384), dtype=np.float32)
    v /= np.linalg.norm(v, axis=1, keepdims=True)
    q = rng.standard_normal((nq, 384), dtype=np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    buf = mb.VectorBuffer(i8ctx, v)
    for mg, mo in MET:
        same(mb.FlatGPUSearch.batch_search_arrays(i8ctx, q, buf, 10, mg),
             O.flat_search(v, q, 10, mo))
    buf.close()
