"""GPU parity of the small-corpus batch search (score tiles + per-query sort,
small_scan.cu) against the oracle: batches of at least 64 queries over at
most 8192 rows, the shape of the centroid steps of both index searches.

Reached three ways: the public flat search with the tensor-core path
switched off, the IVF-flat centroid top-nprobe (host-tier keys) and the
IVF-PQ coarse selection (SIMDDistance keys, 2 x nprobe candidates).  Ids are
compared exactly and distances bit for bit."""
import numpy as np
import pytest

import bench
import meltan_b200 as mb
import oracle as O

pytestmark = pytest.mark.gpu

MET = [(mb.Metric.cosine, O.COSINE), (mb.Metric.l2, O.L2), (mb.Metric.innerProduct, O.IP)]


def same(got, want):
    np.testing.assert_array_equal(got[2], want[2])
    np.testing.assert_array_equal(got[1], want[1])
    np.testing.assert_array_equal(got[0], want[0])


@pytest.mark.parametrize("mg,mo", MET)
@pytest.mark.parametrize("n,dim,nq,k", [
    (1, 8, 64, 10),        # fewer rows than k
    (63, 3, 64, 5),        # ragged row tile, dims below one staging step
    (64, 64, 65, 64),      # exact tiles, one query past a query tile
    (65, 65, 100, 1),      # k = 1: the block-minimum select
    (1000, 128, 130, 256), # k at the public cap
    (4096, 130, 64, 10),   # dims across three staging steps
    (8192, 384, 96, 100),  # the largest corpus the path takes
])
def test_small_batch_flat_parity(ctx, mg, mo, n, dim, nq, k):
    rng = np.random.default_rng(n + dim)
    v = rng.standard_normal((n, dim), dtype=np.float32)
    if n >= 8:
        v[3] = v[5]        # duplicate rows: equal distances ordered by id
        v[7] = 0.0         # zero row: the cosine denominator guard
    q = rng.standard_normal((nq, dim), dtype=np.float32)
    q[1] = 0.0             # zero query: -0 inner products
    ctx.set_tensor_core_batch(0)
    try:
        buf = mb.VectorBuffer(ctx, v)
        got = mb.FlatGPUSearch.batch_search_arrays(ctx, q, buf, k, mg)
        buf.close()
    finally:
        ctx.set_tensor_core_batch(16)
    same(got, O.flat_search(v, q, k, mo))


@pytest.mark.parametrize("mg,mo", MET)
def test_small_batch_ivf_centroid_step(ctx, mg, mo):
    v, q = bench.make_mixture(20000, 64, 50, 100, seed=7)
    rng = np.random.default_rng(8)
    cent = v[rng.choice(len(v), 96, replace=False)].copy()
    assign = O.ivf_assign(v, cent, mo)
    off, ids, packed, pn = O.ivf_layout(v, assign, len(cent))
    part = mb.Partition(ctx, cent, packed, ids, off)
    for nprobe, k in ((1, 10), (8, 25), (96, 5)):
        same(mb.IVFFlatSearch.search_arrays(ctx, q, part, k, nprobe, mg),
             O.ivf_search(cent, packed, pn, ids, off, q, k, nprobe, mo))
    part.close()


@pytest.mark.parametrize("metric", [O.L2, O.COSINE, O.IP])
def test_small_batch_ivfpq_coarse_step(ctx, metric):
    rng = np.random.default_rng(12)
    v, q = bench.make_mixture(4000, 32, 16, 80, sigma=0.2, seed=12)
    coarse = v[rng.choice(len(v), 40, replace=False)].copy()
    coarse[5] = coarse[9]  # equal coarse scores: BoundedSortedList order
    cb = (rng.standard_normal((8, 256, 4)) * 0.1).astype(np.float32)
    codes, assign = mb.pq_encode(ctx, v, coarse, cb, mb.Metric(metric))
    flat = np.argsort(assign, kind="stable").astype(np.uint32)
    off = np.concatenate([[0], np.cumsum(np.bincount(assign, minlength=40))]).astype(np.int64)
    ix = mb.IVFPQIndex(ctx, coarse, cb, codes, (off, flat), metric=mb.Metric(metric))
    for nprobe, k in ((1, 10), (4, 10), (16, 57), (40, 3)):
        same(ix.search_arrays(q, k, nprobe),
             O.ivfpq_search(coarse, cb, codes, off, flat, q, k, nprobe, metric))
    ix.close()
