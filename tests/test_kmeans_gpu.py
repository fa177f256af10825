"""Index training on the device against the oracle's restatement of
KMeans.cluster's Lloyd loop (Sources/MetalANNSCore/KMeans.swift:95-254) and
ProductQuantizer.train (ProductQuantizer.swift:10-86): centroids, codebooks
and assignments bit-equal, iteration counts equal, for the sequential and
the chunked (useParallelLloyd) summation orders, every SIMDDistance metric,
subspaces, empty clusters, duplicate rows and ties."""
import numpy as np
import pytest

import bench
import meltan_b200 as mb
import oracle as O
from meltan_b200 import train

pytestmark = pytest.mark.gpu

MET = [(mb.Metric.cosine, O.COSINE), (mb.Metric.l2, O.L2), (mb.Metric.innerProduct, O.IP)]


def same(got, want):
    np.testing.assert_array_equal(got[0], want[0])
    np.testing.assert_array_equal(got[1], want[1])
    assert got[2] == want[2]


@pytest.mark.parametrize("mg,mo", MET)
@pytest.mark.parametrize("n,dim,k,workers", [
    (100, 16, 5, 8),      # n < 512: one running sum
    (3000, 24, 40, 1),    # one worker
    (3000, 24, 40, 16),   # chunked sums
    (4099, 7, 64, 10),    # uneven chunks, odd width
    (700, 48, 6, 16),     # k < 8: sequential despite workers
])
def test_lloyd_equals_oracle(ctx, mg, mo, n, dim, k, workers):
    v, _ = bench.make_mixture(n, dim, max(2, k // 2), 1, sigma=0.4, seed=n + k)
    rng = np.random.default_rng(k)
    init = v[rng.choice(n, k, replace=False)].copy()
    same(train.kmeans_lloyd(ctx, v, init, 12, mg, workers),
         O.kmeans_lloyd(v, init, 12, mo, workers))


def test_lloyd_edge_cases(ctx):
    rng = np.random.default_rng(7)
    v = rng.standard_normal((900, 10), dtype=np.float32)
    # duplicated rows and duplicated initial centroids (ties: the lower index
    # wins), a far centroid that stays empty, zero iterations, k = n
    v[300:600] = v[:300]
    init = np.concatenate([v[:6], v[:2], np.full((1, 10), 50, np.float32)])
    for iters in (0, 1, 3, 50):
        same(train.kmeans_lloyd(ctx, v, init, iters, mb.Metric.l2, 12),
             O.kmeans_lloyd(v, init, iters, O.L2, 12))
    small = v[:9]
    same(train.kmeans_lloyd(ctx, small, small, 5, mb.Metric.cosine, 4),
         O.kmeans_lloyd(small, small, 5, O.COSINE, 4))
    with pytest.raises(mb.ConstructionFailed):
        train.kmeans_lloyd(ctx, small, v[:10], 5, mb.Metric.l2, 1)  # k > n
    with pytest.raises(mb.ConstructionFailed):
        train.kmeans_lloyd(ctx, v[:0], v[:1], 5, mb.Metric.l2, 1)   # empty


def test_lloyd_subspace(ctx):
    """KMeans.clusterSubspace: rows' [offset, offset + dim) only."""
    rng = np.random.default_rng(2)
    v = rng.standard_normal((2000, 32), dtype=np.float32)
    init = v[rng.choice(2000, 256, replace=False), 8:16].copy()
    same(train.kmeans_lloyd(ctx, v, init, 10, mb.Metric.l2, 16, offset=8, dim=8),
         O.kmeans_lloyd(v, init, 10, O.L2, 16, offset=8, dim=8))


def test_pq_train_equals_oracle(ctx):
    """ProductQuantizer.train on 1,000 x 128 vectors, m = 8, 8 iterations
    (ProductQuantizerTests.swift:8-24's shape)."""
    v, _ = bench.make_mixture(1000, 128, 20, 1, sigma=0.3, seed=11)
    rng = np.random.default_rng(4)
    m, sub = 8, 16
    init = np.stack([v[rng.choice(1000, 256, replace=False), s * sub:(s + 1) * sub]
                     for s in range(m)])
    for workers in (1, 10):
        got = train.pq_train(ctx, v, init, 8, workers)
        want = O.pq_train_codebooks(v, init, 8, workers)
        np.testing.assert_array_equal(got, want)
    with pytest.raises(mb.ConstructionFailed):
        train.pq_train(ctx, v[:200], init, 8, 1)  # fewer than 256 vectors


def test_partition_and_ivfpq_training_at_size(ctx):
    """The IVF-flat build's sample of a 1M x 384 corpus (nlist 256 -> 16 x 256
    = 4096 rows, stride 244) and its 8 cosine iterations, and IVFPQIndex.train
    on a 32,768 x 128 set with nlist 256 and m = 16, both against the
    oracle."""
    v, _ = bench.make_mixture(1_000_000, 384, 1024, 1, seed=0)
    sample, lists = train.partition_sample(v, 256)
    assert sample.shape == (4096, 384) and lists == 256
    np.testing.assert_array_equal(sample[1], v[244])
    init = sample[::16][:256].copy()
    got = train.train_partition(ctx, v, 256, init, mb.Metric.cosine, workers=16)
    want = O.kmeans_lloyd(sample, init, 8, O.COSINE, 16)[0]
    np.testing.assert_array_equal(got, want)
    del v
    x, _ = bench.make_mixture(32768, 128, 256, 1, seed=3)
    rng = np.random.default_rng(9)
    coarse0 = x[rng.choice(32768, 256, replace=False)].copy()
    books0 = (rng.standard_normal((16, 256, 8)) * 0.05).astype(np.float32)
    coarse, books = train.train_ivfpq(ctx, x, coarse0, books0, 4, mb.Metric.l2, workers=16)
    wc, wa, _ = O.kmeans_lloyd(x, coarse0, 4, O.L2, 16)
    np.testing.assert_array_equal(coarse, wc)
    resid = (x - wc[wa]).astype(np.float32)
    np.testing.assert_array_equal(books, O.pq_train_codebooks(resid, books0, 4, 16))
