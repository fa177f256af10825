"""Index training on the device over the C ABI.

* ``kmeans_lloyd``   -- KMeans.cluster's Lloyd iterations (Sources/
                        MetalANNSCore/KMeans.swift:95-254) from given initial
                        centroids; bit-equal to the reference run on a machine
                        with ``workers`` cores (its chunked summation order).
* ``pq_train``       -- ProductQuantizer.train (Sources/MetalANNSCore/
                        ProductQuantizer.swift:10-86) from initial codebooks.
* ``partition_sample`` / ``train_partition`` -- the IVF-flat build's strided
                        sample and its 8 Lloyd iterations (IVFFlatSearch.
                        buildPartition, IVFFlatSearch.swift:517-551).
* ``train_ivfpq``    -- IVFPQIndex.train (Sources/MetalANNS/IVFPQIndex.swift:
                        54-104): coarse Lloyd, residuals to the assigned
                        centroid, PQ training on the residuals.

The k-means++ seeds (KMeans.swift:256-328) come from Swift's random number
API; callers pass initial centroids instead.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import lib
from .core import Context, Metric, check


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _vp(a):
    return C.c_void_p(a.ctypes.data)


def kmeans_lloyd(ctx: Context, vectors, centroids, max_iterations: int,
                 metric: Metric = Metric.l2, workers: int = 1, offset: int = 0, dim=None):
    """Returns (centroids k x dim, assignments n, centroid updates)."""
    v = _f32(vectors)
    n, stride = v.shape
    dim = stride - offset if dim is None else dim
    cent = np.array(_f32(centroids), copy=True)
    assign = np.empty(n, np.int32)
    it = C.c_int32()
    check(lib().mans_kmeans_lloyd(ctx.handle, _vp(v), n, stride, offset, dim, cent.shape[0],
                                  max_iterations, int(metric), workers, _vp(cent), _vp(assign),
                                  C.byref(it)))
    return cent, assign, it.value


def pq_train(ctx: Context, vectors, codebooks, max_iterations: int = 20, workers: int = 1):
    """Trained codebooks (m x 256 x dim/m) from the initial ones."""
    v = _f32(vectors)
    cb = np.array(_f32(codebooks), copy=True)
    m, ks, _ = cb.shape
    check(lib().mans_pq_train(ctx.handle, _vp(v), v.shape[0], v.shape[1], m, ks, max_iterations,
                              workers, _vp(cb)))
    return cb


def partition_sample(corpus, nlist: int):
    """IVFFlatSearch.buildPartition's k-means sample (IVFFlatSearch.swift:
    527-544): lists = min(max(1, nlist), n); min(n, max(lists, min(4096,
    max(16 lists, lists)))) rows with stride max(1, n / count), topped up by
    rows (count % n) when the stride runs off the end."""
    n = corpus.shape[0]
    lists = min(max(1, nlist), n)
    count = min(n, max(lists, min(4096, max(lists * 16, lists))))
    stride = max(1, n // count)
    idx = list(range(0, n, stride))[:count]
    while len(idx) < count:
        idx.append(len(idx) % n)
    return corpus[np.asarray(idx, np.int64)], lists


def train_partition(ctx: Context, corpus, nlist: int, initial, metric: Metric,
                    workers: int = 1):
    """The centroids buildPartition trains: 8 Lloyd iterations over its
    sample from `initial` (lists x dim)."""
    sample, lists = partition_sample(corpus, nlist)
    cent, _, _ = kmeans_lloyd(ctx, sample, initial[:lists], 8, metric, workers)
    return cent


def train_ivfpq(ctx: Context, vectors, coarse_initial, codebooks_initial, iterations: int,
                metric: Metric = Metric.l2, workers: int = 1):
    """IVFPQIndex.train from initial coarse centroids and codebooks: returns
    (coarse centroids, codebooks).  The residual of a vector is vector -
    centroid, element by element in fp32 (IVFPQIndex.swift:366-368)."""
    v = _f32(vectors)
    coarse, assign, _ = kmeans_lloyd(ctx, v, coarse_initial, iterations, metric, workers)
    resid = (v - coarse[assign]).astype(np.float32)
    books = pq_train(ctx, resid, codebooks_initial, iterations, workers)
    return coarse, books
