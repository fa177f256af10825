"""IVF-flat search over the C ABI (IVFFlatSearch, Sources/MetalANNSCore/
IVFFlatSearch.swift).

``Partition`` holds the reference's partition layout on the device: centroids,
list-contiguous packed rows (packed[p] = corpus[listIDs[p]]) and listOffsets.
``IVFFlatSearch.search`` probes the nprobe nearest lists and scans them
exactly; results ascend by (distance, id).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import lib
from .core import (MAX_TOP_K, ConstructionFailed, Context, DimensionMismatch, Metric,
                   SearchFailed, SearchResult, Workspace, check)

DEFAULT_LIST_COUNT = 256
DEFAULT_NPROBE = 4


def list_count(vector_count: int) -> int:
    """IVFFlatSearch.listCount(for:) (IVFFlatSearch.swift:19-22)."""
    return min(DEFAULT_LIST_COUNT, max(16, vector_count // 64))


def resolved_list_count(requested: int, vector_count: int) -> int:
    """IVFFlatSearch.resolvedListCount (IVFFlatSearch.swift:24-33): 256 means auto."""
    auto = list_count(vector_count)
    if requested == DEFAULT_LIST_COUNT:
        return min(auto, vector_count)
    return min(max(1, requested), vector_count)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


class Partition:
    """Device-resident IVF-flat partition (IVFFlatSearch.Partition layout)."""

    def __init__(self, context: Context, centroids, packed_rows, list_ids, list_offsets):
        c = _f32(centroids)
        pr = _f32(packed_rows)
        ids = np.ascontiguousarray(list_ids, np.uint32)
        off = np.ascontiguousarray(list_offsets, np.int64)
        if c.ndim != 2 or pr.ndim != 2 or (pr.shape[0] and pr.shape[1] != c.shape[1]):
            raise ConstructionFailed("centroids and packed rows must be 2-D with equal width")
        if off.shape[0] != c.shape[0] + 1 or ids.shape[0] != pr.shape[0]:
            raise ConstructionFailed("list offsets / ids do not match the partition shape")
        h = C.c_void_p()
        check(lib().mans_ivf_create(context.handle, C.c_void_p(c.ctypes.data), c.shape[0],
                                    c.shape[1], C.c_void_p(pr.ctypes.data),
                                    C.c_void_p(ids.ctypes.data), C.c_void_p(off.ctypes.data),
                                    pr.shape[0], C.byref(h)))
        self._h = h
        self.context = context
        self.nlist = c.shape[0]
        self.dim = c.shape[1]
        self.count = pr.shape[0]

    @classmethod
    def from_assignment(cls, context: Context, corpus, centroids, assign):
        """Counting-sort layout of buildPartition (IVFFlatSearch.swift:583-614)."""
        corpus = _f32(corpus)
        nlist = len(centroids)
        assign = np.asarray(assign, np.int64)
        order = np.argsort(assign, kind="stable").astype(np.uint32)
        sizes = np.bincount(assign, minlength=nlist)
        offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
        return cls(context, centroids, corpus[order], order, offsets)

    @classmethod
    def build(cls, context: Context, corpus, centroids, metric: Metric):
        """Partition built on the device from an uploaded corpus (a
        VectorBuffer) and trained centroids: IVFFlatSearch.buildPartition
        after its k-means (IVFFlatSearch.swift:559-631)."""
        c = _f32(centroids)
        if c.ndim != 2 or c.shape[1] != corpus.dim:
            raise DimensionMismatch(f"expected {corpus.dim}-wide centroids")
        self = cls.__new__(cls)
        h = C.c_void_p()
        check(lib().mans_ivf_build(context.handle, corpus.handle, C.c_void_p(c.ctypes.data),
                                   c.shape[0], int(metric), C.byref(h)))
        self._h = h
        self.context = context
        self.nlist = c.shape[0]
        self.dim = c.shape[1]
        self.count = corpus.count
        return self

    def layout(self):
        """(list offsets [nlist + 1] int64, list ids [n] uint32)."""
        off = np.empty(self.nlist + 1, np.int64)
        ids = np.empty(self.count, np.uint32)
        check(lib().mans_ivf_layout(self._h, C.c_void_p(off.ctypes.data),
                                    C.c_void_p(ids.ctypes.data)))
        return off, ids

    @property
    def handle(self):
        return self._h

    def close(self):
        if self._h:
            lib().mans_ivf_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def assign_rows(context: Context, corpus, centroids, metric: Metric) -> np.ndarray:
    """IVFFlatSearch.assignRows on the device (IVFFlatSearch.swift:633-703)."""
    c = _f32(centroids)
    out = np.empty(corpus.count, np.int32)
    check(lib().mans_ivf_assign(context.handle, corpus.handle, C.c_void_p(c.ctypes.data),
                                c.shape[0], int(metric), C.c_void_p(out.ctypes.data)))
    return out


class IVFFlatSearch:
    minVectorCount = 256
    defaultListCount = DEFAULT_LIST_COUNT
    defaultNProbe = DEFAULT_NPROBE

    @staticmethod
    def search_arrays(context: Context, queries, partition: Partition, k: int, nprobe: int,
                      metric: Metric):
        q = _f32(np.atleast_2d(queries))
        nq, dim = q.shape
        kout = max(0, min(k, MAX_TOP_K))
        od = np.empty((nq, kout), np.float32)
        oi = np.empty((nq, kout), np.uint32)
        oc = np.empty(nq, np.int32)
        check(lib().mans_ivf_search(context.handle, partition.handle, C.c_void_p(q.ctypes.data),
                                    nq, dim, k, nprobe, int(metric), C.c_void_p(od.ctypes.data),
                                    C.c_void_p(oi.ctypes.data), C.c_void_p(oc.ctypes.data)))
        return od, oi, oc

    @staticmethod
    def search(context: Context, query, partition: Partition, k: int, nprobe: int,
               metric: Metric):
        """IVFFlatSearch.search(query:partition:k:nprobe:metric:) (:115-133)."""
        if k <= 0 or partition.count == 0:
            return []
        if len(query) != partition.dim:
            raise DimensionMismatch(f"expected {partition.dim}, got {len(query)}")
        if metric == Metric.hamming:
            raise SearchFailed("IVF-flat does not support metric .hamming")
        od, oi, oc = IVFFlatSearch.search_arrays(context, [query], partition, k, nprobe, metric)
        return [SearchResult("", float(od[0, i]), int(oi[0, i])) for i in range(oc[0])]

    @staticmethod
    def search_device(context: Context, partition: Partition, ws: Workspace, d_queries: int,
                      nq: int, k: int, nprobe: int, metric: Metric, d_out_dist: int,
                      d_out_ids: int, d_out_counts: int, stream: int = 0) -> None:
        check(lib().mans_ivf_search_device(context.handle, partition.handle, ws.handle,
                                           C.c_void_p(d_queries), nq, k, nprobe, int(metric),
                                           C.c_void_p(d_out_dist), C.c_void_p(d_out_ids),
                                           C.c_void_p(d_out_counts), C.c_void_p(stream)))
